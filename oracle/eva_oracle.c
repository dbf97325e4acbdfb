/* CPU oracle of the EVA02-L tagger forward — TEST INFRASTRUCTURE ONLY (see eva_oracle.h).
 *
 * Restates, in plain C with OpenMP, what the reference computes on the GPU (HoloArchivists/xTagger,
 * src/engine/eva_kernels.cu and src/engine/kern_common.cuh, launch order src/engine/eva.h:226-310), at the same
 * quantisation points, with straightforward loops and double accumulation where the reference uses fp32. The
 * block-scaled weight format (v4) generalises the reference's per-tensor scale (src/tools/export_eva.py:64-66) to
 * one fp32 scale per 128 x 128 block; a v3 file is the special case where every block has the same scale.
 */
#include "eva_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define RESCALE 8.0f /* kern_common.cuh:14 */
#define PSKIP 10.0f  /* kern_common.cuh:15 */
#define EPS 1e-6f    /* kern_common.cuh:16 */

int or_threads(void) { return omp_get_max_threads(); }
/* threads of the oracle's parallel regions from now on (whatever OMP_NUM_THREADS said; torch.distributed.run sets
 * it to 1); returns the new count */
int or_set_threads(int n)
{
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}

/* ---------------------------------------------------------------------------------------------------------------
 * E4M3 (OCP FP8, 1-4-3, bias 7, no infinities, 0x7F / 0xFF NaN, max finite 448). The reference converts with
 * __nv_cvt_float2_to_fp8x2(..., __NV_SATFINITE, __NV_E4M3) (kern_common.cuh:97-100): round to nearest even,
 * finite values beyond 448 saturate, NaN stays NaN. Decode: kcheck.c:237-245 / prune24.py:11-15.
 * ------------------------------------------------------------------------------------------------------------- */
uint8_t or_e4m3(float x)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    const uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return sign | 0x7F;              /* NaN */
    if (a >= 0x43E00000u) return sign | 0x7E;             /* >= 448 (and inf): saturate */
    float f;
    memcpy(&f, &a, 4);
    if (f < 0.015625f) {                                  /* below 2^-6: subnormal grid of 2^-9 */
        const float q = rintf(f * 512.0f);                /* exact scaling, round to nearest even */
        return sign | (uint8_t)q;                         /* q == 8 is the smallest normal, code 0x08 */
    }
    int e = (int)(a >> 23) - 127 + 7;                     /* 1..15 */
    uint32_t m = a & 0x7FFFFFu;
    uint32_t keep = m >> 20, rem = m & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (keep & 1))) keep++;
    if (keep == 8) {
        keep = 0;
        e++;
    }
    if (e > 15 || (e == 15 && keep == 7)) return sign | 0x7E;
    return sign | (uint8_t)((e << 3) | keep);
}

float or_e4m3_dec(uint8_t b)
{
    const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    if ((b & 0x7F) == 0x7F) return NAN;
    const float v = e ? ldexpf(1.0f + m / 8.0f, e - 7) : ldexpf(m / 8.0f, -6);
    return s ? -v : v;
}

void or_e4m3_n(const float *x, uint8_t *y, size_t n)
{
#pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; i++) y[i] = or_e4m3(x[i]);
}

void or_e4m3_dec_n(const uint8_t *x, float *y, size_t n)
{
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = or_e4m3_dec((uint8_t)i);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; i++) y[i] = lut[x[i]];
}

uint16_t or_f2h(float x)
{
    _Float16 h = (_Float16)x;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

float or_h2f(uint16_t u)
{
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

void or_f2h_n(const float *x, uint16_t *y, size_t n)
{
#pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; i++) y[i] = or_f2h(x[i]);
}

void or_h2f_n(const uint16_t *x, float *y, size_t n)
{
#pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; i++) y[i] = or_h2f(x[i]);
}

static float h16r(float x) { return or_h2f(or_f2h(x)); } /* round through fp16 */

/* ---------------------------------------------------------------------------------------------------------------
 * GEMMs. Dequantise-then-matmul: each 128-wide K block is an exact-product fp32 dot (E4M3 x E4M3 products are
 * exact in fp32), blocks are combined in double with their scales. Same result as the reference's
 * gemm8 (kern_common.cuh:305-356) up to summation order.
 * ------------------------------------------------------------------------------------------------------------- */
static float dotf(const float *a, const float *b, int n)
{
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int e = 0; e < 8; e++) s[e] += a[i + e] * b[i + e];
    float t = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
    for (; i < n; i++) t += a[i] * b[i];
    return t;
}

/* out[i][j] = ascale * sum_kb ws[j/128][kb] * dot_kb(A[i], W[j]); ws NULL = all ones */
static void gemm_f(const float *A, int m, int k, const float *W, int n, const float *ws, float ascale, float *out)
{
    const int nkb = (k + 127) / 128;
    const int RB = 16;
#pragma omp parallel for schedule(dynamic)
    for (int ib = 0; ib < m; ib += RB) {
        const int ie = ib + RB < m ? ib + RB : m;
        for (int j = 0; j < n; j++) {
            const float *wr = W + (size_t)j * k;
            const float *sr = ws ? ws + (size_t)(j / 128) * nkb : NULL;
            for (int i = ib; i < ie; i++) {
                const float *ar = A + (size_t)i * k;
                double acc = 0.0;
                for (int b = 0; b < nkb; b++) {
                    const int k0 = b * 128, kl = k - k0 < 128 ? k - k0 : 128;
                    const float s = dotf(ar + k0, wr + k0, kl);
                    acc += (sr ? (double)sr[b] : 1.0) * (double)s;
                }
                out[(size_t)i * n + j] = (float)(ascale * acc);
            }
        }
    }
}

void or_gemm_e4m3(const uint8_t *a, int m, int k, const uint8_t *w, int n, const float *ws, float ascale, float *out)
{
    float *A = malloc((size_t)m * k * 4), *W = malloc((size_t)n * k * 4);
    or_e4m3_dec_n(a, A, (size_t)m * k);
    or_e4m3_dec_n(w, W, (size_t)n * k);
    gemm_f(A, m, k, W, n, ws, ascale, out);
    free(A);
    free(W);
}

void or_gemm_f16(const uint16_t *a, int m, int k, const uint16_t *w, int n, float *out)
{
    float *A = malloc((size_t)m * k * 4), *W = malloc((size_t)n * k * 4);
    or_h2f_n(a, A, (size_t)m * k);
    or_h2f_n(w, W, (size_t)n * k);
    gemm_f(A, m, k, W, n, NULL, 1.0f, out);
    free(A);
    free(W);
}

/* ---------------------------------------------------------------------------------------------------------------
 * LayerNorm + activation quantisation: ln_row<1> (kern_common.cuh:147-186): two-pass mean / variance over 1024,
 * eps 1e-6, (x - mean) * rstd * g + b, * qs, E4M3.
 * ------------------------------------------------------------------------------------------------------------- */
void or_ln_e4m3(const uint16_t *x, const float *g, const float *b, int rows, float qs, uint8_t *y)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float v[OR_D];
        double s = 0, q = 0;
        for (int i = 0; i < OR_D; i++) {
            v[i] = or_h2f(x[(size_t)r * OR_D + i]);
            s += v[i];
        }
        const float mean = (float)(s / OR_D);
        for (int i = 0; i < OR_D; i++) q += (double)(v[i] - mean) * (v[i] - mean);
        const float rstd = 1.0f / sqrtf((float)(q / OR_D) + EPS);
        for (int i = 0; i < OR_D; i++) y[(size_t)r * OR_D + i] = or_e4m3(((v[i] - mean) * rstd * g[i] + b[i]) * qs);
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * QKV epilogue (k_qkv, eva_kernels.cu:60-113): acc is the dequantised projection [rows][3072] (q | k | v).
 * q, k: * cq / ck, then for patch tokens (t >= 1) rotate pair (2j, 2j+1) of each head by angle j of
 * cs[t - 1][j] = (cos, sin); E4M3. v: * cv, E4M3. Layouts of this library's attention (the reference permutes head
 * dims and transposes V for its mma.sync fragments instead): q8 / k8 / v8 [img][16][TP][64]; pads untouched.
 * ------------------------------------------------------------------------------------------------------------- */
void or_qkv_epilogue(const float *acc, int rows, const float *cs, float cq, float ck, float cv, uint8_t *q8,
                     uint8_t *k8, uint8_t *v8)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const int b = r / OR_T, t = r % OR_T;
        const float *a = acc + (size_t)r * 3 * OR_D;
        for (int p = 0; p < 2; p++) {
            const float sc = p ? ck : cq;
            uint8_t *dst = p ? k8 : q8;
            for (int h = 0; h < OR_NH; h++)
                for (int j = 0; j < 32; j++) {
                    float f0 = a[p * OR_D + h * 64 + 2 * j] * sc, f1 = a[p * OR_D + h * 64 + 2 * j + 1] * sc;
                    if (t) {
                        const float c = cs[((size_t)(t - 1) * 32 + j) * 2], s = cs[((size_t)(t - 1) * 32 + j) * 2 + 1];
                        const float g0 = f0 * c - f1 * s;
                        f1 = f1 * c + f0 * s;
                        f0 = g0;
                    }
                    uint8_t *o = dst + (((size_t)b * OR_NH + h) * OR_TP + t) * 64;
                    o[2 * j] = or_e4m3(f0);
                    o[2 * j + 1] = or_e4m3(f1);
                }
        }
        for (int h = 0; h < OR_NH; h++)
            for (int d = 0; d < 64; d++)
                v8[(((size_t)b * OR_NH + h) * OR_TP + t) * 64 + d] = or_e4m3(a[2 * OR_D + h * 64 + d] * cv);
    }
}

/* ---------------------------------------------------------------------------------------------------------------
 * Attention (flash8, kern_common.cuh:403-543). Query rows go in slices of slice_rows consecutive rows (the reference:
 * 16, one warp's rows, kern_common.cuh:433-434 and 470-481; slices start at multiples of slice_rows and run past
 * token 1024 into the zero query rows of the padding, which take part in the decisions as in the reference), keys
 * in tiles of key_tile (the reference: 64):
 *   m = -1e30, l = 0, O = 0 per row; per tile: tm = max of the row's scores over the tile's keys (< 1025)
 *   lazy rescale (kern_common.cuh:484-493): if some row of the slice has max(m, tm) > m + RESCALE / sinv, every
 *     row of the slice takes mn = max(m, tm): sc = exp2((m - mn) sinv); l *= sc; O *= sc; m = mn
 *   dead tile (kern_common.cuh:496-499): if every row of the slice has tm < m - PSKIP / sinv, the tile adds nothing
 *   else, every row: p = exp2(s sinv - m sinv) (one fma); l += p; O += E4M3(p) * V
 *   out = E4M3(fp16(O * (vo / l))) (the reference stages the output as fp16, kern_common.cuh:527-541).
 * ------------------------------------------------------------------------------------------------------------- */
void or_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg, float sinv, float vo,
                  int key_tile, int slice_rows, uint8_t *out)
{
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = or_e4m3_dec((uint8_t)i);
    const float thr = RESCALE / sinv, dthr = PSKIP / sinv;
    const int SR = slice_rows, nslices = (OR_T + SR - 1) / SR;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < nimg; b++)
        for (int h = 0; h < OR_NH; h++) {
            const size_t bh = (size_t)b * OR_NH + h;
            float *K = malloc((size_t)OR_T * 64 * 4), *V = malloc((size_t)OR_T * 64 * 4);
            float *S = malloc((size_t)SR * OR_T * 4), *o = malloc((size_t)SR * 64 * 4);
            float *m = malloc(SR * 4), *l = malloc(SR * 4), *tm = malloc(SR * 4);
            for (int t = 0; t < OR_T; t++)
                for (int d = 0; d < 64; d++) {
                    K[t * 64 + d] = lut[k8[(bh * OR_TP + t) * 64 + d]];
                    V[t * 64 + d] = lut[v8[(bh * OR_TP + t) * 64 + d]];
                }
            for (int g = 0; g < nslices; g++) {
                for (int i = 0; i < SR; i++) {   /* rows past 1024 read the zero padding of q8 (1152 rows) */
                    float q[64];
                    for (int d = 0; d < 64; d++) q[d] = lut[q8[(bh * OR_TP + g * SR + i) * 64 + d]];
                    for (int t = 0; t < OR_T; t++) S[i * OR_T + t] = dotf(q, K + t * 64, 64);
                    for (int d = 0; d < 64; d++) o[i * 64 + d] = 0.f;
                    m[i] = -1e30f;
                    l[i] = 0.f;
                }
                for (int t0 = 0; t0 < OR_T; t0 += key_tile) {
                    const int t1 = t0 + key_tile < OR_T ? t0 + key_tile : OR_T;
                    int resc = 0, dead = 1;
                    for (int i = 0; i < SR; i++) {
                        tm[i] = -INFINITY;
                        for (int t = t0; t < t1; t++) tm[i] = fmaxf(tm[i], S[i * OR_T + t]);
                        if (fmaxf(m[i], tm[i]) > m[i] + thr) resc = 1;
                    }
                    if (resc)
                        for (int i = 0; i < SR; i++) {
                            const float mn = fmaxf(m[i], tm[i]), sc = exp2f((m[i] - mn) * sinv);
                            l[i] *= sc;
                            for (int d = 0; d < 64; d++) o[i * 64 + d] *= sc;
                            m[i] = mn;
                        }
                    for (int i = 0; i < SR; i++)
                        if (!(tm[i] < m[i] - dthr)) dead = 0;
                    if (dead) continue;
                    for (int i = 0; i < SR; i++)
                        for (int t = t0; t < t1; t++) {
                            const float p = exp2f(fmaf(S[i * OR_T + t], sinv, -m[i] * sinv));
                            l[i] += p;
                            const float pq = lut[or_e4m3(p)];
                            if (pq != 0.f)
                                for (int d = 0; d < 64; d++) o[i * 64 + d] += pq * V[t * 64 + d];
                        }
                }
                for (int i = 0; i < SR; i++) {
                    const int qi = g * SR + i;
                    if (qi >= OR_T) break;
                    const float f = vo / l[i];
                    uint8_t *dst = out + ((size_t)b * OR_T + qi) * OR_D + h * 64;
                    for (int d = 0; d < 64; d++) dst[d] = or_e4m3(h16r(o[i * 64 + d] * f));
                }
            }
            free(K);
            free(V);
            free(S);
            free(o);
            free(m);
            free(l);
            free(tm);
        }
}

/* residual update, fp16 stream (k_oproj, eva_kernels.cu:148-161): x = fp16(x + acc) */
void or_resid_add(uint16_t *x, const float *acc, int rows)
{
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < (size_t)rows * OR_D; i++) x[i] = or_f2h(or_h2f(x[i]) + acc[i]);
}

/* ---------------------------------------------------------------------------------------------------------------
 * fc1 epilogue (k_fc1, eva_kernels.cu:233-278): acc [rows][5472] dequantised, rows of W12 interleave g / x in
 * 16-unit chunks (export_eva.py:60-62): column 32c + i is g of unit 16c + i, column 32c + 16 + i is x.
 * u = x * 0.5 g (1 + tanh(g / 2)); h8 = E4M3(u * rs[unit]); row statistics sum u, sum u^2 (double here).
 * ------------------------------------------------------------------------------------------------------------- */
void or_fc1_epilogue(const float *acc, int rows, const float *rs, uint8_t *h8, double *rowsum, double *rowsq)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        double s = 0, q = 0;
        for (int c = 0; c < OR_HIDP / 16; c++)
            for (int i = 0; i < 16; i++) {
                const float g = acc[(size_t)r * OR_N12 + 32 * c + i], xv = acc[(size_t)r * OR_N12 + 32 * c + 16 + i];
                const float u = xv * (0.5f * g * (1.0f + tanhf(0.5f * g)));
                s += u;
                q += (double)u * u;
                h8[(size_t)r * OR_HIDP + 16 * c + i] = or_e4m3(u * rs[16 * c + i]);
            }
        rowsum[r] = s;
        rowsq[r] = q;
    }
}

/* fc2 epilogue with the MLP LayerNorm folded in (k_fc2, eva_kernels.cu:301-333):
 * mean = sum / 2730, rstd = 1 / sqrt(sumsq / 2730 - mean^2 + eps); x = fp16(x + rstd (acc - mean c) + d) */
void or_fc2_epilogue(uint16_t *x, const float *acc, int rows, const double *rowsum, const double *rowsq,
                     const float *c, const float *d)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const float mean = (float)(rowsum[r] / OR_HID);
        const float rstd = 1.0f / sqrtf((float)(rowsq[r] / OR_HID) - mean * mean + EPS);
        for (int n = 0; n < OR_D; n++) {
            const size_t i = (size_t)r * OR_D + n;
            x[i] = or_f2h(or_h2f(x[i]) + rstd * acc[i] - mean * rstd * c[n] + d[n]);
        }
    }
}

/* patch embedding + position (k_pe + k_embed, eva_kernels.cu:21-33, 126-130; kern_common.cuh:362-386):
 * x[img][1 + p] = fp16(fp16(in[img][p] . pe^T) + pos[1 + p]); x[img][0] = fp16(pos[0]) (cls folded into pos[0]) */
void or_patch_embed(const uint16_t *in, int nimg, const uint16_t *pe, const float *pos, uint16_t *x)
{
    float *acc = malloc((size_t)nimg * OR_NP * OR_D * 4);
    or_gemm_f16(in, nimg * OR_NP, OR_K0P, pe, OR_D, acc);
#pragma omp parallel for schedule(static)
    for (int b = 0; b < nimg; b++) {
        for (int n = 0; n < OR_D; n++) x[(size_t)b * OR_T * OR_D + n] = or_f2h(pos[n]);
        for (int p = 0; p < OR_NP; p++)
            for (int n = 0; n < OR_D; n++)
                x[((size_t)b * OR_T + 1 + p) * OR_D + n] =
                    or_f2h(h16r(acc[((size_t)b * OR_NP + p) * OR_D + n]) + pos[(size_t)(1 + p) * OR_D + n]);
    }
    free(acc);
}

/* mean pool over patch tokens (k_pool, eva_kernels.cu:404-431) + fc_norm (k_lnh, kern_common.cuh:188-192)
 * -> pn fp16; pn8 = E4M3(pn * qs) for an FP8 head (this library's addition) */
void or_pool_ln(const uint16_t *x, int nimg, const float *g, const float *b, float *pool, uint16_t *pn, uint8_t *pn8,
                float qs)
{
    for (int im = 0; im < nimg; im++) {
        float *pl = pool + (size_t)im * OR_D;
        for (int n = 0; n < OR_D; n++) {
            double s = 0;
            for (int t = 1; t < OR_T; t++) s += or_h2f(x[((size_t)im * OR_T + t) * OR_D + n]);
            pl[n] = (float)(s / (OR_T - 1));
        }
        double s = 0, q = 0;
        for (int n = 0; n < OR_D; n++) s += pl[n];
        const float mean = (float)(s / OR_D);
        for (int n = 0; n < OR_D; n++) q += (double)(pl[n] - mean) * (pl[n] - mean);
        const float rstd = 1.0f / sqrtf((float)(q / OR_D) + EPS);
        for (int n = 0; n < OR_D; n++) {
            const uint16_t h = or_f2h((pl[n] - mean) * rstd * g[n] + b[n]);
            pn[(size_t)im * OR_D + n] = h;
            if (pn8) pn8[(size_t)im * OR_D + n] = or_e4m3(or_h2f(h) * qs);
        }
    }
}

/* tag head (k_headmv, kern_common.cuh:695-727): out = sigmoid(pn . hw^T + hb) */
void or_head_f16(const uint16_t *pn, int nimg, const uint16_t *hw, const float *hb, int nt, float *out)
{
    float *lg = malloc((size_t)nimg * nt * 4);
    or_gemm_f16(pn, nimg, OR_D, hw, nt, lg);
    for (int b = 0; b < nimg; b++)
        for (int j = 0; j < nt; j++) out[(size_t)b * nt + j] = 1.0f / (1.0f + expf(-(lg[(size_t)b * nt + j] + hb[j])));
    free(lg);
}

/* FP8 block-scaled head (this library's addition): logits = ascale * sum_kb hws[tag/128][kb] * dot_kb */
void or_head_e4m3(const uint8_t *pn8, int nimg, const uint8_t *hw8, const float *hws, float ascale, const float *hb,
                  int nt, float *out)
{
    float *lg = malloc((size_t)nt * nimg * 4);
    float *A = malloc((size_t)nt * OR_D * 4), *B = malloc((size_t)nimg * OR_D * 4);
    or_e4m3_dec_n(hw8, A, (size_t)nt * OR_D);
    or_e4m3_dec_n(pn8, B, (size_t)nimg * OR_D);
    /* weights as the row operand: scale row = tag block */
    for (int j = 0; j < nt; j++)
        for (int b = 0; b < nimg; b++) {
            double acc = 0;
            for (int kb = 0; kb < OR_D / 128; kb++)
                acc += (double)hws[(size_t)(j / 128) * (OR_D / 128) + kb] *
                       dotf(A + (size_t)j * OR_D + kb * 128, B + (size_t)b * OR_D + kb * 128, 128);
            lg[(size_t)j * nimg + b] = (float)(ascale * acc);
        }
    for (int b = 0; b < nimg; b++)
        for (int j = 0; j < nt; j++) out[(size_t)b * nt + j] = 1.0f / (1.0f + expf(-(lg[(size_t)j * nimg + b] + hb[j])));
    free(lg);
    free(A);
    free(B);
}

/* ---------------------------------------------------------------------------------------------------------------
 * Model file reader. Layout (eva.h:378-430, writer export_eva.py:119-153): 16-byte header "EVA2", version, nt,
 * blob bytes, zero pad to 256, then 256-byte-aligned tensors. v4 (block-scaled, this library) adds nl (header
 * word 4) and head flags (word 5), and follows every E4M3 matrix with its fp32 block scales; v3's per-tensor scale
 * expands to uniform blocks.
 * ------------------------------------------------------------------------------------------------------------- */
typedef struct {
    float *ln1w, *ln1b, *ln2w, *ln2b, *rs, *c, *d;
    uint8_t *wqkv, *wo, *w12, *w2;
    float *sqkv, *so, *s12, *s2; /* block scales (v3: expanded) */
    float adq[4], cq, ck, cv, sinv, vo;
} or_layer;

typedef struct {
    uint8_t *blob;
    int ver, nt, ntp, nl, head8;
    float *table, *pos, *cs, *fnw, *fnb, *hb, *hws, head_adq;
    uint16_t *pe, *hw16;
    uint8_t *hw8;
    or_layer *L;
} or_model;

static size_t take(size_t *off, size_t bytes)
{
    const size_t o = (*off + 255) & ~(size_t)255;
    *off = o + bytes;
    return o;
}

static float *expand_scale(float s, int n, int k)
{
    const int nb = (n + 127) / 128, kb = (k + 127) / 128;
    float *p = malloc((size_t)nb * kb * 4);
    for (int i = 0; i < nb * kb; i++) p[i] = s;
    return p;
}

static int model_load(const char *path, or_model *M)
{
    memset(M, 0, sizeof(*M));
    FILE *f = fopen(path, "rb");
    uint32_t hdr[6];
    if (!f || fread(hdr, 4, 6, f) != 6 || memcmp(hdr, "EVA2", 4) || (hdr[1] != 3 && hdr[1] != 4)) {
        fprintf(stderr, "oracle: %s is not an eva02.bin v3/v4\n", path);
        if (f) fclose(f);
        return -1;
    }
    M->ver = (int)hdr[1];
    M->nt = (int)hdr[2];
    M->ntp = (M->nt + 7) & ~7;
    const size_t bytes = hdr[3];
    M->nl = M->ver == 4 && hdr[4] ? (int)hdr[4] : 24;
    M->head8 = M->ver == 4 && (hdr[5] & 1);
    M->blob = malloc(bytes);
    if (fseek(f, 256, SEEK_SET) || fread(M->blob, 1, bytes, f) != bytes) {
        fprintf(stderr, "oracle: short read of %s\n", path);
        fclose(f);
        return -1;
    }
    fclose(f);
    uint8_t *B = M->blob;
    size_t off = 0;
    const int v4 = M->ver == 4;
    M->table = (float *)(B + take(&off, (size_t)M->nl * 12 * 4));
    M->pe = (uint16_t *)(B + take(&off, (size_t)OR_D * OR_K0P * 2));
    M->pos = (float *)(B + take(&off, (size_t)OR_T * OR_D * 4));
    M->cs = (float *)(B + take(&off, (size_t)OR_NP * 32 * 2 * 4));
    M->L = calloc(M->nl, sizeof(or_layer));
    for (int i = 0; i < M->nl; i++) {
        or_layer *L = &M->L[i];
        const float *tb = M->table + i * 12;
        L->ln1w = (float *)(B + take(&off, OR_D * 4));
        L->ln1b = (float *)(B + take(&off, OR_D * 4));
        L->wqkv = B + take(&off, (size_t)3 * OR_D * OR_D);
        if (v4) L->sqkv = (float *)(B + take(&off, (size_t)24 * 8 * 4));
        L->wo = B + take(&off, (size_t)OR_D * OR_D);
        if (v4) L->so = (float *)(B + take(&off, (size_t)8 * 8 * 4));
        L->ln2w = (float *)(B + take(&off, OR_D * 4));
        L->ln2b = (float *)(B + take(&off, OR_D * 4));
        L->w12 = B + take(&off, (size_t)OR_N12 * OR_D);
        if (v4) L->s12 = (float *)(B + take(&off, (size_t)43 * 8 * 4));
        L->rs = (float *)(B + take(&off, OR_HIDP * 4));
        L->w2 = B + take(&off, (size_t)OR_D * OR_HIDP);
        if (v4) L->s2 = (float *)(B + take(&off, (size_t)8 * 22 * 4));
        L->c = (float *)(B + take(&off, OR_D * 4));
        L->d = (float *)(B + take(&off, OR_D * 4));
        if (!v4) {
            L->sqkv = expand_scale(tb[0], 3 * OR_D, OR_D);
            L->so = expand_scale(tb[1], OR_D, OR_D);
            L->s12 = expand_scale(tb[2], OR_N12, OR_D);
            L->s2 = expand_scale(tb[3], OR_D, OR_HIDP);
        }
        for (int g = 0; g < 4; g++) L->adq[g] = tb[4 + g];
        /* eva.h:408-418 */
        L->cq = 1.0f / tb[8];
        L->ck = 1.0f / tb[9];
        L->cv = 1.0f / tb[10];
        L->sinv = tb[8] * tb[9];
        L->vo = (1.0f / tb[5]) * tb[10];
    }
    M->fnw = (float *)(B + take(&off, OR_D * 4));
    M->fnb = (float *)(B + take(&off, OR_D * 4));
    if (M->head8) {
        const float *hs = (const float *)(B + take(&off, 16));
        M->head_adq = hs[0];
        M->hw8 = B + take(&off, (size_t)M->ntp * OR_D);
        M->hws = (float *)(B + take(&off, (size_t)((M->ntp + 127) / 128) * 8 * 4));
    } else {
        M->hw16 = (uint16_t *)(B + take(&off, (size_t)M->ntp * OR_D * 2));
    }
    M->hb = (float *)(B + take(&off, (size_t)M->ntp * 4));
    if (off != bytes) {
        fprintf(stderr, "oracle: weight layout mismatch (%zu vs %zu bytes)\n", off, bytes);
        return -1;
    }
    return 0;
}

static void model_free(or_model *M)
{
    if (M->ver == 3 && M->L)
        for (int i = 0; i < M->nl; i++) {
            free(M->L[i].sqkv);
            free(M->L[i].so);
            free(M->L[i].s12);
            free(M->L[i].s2);
        }
    free(M->L);
    free(M->blob);
}

int or_model_nt(const char *model)
{
    FILE *f = fopen(model, "rb");
    uint32_t hdr[4];
    int nt = -1;
    if (f && fread(hdr, 4, 4, f) == 4 && !memcmp(hdr, "EVA2", 4)) nt = (int)hdr[2];
    if (f) fclose(f);
    return nt;
}

/* The forward of eva_forward (eva.h:252-307) for nimg inputs. */
int or_forward(const char *model, const uint16_t *in, int nimg, int key_tile, int slice_rows, float *scores,
               uint16_t *pn_out)
{
    or_model M;
    if (model_load(model, &M)) return -1;
    const int rows = nimg * OR_T;
    uint16_t *x = malloc((size_t)rows * OR_D * 2);
    uint8_t *h = malloc((size_t)rows * OR_D);
    float *acc = malloc((size_t)rows * OR_N12 * 4);
    uint8_t *q8 = calloc((size_t)nimg * OR_NH * OR_TP * 64, 1), *k8 = calloc((size_t)nimg * OR_NH * OR_TP * 64, 1);
    uint8_t *v8 = calloc((size_t)nimg * OR_NH * OR_TP * 64, 1);
    uint8_t *h8 = malloc((size_t)rows * OR_HIDP);
    double *rsum = malloc((size_t)rows * 8), *rsq = malloc((size_t)rows * 8);
    or_patch_embed(in, nimg, M.pe, M.pos, x);
    for (int i = 0; i < M.nl; i++) {
        or_layer *L = &M.L[i];
        or_ln_e4m3(x, L->ln1w, L->ln1b, rows, 1.0f / L->adq[0], h);
        or_gemm_e4m3(h, rows, OR_D, L->wqkv, 3 * OR_D, L->sqkv, L->adq[0], acc);
        or_qkv_epilogue(acc, rows, M.cs, L->cq, L->ck, L->cv, q8, k8, v8);
        or_attention(q8, k8, v8, nimg, L->sinv, L->vo, key_tile, slice_rows, h);
        or_gemm_e4m3(h, rows, OR_D, L->wo, OR_D, L->so, L->adq[1], acc);
        or_resid_add(x, acc, rows);
        or_ln_e4m3(x, L->ln2w, L->ln2b, rows, 1.0f / L->adq[2], h);
        or_gemm_e4m3(h, rows, OR_D, L->w12, OR_N12, L->s12, L->adq[2], acc);
        or_fc1_epilogue(acc, rows, L->rs, h8, rsum, rsq);
        or_gemm_e4m3(h8, rows, OR_HIDP, L->w2, OR_D, L->s2, L->adq[3], acc);
        or_fc2_epilogue(x, acc, rows, rsum, rsq, L->c, L->d);
    }
    float *pool = malloc((size_t)nimg * OR_D * 4);
    uint16_t *pn = malloc((size_t)nimg * OR_D * 2);
    uint8_t *pn8 = M.head8 ? malloc((size_t)nimg * OR_D) : NULL;
    or_pool_ln(x, nimg, M.fnw, M.fnb, pool, pn, pn8, M.head8 ? 1.0f / M.head_adq : 1.0f);
    if (M.head8) or_head_e4m3(pn8, nimg, M.hw8, M.hws, M.head_adq, M.hb, M.nt, scores);
    else or_head_f16(pn, nimg, M.hw16, M.hb, M.nt, scores);
    if (pn_out) memcpy(pn_out, pn, (size_t)nimg * OR_D * 2);
    free(pool);
    free(pn);
    free(pn8);
    free(x);
    free(h);
    free(acc);
    free(q8);
    free(k8);
    free(v8);
    free(h8);
    free(rsum);
    free(rsq);
    model_free(&M);
    return 0;
}

/* ---------------------------------------------------------------------------------------------------------------
 * 2:4 selection (prune24.py:44-56): per row, per group of 4 consecutive k, score = |E4M3^-1(w)| (magnitude) or
 * |w| * colmax|w| (Wanda); the 2 lowest are zeroed. np.argsort of 4 scores is a stable sort, so on ties the lower
 * index counts as lower and is dropped first.
 * ------------------------------------------------------------------------------------------------------------- */
void or_prune24(uint8_t *w, int n, int k, int wanda)
{
    float *cm = calloc((size_t)k, 4);
    if (wanda)
        for (int i = 0; i < n; i++)
            for (int j = 0; j < k; j++) {
                const float v = fabsf((w[(size_t)i * k + j] & 0x7F) == 0x7F ? 0.f : or_e4m3_dec(w[(size_t)i * k + j]));
                if (v > cm[j]) cm[j] = v;
            }
    for (int i = 0; i < n; i++)
        for (int j0 = 0; j0 + 4 <= k; j0 += 4) {
            float s[4];
            int idx[4] = {0, 1, 2, 3};
            for (int e = 0; e < 4; e++) {
                const uint8_t b = w[(size_t)i * k + j0 + e];
                const float v = fabsf((b & 0x7F) == 0x7F ? 0.f : or_e4m3_dec(b));
                s[e] = wanda ? v * cm[j0 + e] : v;
            }
            /* stable insertion sort by score */
            for (int a = 1; a < 4; a++)
                for (int c = a; c > 0 && s[idx[c]] < s[idx[c - 1]]; c--) {
                    const int t = idx[c];
                    idx[c] = idx[c - 1];
                    idx[c - 1] = t;
                }
            w[(size_t)i * k + j0 + idx[0]] = 0;
            w[(size_t)i * k + j0 + idx[1]] = 0;
        }
    free(cm);
}

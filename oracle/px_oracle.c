/* CPU oracle of the PixAI tagger forward (ViTDet-L, 1008^2) — TEST INFRASTRUCTURE ONLY (see eva_oracle.h).
 *
 * Restates, in plain C with OpenMP, the reference's FP8 PixAI engine (HoloArchivists/xTagger, src/engine/px.h:115-
 * 190 for the launch order, src/engine/px_kernels.cu for the kernels, kern_common.cuh for the shared LayerNorm,
 * flash attention and tag head) at the same quantisation points, with double accumulation where the reference uses
 * fp32. Tokens are window-major throughout; attention runs over sequences of L tokens (576 per window, 5184 for the
 * global blocks). Activation and q / k / v layouts are this library's: q8 / k8 / v8 [sequence][16][L][64] (the
 * reference permutes head dims and transposes V for its mma.sync fragments; values are the same).
 */
#include "eva_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define PX_T 5184
#define PX_LW 576
#define PX_HID 4736
#define PX_QKV 3072
#define RESCALE 8.0f  /* kern_common.cuh:14 */
#define PSKIP 10.0f   /* kern_common.cuh:15 */
#define EPS_LN 1e-6f  /* k_ln, kern_common.cuh:16 */
#define EPS_PX 1e-5f  /* k_pembed / k_phln, px_kernels.cu:44, 376 */
#define PCH 144       /* attention-pool token chunk, px_kernels.cu:446 */

static float h16(float x) { return or_h2f(or_f2h(x)); }

/* Row LayerNorm statistics over 1024 values (double sums): mean, 1 / sqrt(var + eps). */
static void ln_stats(const float *v, float eps, float *mean, float *rstd)
{
    double s = 0, q = 0;
    for (int i = 0; i < OR_D; i++) s += v[i];
    const float m = (float)(s / OR_D);
    for (int i = 0; i < OR_D; i++) q += (double)(v[i] - m) * (v[i] - m);
    *mean = m;
    *rstd = 1.0f / sqrtf((float)(q / OR_D) + eps);
}

/* k_ppe + k_pembed (px_kernels.cu:16-52, 131-136): x = fp16(acc) of the patch GEMM; then
 * x = fp16(LN_pre(x + pos[t]) * w + b), eps 1e-5, t = row % 5184 (window-major). */
void or_px_embed(const uint16_t *in, int rows, const uint16_t *pe, const float *pos, const float *w, const float *b,
                 uint16_t *x)
{
    float *acc = malloc((size_t)rows * OR_D * 4);
    or_gemm_f16(in, rows, OR_K0P, pe, OR_D, acc);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float v[OR_D], mean, rstd;
        const float *p = pos + (size_t)(r % PX_T) * OR_D;
        for (int i = 0; i < OR_D; i++) v[i] = h16(acc[(size_t)r * OR_D + i]) + p[i];
        ln_stats(v, EPS_PX, &mean, &rstd);
        for (int i = 0; i < OR_D; i++) x[(size_t)r * OR_D + i] = or_f2h((v[i] - mean) * rstd * w[i] + b[i]);
    }
    free(acc);
}

/* QKV epilogue (k_pqkv, px_kernels.cu:60-129): acc = alpha X Wqkv^T [rows][3072]; f = (acc + bias) * cq / ck / cv;
 * q, k: interleaved RoPE on every token, pair (2j, 2j + 1) of a head by angle j of cs[t][j], t = row % L; E4M3.
 * Row r -> sequence s = r / L, token t: q8 / k8 / v8 [s][16][L][64]. */
void or_px_qkv_epilogue(const float *acc, int rows, int L, const float *bias, const float *cs, float cq, float ck,
                        float cv, uint8_t *q8, uint8_t *k8, uint8_t *v8)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const int s = r / L, t = r % L;
        const float *a = acc + (size_t)r * PX_QKV;
        for (int p = 0; p < 3; p++) {
            const float sc = p == 0 ? cq : p == 1 ? ck : cv;
            uint8_t *dst = p == 0 ? q8 : p == 1 ? k8 : v8;
            for (int h = 0; h < OR_NH; h++) {
                uint8_t *o = dst + (((size_t)s * OR_NH + h) * L + t) * 64;
                for (int j = 0; j < 32; j++) {
                    const int n = p * OR_D + h * 64 + 2 * j;
                    float f0 = (a[n] + bias[n]) * sc, f1 = (a[n + 1] + bias[n + 1]) * sc;
                    if (p < 2) {
                        const float c = cs[((size_t)t * 32 + j) * 2], sn = cs[((size_t)t * 32 + j) * 2 + 1];
                        const float g0 = f0 * c - f1 * sn;
                        f1 = f1 * c + f0 * sn;
                        f0 = g0;
                    }
                    o[2 * j] = or_e4m3(f0);
                    o[2 * j + 1] = or_e4m3(f1);
                }
            }
        }
    }
}

/* flash8<L> (kern_common.cuh:403-543) over nseq sequences of L tokens: the same walk as or_attention, with query
 * slices of slice_rows rows (16: one reference warp) and key tiles of key_tile keys (64), all within the sequence.
 * out[(s L + t)][h 64 + d] = E4M3(fp16(O (vo / l))). */
void or_px_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nseq, int L, float sinv, float vo,
                     int key_tile, int slice_rows, uint8_t *out)
{
    float lut[256];
    for (int i = 0; i < 256; i++) lut[i] = or_e4m3_dec((uint8_t)i);
    const float thr = RESCALE / sinv, dthr = PSKIP / sinv;
    const int SR = slice_rows;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int sq = 0; sq < nseq; sq++)
        for (int h = 0; h < OR_NH; h++) {
            const size_t base = ((size_t)sq * OR_NH + h) * L;
            float *K = malloc((size_t)L * 64 * 4), *V = malloc((size_t)L * 64 * 4);
            float *S = malloc((size_t)SR * L * 4), *o = malloc((size_t)SR * 64 * 4);
            float *m = malloc(SR * 4), *l = malloc(SR * 4), *tm = malloc(SR * 4);
            for (int t = 0; t < L; t++)
                for (int d = 0; d < 64; d++) {
                    K[t * 64 + d] = lut[k8[(base + t) * 64 + d]];
                    V[t * 64 + d] = lut[v8[(base + t) * 64 + d]];
                }
            for (int g = 0; g < L; g += SR) {
                for (int i = 0; i < SR; i++) {
                    float q[64];
                    for (int d = 0; d < 64; d++) q[d] = lut[q8[(base + g + i) * 64 + d]];
                    for (int t = 0; t < L; t++) {
                        float s4[4] = {0, 0, 0, 0};
                        for (int d = 0; d < 64; d += 4)
                            for (int e = 0; e < 4; e++) s4[e] += q[d + e] * K[t * 64 + d + e];
                        S[(size_t)i * L + t] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
                    }
                    for (int d = 0; d < 64; d++) o[i * 64 + d] = 0.f;
                    m[i] = -1e30f;
                    l[i] = 0.f;
                }
                for (int t0 = 0; t0 < L; t0 += key_tile) {
                    const int t1 = t0 + key_tile < L ? t0 + key_tile : L;
                    int resc = 0, dead = 1;
                    for (int i = 0; i < SR; i++) {
                        tm[i] = -INFINITY;
                        for (int t = t0; t < t1; t++) tm[i] = fmaxf(tm[i], S[(size_t)i * L + t]);
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
                            const float p = exp2f(fmaf(S[(size_t)i * L + t], sinv, -m[i] * sinv));
                            l[i] += p;
                            const float pq = lut[or_e4m3(p)];
                            if (pq != 0.f)
                                for (int d = 0; d < 64; d++) o[i * 64 + d] += pq * V[t * 64 + d];
                        }
                }
                for (int i = 0; i < SR; i++) {
                    const float f = vo / l[i];
                    uint8_t *dst = out + ((size_t)sq * L + g + i) * OR_D + h * 64;
                    for (int d = 0; d < 64; d++) dst[d] = or_e4m3(h16(o[i * 64 + d] * f));
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

/* residual with bias (resgemm, px_kernels.cu:157-187): x = fp16(x + acc + bias[col]), acc = alpha A W^T */
void or_px_resid_bias(uint16_t *x, const float *acc, const float *bias, int rows)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int n = 0; n < OR_D; n++) {
            const size_t i = (size_t)r * OR_D + n;
            x[i] = or_f2h(or_h2f(x[i]) + acc[i] + bias[n]);
        }
}

/* fc1 + GELU (k_pfc1, px_kernels.cu:203-239): v = acc + b1; v *= 0.5 (1 + erf(v / sqrt 2)); u8 = E4M3(v * rs) */
void or_px_fc1_epilogue(const float *acc, int rows, const float *b1, const float *rs, uint8_t *u8)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int n = 0; n < PX_HID; n++) {
            float v = acc[(size_t)r * PX_HID + n] + b1[n];
            v *= 0.5f * (1.0f + erff(v * 0.70710678f));
            u8[(size_t)r * PX_HID + n] = or_e4m3(v * rs[n]);
        }
}

/* Attention-pool head (px.h:168-189; k_phln, k_phscore, k_phsoft, k_phpool, k_phv, px_kernels.cu:347-503; k_headmv,
 * kern_common.cuh:695-727): y = fp16(LN_head(x) + hpos[t]) (eps 1e-5); s[t][h] = U[h] . y[t]; per (image, head)
 * P = fp16(exp2(s - max) / sum); pooled[h] = sum_t P[h][t] y[t] (fp32 sums per 144-token chunk, chunks added in
 * order); o[n] = fp16(Wv[n] . pooled[n / 64]); scores = sigmoid(hw o + hb). o (optional): [nimg][1024] fp16. */
void or_px_head(const uint16_t *x, int nimg, const float *w, const float *b, const float *U, const uint16_t *hpos,
                const uint16_t *wv, const uint16_t *hw, const float *hb, int nt, float *scores, uint16_t *o_out)
{
    const size_t rows = (size_t)nimg * PX_T;
    uint16_t *y = malloc(rows * OR_D * 2);
    float *s = malloc(rows * 16 * 4);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; r++) {
        float v[OR_D], mean, rstd, yf[OR_D];
        for (int i = 0; i < OR_D; i++) v[i] = or_h2f(x[r * OR_D + i]);
        ln_stats(v, EPS_PX, &mean, &rstd);
        const uint16_t *hp = hpos + (r % PX_T) * OR_D;
        for (int i = 0; i < OR_D; i++) {
            y[r * OR_D + i] = or_f2h((v[i] - mean) * rstd * w[i] + b[i] + or_h2f(hp[i]));
            yf[i] = or_h2f(y[r * OR_D + i]);
        }
        for (int h = 0; h < 16; h++) {
            double a = 0;
            for (int i = 0; i < OR_D; i++) a += (double)U[(size_t)h * OR_D + i] * yf[i];
            s[r * 16 + h] = (float)a;
        }
    }
    uint16_t *o = malloc((size_t)nimg * OR_D * 2);
#pragma omp parallel for collapse(2) schedule(static)
    for (int im = 0; im < nimg; im++)
        for (int h = 0; h < 16; h++) {
            const float *sb = s + (size_t)im * PX_T * 16 + h;
            float m = -1e30f;
            double l = 0;
            for (int t = 0; t < PX_T; t++) m = fmaxf(m, sb[(size_t)t * 16]);
            for (int t = 0; t < PX_T; t++) l += exp2f(sb[(size_t)t * 16] - m);
            const float li = (float)(1.0 / l);
            float *P = malloc(PX_T * 4);
            for (int t = 0; t < PX_T; t++) P[t] = h16(exp2f(sb[(size_t)t * 16] - m) * li);
            double pooled[OR_D];
            for (int n = 0; n < OR_D; n++) pooled[n] = 0;
            for (int t = 0; t < PX_T; t++) {
                if (P[t] == 0.f) continue;
                const uint16_t *yr = y + ((size_t)im * PX_T + t) * OR_D;
                for (int n = 0; n < OR_D; n++) pooled[n] += (double)P[t] * or_h2f(yr[n]);
            }
            for (int n = 64 * h; n < 64 * h + 64; n++) {
                double a = 0;
                for (int d = 0; d < OR_D; d++) a += (double)or_h2f(wv[(size_t)n * OR_D + d]) * pooled[d];
                o[(size_t)im * OR_D + n] = or_f2h((float)a);
            }
            free(P);
        }
    or_head_f16(o, nimg, hw, hb, nt, scores);
    if (o_out) memcpy(o_out, o, (size_t)nimg * OR_D * 2);
    free(o);
    free(y);
    free(s);
}

/* ---------------------------------------------------------------------------------------------------------------
 * Model file (px.h:196-245, export_pixai.py:119-146) and the whole forward (px.h:115-190, FP8 path).
 * ------------------------------------------------------------------------------------------------------------- */
typedef struct {
    float *ln1w, *ln1b, *bqkv, *bo, *ln2w, *ln2b, *b1, *rs, *b2;
    uint8_t *wqkv, *wo, *w1, *w2;
    const float *tb;
} px_layer;

typedef struct {
    uint8_t *blob;
    int nt, ntp, nl;
    uint32_t gmask;
    float *table, *pos, *lnpw, *lnpb, *csw, *csg, *hnw, *hnb, *U, *hb;
    uint16_t *pe, *hpos, *wv, *hw;
    px_layer *L;
} px_model;

static void *tk(px_model *M, size_t *off, size_t bytes)
{
    const size_t o = (*off + 255) & ~(size_t)255;
    *off = o + bytes;
    return M->blob + o;
}

static int px_load(const char *path, px_model *M)
{
    memset(M, 0, sizeof(*M));
    FILE *f = fopen(path, "rb");
    uint32_t hdr[6];
    if (!f || fread(hdr, 4, 6, f) != 6 || memcmp(hdr, "PXAI", 4) || hdr[1] != 3) {
        fprintf(stderr, "px oracle: %s is not a pixai.bin v3\n", path);
        if (f) fclose(f);
        return -1;
    }
    M->nt = (int)hdr[2];
    M->ntp = (M->nt + 7) & ~7;
    M->nl = hdr[4] ? (int)hdr[4] : 32;
    M->gmask = hdr[5];
    const size_t bytes = hdr[3];
    M->blob = malloc(bytes);
    if (!M->blob || fseek(f, 256, SEEK_SET) || fread(M->blob, 1, bytes, f) != bytes) {
        fprintf(stderr, "px oracle: cannot read %s\n", path);
        fclose(f);
        free(M->blob);
        return -1;
    }
    fclose(f);
    size_t off = 0;
    M->table = tk(M, &off, (size_t)M->nl * 12 * 4);
    M->pe = tk(M, &off, (size_t)OR_D * OR_K0P * 2);
    M->pos = tk(M, &off, (size_t)PX_T * OR_D * 4);
    M->lnpw = tk(M, &off, OR_D * 4);
    M->lnpb = tk(M, &off, OR_D * 4);
    M->csw = tk(M, &off, (size_t)PX_LW * 64 * 4);
    M->csg = tk(M, &off, (size_t)PX_T * 64 * 4);
    M->L = calloc(M->nl, sizeof(px_layer));
    for (int i = 0; i < M->nl; i++) {
        px_layer *L = &M->L[i];
        L->tb = M->table + (size_t)i * 12;
        L->ln1w = tk(M, &off, OR_D * 4);
        L->ln1b = tk(M, &off, OR_D * 4);
        L->wqkv = tk(M, &off, (size_t)PX_QKV * OR_D);
        L->bqkv = tk(M, &off, PX_QKV * 4);
        L->wo = tk(M, &off, (size_t)OR_D * OR_D);
        L->bo = tk(M, &off, OR_D * 4);
        L->ln2w = tk(M, &off, OR_D * 4);
        L->ln2b = tk(M, &off, OR_D * 4);
        L->w1 = tk(M, &off, (size_t)PX_HID * OR_D);
        L->b1 = tk(M, &off, PX_HID * 4);
        L->rs = tk(M, &off, PX_HID * 4);
        L->w2 = tk(M, &off, (size_t)OR_D * PX_HID);
        L->b2 = tk(M, &off, OR_D * 4);
    }
    M->hnw = tk(M, &off, OR_D * 4);
    M->hnb = tk(M, &off, OR_D * 4);
    M->U = tk(M, &off, 16 * OR_D * 4);
    M->hpos = tk(M, &off, (size_t)PX_T * OR_D * 2);
    M->wv = tk(M, &off, (size_t)OR_D * OR_D * 2);
    M->hw = tk(M, &off, (size_t)M->ntp * OR_D * 2);
    M->hb = tk(M, &off, (size_t)M->ntp * 4);
    if (off != bytes) {
        fprintf(stderr, "px oracle: layout mismatch (%zu vs %zu bytes)\n", off, bytes);
        free(M->L);
        free(M->blob);
        return -1;
    }
    return 0;
}

int or_px_model_nt(const char *model)
{
    px_model M;
    if (px_load(model, &M)) return -1;
    free(M.L);
    free(M.blob);
    return M.nt;
}

static int px_global(const px_model *M, int i) { return M->gmask ? (int)((M->gmask >> i) & 1) : (i & 7) == 7; }

int or_px_forward(const char *model, const uint16_t *in, int nimg, int key_tile, int slice_rows, float *scores,
                  uint16_t *o_out)
{
    px_model M;
    if (px_load(model, &M)) return -1;
    const int rows = nimg * PX_T;
    uint16_t *x = malloc((size_t)rows * OR_D * 2);
    uint8_t *h8 = malloc((size_t)rows * OR_D), *u8 = malloc((size_t)rows * PX_HID);
    uint8_t *q8 = malloc((size_t)rows * OR_D), *k8 = malloc((size_t)rows * OR_D), *v8 = malloc((size_t)rows * OR_D);
    float *acc = malloc((size_t)rows * PX_HID * 4);
    or_px_embed(in, rows, M.pe, M.pos, M.lnpw, M.lnpb, x);
    for (int i = 0; i < M.nl; i++) {
        const px_layer *L = &M.L[i];
        const float *t = L->tb;
        const int glob = px_global(&M, i), Ls = glob ? PX_T : PX_LW;
        /* multipliers of px.h:224-235 */
        const float cq = 1.0f / t[8], ck = 1.0f / t[9], cv = 1.0f / t[10], sinv = t[8] * t[9];
        const float vo = (1.0f / t[5]) * t[10];
        or_ln_e4m3(x, L->ln1w, L->ln1b, rows, 1.0f / t[4], h8);
        or_gemm_e4m3(h8, rows, OR_D, L->wqkv, PX_QKV, NULL, t[0] * t[4], acc);
        or_px_qkv_epilogue(acc, rows, Ls, L->bqkv, glob ? M.csg : M.csw, cq, ck, cv, q8, k8, v8);
        or_px_attention(q8, k8, v8, rows / Ls, Ls, sinv, vo, key_tile, slice_rows, h8);
        or_gemm_e4m3(h8, rows, OR_D, L->wo, OR_D, NULL, t[1] * t[5], acc);
        or_px_resid_bias(x, acc, L->bo, rows);
        or_ln_e4m3(x, L->ln2w, L->ln2b, rows, 1.0f / t[6], h8);
        or_gemm_e4m3(h8, rows, OR_D, L->w1, PX_HID, NULL, t[2] * t[6], acc);
        or_px_fc1_epilogue(acc, rows, L->b1, L->rs, u8);
        or_gemm_e4m3(u8, rows, PX_HID, L->w2, OR_D, NULL, t[3] * t[7], acc);
        or_px_resid_bias(x, acc, L->b2, rows);
    }
    or_px_head(x, nimg, M.hnw, M.hnb, M.U, M.hpos, M.wv, M.hw, M.hb, M.nt, scores, o_out);
    free(x);
    free(h8);
    free(u8);
    free(q8);
    free(k8);
    free(v8);
    free(acc);
    free(M.L);
    free(M.blob);
    return 0;
}

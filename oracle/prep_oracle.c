/* CPU oracle of the GPU preprocessing (TEST INFRASTRUCTURE ONLY: tests/ import it as the checker; the product path
 * never calls it). Restates the wd path of src/core/procimg.h: a decoded RGBA / RGBX image (rows `stride` bytes
 * apart) -> alpha over white -> 2x2 box pyramid -> a crop rect resampled into a 448 x 448 white square with the
 * antialiased bicubic -> fp16 in [-1, 1], BGR planes, patch-operand layout (eva.h:15-16).
 *
 * Parity: procimg.h includes the Windows-only engine headers and cannot be built whole here; its preprocessing
 * functions are cut out of it and compiled with the reference's release flags by tests/golden/make_prep_golden.py,
 * and this restatement is bit-identical to them on every case of tests/golden/golden_prep.json (besides the tests'
 * exact known answers); the GPU kernels are checked against it bit for bit. Float arithmetic follows the
 * reference's source order with one rounding per operation (this file is compiled with -ffp-contract=off), and
 * fmaf where the reference computes a fused multiply-add: its intrinsics (_mm256_fmadd_ps in pi_vrow, _mm_fmadd_ps in
 * pi_hrow and pi_idrow) and the products its compiler contracts (pi_cubic, the white-tap constant of pi_axis). */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "eva_oracle.h"

#define OR_S 448
#define OR_LV 12
#define OR_PYRMIN (2 * OR_S) /* procimg.h:467 */

/* x / 255 rounded, exact for x in [0, 65025] (PI_DIV255, procimg.h:584) */
uint32_t or_div255(uint32_t x) { return (x + 128 + ((x + 128) >> 8)) >> 8; }

/* Alpha over white in place, X = 255 (pi_row_rgbx, procimg.h:602-630); without alpha only X is set. */
void or_over_white(uint8_t *img, int w, int h, int stride, int alpha)
{
    for (int y = 0; y < h; y++) {
        uint8_t *p = img + (size_t)y * stride;
        for (int x = 0; x < w; x++, p += 4) {
            if (alpha) {
                const uint32_t a = p[3], ia = 255 * (255 - a);
                for (int c = 0; c < 3; c++) p[c] = (uint8_t)or_div255(p[c] * a + ia);
            }
            p[3] = 255;
        }
    }
}

/* One 2x2 box level (pi_half, procimg.h:635-660): the two rows average rounding up, then the two columns rounding
 * down. d is (sw >> 1) x (sh >> 1) pixels, rows dstride bytes apart. */
void or_half(const uint8_t *s, int sw, int sh, int sstride, uint8_t *d, int dstride)
{
    const int wn = sw >> 1, hn = sh >> 1;
    for (int y = 0; y < hn; y++) {
        const uint8_t *r0 = s + (size_t)2 * y * sstride, *r1 = r0 + sstride;
        uint8_t *o = d + (size_t)y * dstride;
        for (int x = 0; x < wn; x++)
            for (int c = 0; c < 4; c++) {
                const uint32_t ve = (r0[8 * x + c] + r1[8 * x + c] + 1u) >> 1;
                const uint32_t vo = (r0[8 * x + 4 + c] + r1[8 * x + 4 + c] + 1u) >> 1;
                o[4 * x + c] = (uint8_t)((ve + vo) >> 1);
            }
    }
}

typedef struct {
    int nlv, lw[OR_LV], lh[OR_LV], ls[OR_LV];
    const uint8_t *lv[OR_LV];
    uint8_t *blk;
} or_pyr;

/* Levels 1.. while the next level's long side stays >= 896 (pi_pyramid, procimg.h:665-690). */
static void pyr_build(or_pyr *p, const uint8_t *img, int w, int h, int stride)
{
    size_t total = 0;
    int n;
    p->lw[0] = w;
    p->lh[0] = h;
    p->ls[0] = stride;
    p->lv[0] = img;
    for (n = 1; n < OR_LV; n++) {
        const int m = p->lw[n - 1] > p->lh[n - 1] ? p->lw[n - 1] : p->lh[n - 1];
        if ((m >> 1) < OR_PYRMIN || p->lw[n - 1] < 2 || p->lh[n - 1] < 2) break;
        p->lw[n] = p->lw[n - 1] >> 1;
        p->lh[n] = p->lh[n - 1] >> 1;
        p->ls[n] = p->lw[n] * 4;
        total += (size_t)p->ls[n] * p->lh[n];
    }
    p->nlv = n;
    p->blk = n > 1 ? malloc(total) : NULL;
    uint8_t *b = p->blk;
    for (int L = 1; L < n; L++) {
        or_half(p->lv[L - 1], p->lw[L - 1], p->lh[L - 1], p->ls[L - 1], b, p->ls[L]);
        p->lv[L] = b;
        b += (size_t)p->ls[L] * p->lh[L];
    }
}

/* Keys bicubic, a = -0.5 (pi_cubic, procimg.h:751-756), as the reference's release build computes it: GCC at -O3 with
 * FMA available (src/CMakeLists.txt:38,73) contracts each multiply whose product feeds one add into a fused
 * multiply-add, so (1.5 x - 2.5) x x + 1 is fma(fma(1.5, x, -2.5) x, x, 1) and the second branch a chain of three. */
static float cubic(float x)
{
    x = x < 0 ? -x : x;
    return x < 1.0f ? fmaf(fmaf(1.5f, x, -2.5f) * x, x, 1.0f)
         : x < 2.0f ? fmaf(fmaf(fmaf(-0.5f, x, 2.5f), x, -4.0f), x, 2.0f) : 0.0f;
}

/* One axis of the resample (pi_axis, procimg.h:761-795): virtual white square [0, side) -> [0, S), content at
 * [off, off + len); output i reads content [s[i], s[i] + n[i]) with weights w[i * mt ..] scaled by sc, and k[i]
 * carries the white taps plus add. */
static void axis(int S, int side, int off, int len, int mt, float sc, float add, float *w, int *s, int *n, float *k)
{
    const float scale = (float)side / (float)S;
    const float fs = scale > 1.0f ? scale : 1.0f;
    const float support = 2.0f * fs;
    const float ss = 1.0f / fs;
    const int end = off + len;
    for (int i = 0; i < S; i++) {
        float *wi = w + (size_t)i * mt;
        const float center = ((float)i + 0.5f) * scale;
        int lo = (int)(center - support + 0.5f);
        lo = lo < 0 ? 0 : lo;
        int hi = (int)(center + support + 0.5f);
        hi = hi > side ? side : hi;
        const int a = lo > off ? lo : off;
        int b = hi < end ? hi : end;
        b = b < a ? a : b;
        float sum = 0.0f, white = 0.0f;
        for (int j = lo; j < hi; j++) {
            const float wt = cubic(((float)j - center + 0.5f) * ss);
            sum += wt;
            white += j < a || j >= b ? wt : 0.0f;
            wi[j - lo] = wt;
        }
        memmove(wi, wi + (a - lo), (size_t)(b - a) * sizeof(float));
        sum = sc / sum;
        for (int j = 0; j < b - a; j++) wi[j] *= sum;
        s[i] = a - off;
        n[i] = b - a;
        k[i] = fmaf(255.0f * white, sum, add);   /* contracted in the reference's build, as cubic */
    }
}

static uint16_t f2h(float v)
{
    uint16_t h;
    or_f2h_n(&v, &h, 1);
    return h;
}

/* Operand index of output pixel (i, j), channel plane q (0 B, 1 G, 2 R): patch (i / 14) * 32 + j / 14, column
 * q * 196 + (i % 14) * 14 + j % 14 (procimg.h:1607 and the band layout of pi_prep). */
static size_t opidx(int i, int j, int q) { return ((size_t)(i / 14) * 32 + j / 14) * 592 + q * 196 + (i % 14) * 14 + j % 14; }

/* Crop (x0, y0, cw, ch) of level 0 -> one model input (pi_prep, procimg.h:926-969, with pi_level, pi_lsrc,
 * pi_vrow, pi_hrow and pi_idrow). out: 1024 x 592 halves; pad columns 588..591 are written as zero. */
static void prep_crop(const or_pyr *p, int x0, int y0, int cw, int ch, uint16_t *out)
{
    const int S = OR_S;
    int L = 0;
    const int side0 = cw > ch ? cw : ch;
    while (L + 1 < p->nlv && (side0 >> (L + 1)) >= 2 * S) L++;
    /* the rect on level L (clipped, at least one pixel) */
    int x1 = (x0 + cw) >> L, y1 = (y0 + ch) >> L;
    x1 = x1 < p->lw[L] ? x1 : p->lw[L];
    y1 = y1 < p->lh[L] ? y1 : p->lh[L];
    x0 >>= L;
    y0 >>= L;
    x0 = x0 < p->lw[L] ? x0 : p->lw[L] - 1;
    y0 = y0 < p->lh[L] ? y0 : p->lh[L] - 1;
    cw = x1 > x0 ? x1 - x0 : 1;
    ch = y1 > y0 ? y1 - y0 : 1;
    const size_t stride = p->ls[L];
    const uint8_t *src = p->lv[L] + (size_t)y0 * stride + (size_t)x0 * 4;
    const int side = cw > ch ? cw : ch;
    for (int pt = 0; pt < 1024; pt++)
        for (int c = 588; c < 592; c++) out[(size_t)pt * 592 + c] = 0;
    if (side == S) {
        const int ox = (S - cw) >> 1, oy = (S - ch) >> 1;
        const float sc = 1.0f / 127.5f;
        for (int i = 0; i < S; i++) {
            const int r = i - oy;
            for (int j = 0; j < S; j++) {
                const int cj = j - ox;
                if (r < 0 || r >= ch || cj < 0 || cj >= cw) {
                    for (int q = 0; q < 3; q++) out[opidx(i, j, q)] = 0x3C00;
                    continue;
                }
                const uint8_t *px = src + (size_t)r * stride + (size_t)cj * 4;
                for (int q = 0; q < 3; q++) out[opidx(i, j, q)] = f2h(fmaf((float)px[2 - q], sc, -1.0f));
            }
        }
        return;
    }
    const int mt = 2 * (int)(2.0f * (side > S ? (float)side / (float)S : 1.0f) + 1.0f) + 2;
    float *wx = malloc((size_t)S * mt * sizeof(float)), *wy = malloc((size_t)S * mt * sizeof(float));
    float *kx = malloc(S * sizeof(float)), *ky = malloc(S * sizeof(float));
    int *sx = malloc(S * sizeof(int)), *nx = malloc(S * sizeof(int)), *sy = malloc(S * sizeof(int)), *ny = malloc(S * sizeof(int));
    float *tmp = malloc((size_t)cw * 4 * sizeof(float));
    axis(S, side, (side - cw) >> 1, cw, mt, 1.0f / 127.5f, -1.0f, wx, sx, nx, kx);
    axis(S, side, (side - ch) >> 1, ch, mt, 1.0f, 0.0f, wy, sy, ny, ky);
    for (int i = 0; i < S; i++) {
        const float *w = wy + (size_t)i * mt;
        for (int x = 0; x < cw * 4; x++) {
            float a = ky[i];
            for (int j = 0; j < ny[i]; j++) a = fmaf(w[j], (float)src[(size_t)(sy[i] + j) * stride + x], a);
            tmp[x] = a;
        }
        for (int j = 0; j < S; j++) {
            const float *wj = wx + (size_t)j * mt;
            for (int q = 0; q < 3; q++) {
                float a = kx[j];
                for (int t = 0; t < nx[j]; t++) a = fmaf(wj[t], tmp[4 * (sx[j] + t) + (2 - q)], a);
                a = a > -1.0f ? a : -1.0f;  /* _mm_max_ps(acc, -1) then _mm_min_ps(., 1) */
                a = a < 1.0f ? a : 1.0f;
                out[opidx(i, j, q)] = f2h(a);
            }
        }
    }
    free(wx), free(wy), free(kx), free(ky), free(sx), free(nx), free(sy), free(ny), free(tmp);
}

/* Whole pipeline for one image: img (RGBA, modified in place: alpha over white), then the crop. */
void or_prep(uint8_t *img, int w, int h, int stride, int alpha, int x0, int y0, int cw, int ch, uint16_t *out)
{
    or_pyr p;
    or_over_white(img, w, h, stride, alpha);
    pyr_build(&p, img, w, h, stride);
    prep_crop(&p, x0, y0, cw, ch, out);
    free(p.blk);
}

/* Number of pyramid levels and the level a crop side resamples from (for the tests). */
int or_prep_level(int w, int h, int side)
{
    int lw = w, lh = h, nlv = 1, L = 0;
    while (nlv < OR_LV) {
        const int m = lw > lh ? lw : lh;
        if ((m >> 1) < OR_PYRMIN || lw < 2 || lh < 2) break;
        lw >>= 1;
        lh >>= 1;
        nlv++;
    }
    while (L + 1 < nlv && (side >> (L + 1)) >= 2 * OR_S) L++;
    return L;
}

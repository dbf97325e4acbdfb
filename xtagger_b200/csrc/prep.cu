// GPU preprocessing: a decoded RGBA / RGBX image on the device -> one model input (the fp16 patch operand of
// eva.h:15-16), the work xTagger does on the host in src/core/procimg.h (pi_ingest / pi_prep, wd path):
//   1. alpha over white in place, X = 255 (pi_row_rgbx, procimg.h:602-630: c' = (c a + 255 (255 - a)) / 255,
//      rounded exactly: PI_DIV255, procimg.h:584);
//   2. the 2x2 box pyramid, levels while the long side stays >= 896 (pi_pyramid / pi_half, procimg.h:635-690:
//      rows average rounding up, then columns rounding down);
//   3. a crop rect (x0, y0, cw, ch) of level 0 taken from the coarsest level that still leaves a factor >= 2
//      (pi_level / pi_lsrc, procimg.h:692-717) and resampled into a 448 x 448 white square, content centred, with
//      the antialiased Keys bicubic (a = -0.5) in two separable passes whose weights fold in the white taps and the
//      [-1, 1] normalisation (pi_axis / pi_vrow / pi_hrow, procimg.h:751-868); a rect whose long side is already 448
//      is only normalised and white-padded (pi_idrow, procimg.h:874-905);
//   4. fp16 (round to nearest even), BGR planes, patch-operand layout: pixel (i, j) channel plane q at patch
//      (i / 14) * 32 + j / 14, column q * 196 + (i % 14) * 14 + j % 14; columns 588..591 zero.
// The arithmetic is the reference's operation for operation: integer steps exactly, the filter weights with one
// rounding per operation in source order (explicit _rn intrinsics, so the compiler fuses nothing on its own) and a
// fused multiply-add exactly where the reference's release build has one (the products GCC -O3 contracts in
// pi_cubic and pi_axis), and the two passes as chains of fused multiply-adds in tap order, as the reference's
// _mm256_fmadd_ps / _mm_fmadd_ps. The outputs are bit-identical to procimg.h's own functions compiled with the
// reference's flags (tests/golden/golden_prep.json).
//
// Kernels (all HBM / L2-bound byte and fp32 work): k_over_white (one pixel per thread), k_half (one output pixel per
// thread), k_axis (one output index per thread, both axes), k_vpass (one source pixel of one output row per thread:
// four channel accumulators over the vertical taps), k_hpass (one output pixel per thread: three channel
// accumulators over the horizontal taps), k_ident (the scale-1 case).
#include <algorithm>

#include "../../include/xtagger_b200.h"
#include "host.h"
#include "ops.h"

namespace xtb {

constexpr int PREP_S = 448;                 // model side (EVA_S)
constexpr int PREP_LV = 12;                 // pyramid levels at most (procimg.h:466)
constexpr int PREP_PYRMIN = 2 * PREP_S;     // procimg.h:467

__device__ __forceinline__ uint32_t div255(uint32_t x) { return (x + 128 + ((x + 128) >> 8)) >> 8; }

__global__ void k_over_white(uint8_t *img, int w, int stride, int alpha)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= w) return;
    uint32_t *p = (uint32_t *)(img + (size_t)y * stride) + x;
    uint32_t v = *p;
    if (alpha) {
        const uint32_t a = v >> 24, ia = 255 * (255 - a);
        v = div255((v & 255) * a + ia) | (div255(((v >> 8) & 255) * a + ia) << 8) | (div255(((v >> 16) & 255) * a + ia) << 16);
    }
    *p = v | 0xFF000000u;
}

__global__ void k_half(const uint8_t *s, int sstride, uint8_t *d, int wn, int dstride)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= wn) return;
    const uint8_t *r0 = s + (size_t)2 * y * sstride + 8 * x, *r1 = r0 + sstride;
    const uint32_t a0 = *(const uint32_t *)r0, a1 = *(const uint32_t *)(r0 + 4);
    const uint32_t b0 = *(const uint32_t *)r1, b1 = *(const uint32_t *)(r1 + 4);
    uint32_t o = 0;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint32_t ve = (((a0 >> 8 * c) & 255) + ((b0 >> 8 * c) & 255) + 1) >> 1;
        const uint32_t vo = (((a1 >> 8 * c) & 255) + ((b1 >> 8 * c) & 255) + 1) >> 1;
        o |= ((ve + vo) >> 1) << 8 * c;
    }
    *(uint32_t *)(d + (size_t)y * dstride + 4 * x) = o;
}

// Keys bicubic, a = -0.5 (pi_cubic), as the reference's release build evaluates it (GCC -O3 with FMA contracts every
// product that feeds one add): fma(fma(1.5, x, -2.5) x, x, 1) and a chain of three fused multiply-adds.
__device__ __forceinline__ float cubic_rn(float x)
{
    x = fabsf(x);
    if (x < 1.0f) return __fmaf_rn(__fmul_rn(__fmaf_rn(1.5f, x, -2.5f), x), x, 1.0f);
    if (x < 2.0f) return __fmaf_rn(__fmaf_rn(__fmaf_rn(-0.5f, x, 2.5f), x, -4.0f), x, 2.0f);
    return 0.0f;
}

struct AxisArgs {
    int side, off, len, mt;
    float sc, add;
    float *w, *k;
    int *s, *n;
};

// pi_axis for one output index i of one axis (blockIdx.y: 0 x, 1 y)
__global__ void k_axis(AxisArgs ax, AxisArgs ay)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= PREP_S) return;
    const AxisArgs &A = blockIdx.y ? ay : ax;
    const float scale = __fdiv_rn((float)A.side, (float)PREP_S);
    const float fs = scale > 1.0f ? scale : 1.0f;
    const float support = __fmul_rn(2.0f, fs);
    const float ss = __fdiv_rn(1.0f, fs);
    const int end = A.off + A.len;
    const float center = __fmul_rn(__fadd_rn((float)i, 0.5f), scale);
    int lo = __float2int_rz(__fadd_rn(__fsub_rn(center, support), 0.5f));
    lo = lo < 0 ? 0 : lo;
    int hi = __float2int_rz(__fadd_rn(__fadd_rn(center, support), 0.5f));
    hi = hi > A.side ? A.side : hi;
    const int a = lo > A.off ? lo : A.off;
    int b = hi < end ? hi : end;
    b = b < a ? a : b;
    float *wi = A.w + (size_t)i * A.mt;
    float sum = 0.0f, white = 0.0f;
    for (int j = lo; j < hi; j++) {
        const float wt = cubic_rn(__fmul_rn(__fadd_rn(__fsub_rn((float)j, center), 0.5f), ss));
        sum = __fadd_rn(sum, wt);
        const bool out = j < a || j >= b;
        white = __fadd_rn(white, out ? wt : 0.0f);
        if (!out) wi[j - a] = wt;
    }
    sum = __fdiv_rn(A.sc, sum);
    for (int j = 0; j < b - a; j++) wi[j] = __fmul_rn(wi[j], sum);
    A.s[i] = a - A.off;
    A.n[i] = b - a;
    A.k[i] = __fmaf_rn(__fmul_rn(255.0f, white), sum, A.add);  // contracted in the reference's build, as cubic_rn
}

// Vertical pass for output row blockIdx.y: tmp[i][4 px + c] = k[i] + sum_j w[i][j] src[s[i] + j][px][c] (FMA chain)
__global__ void k_vpass(const uint8_t *src, int stride, int cw, int mt, const float *wy, const int *sy, const int *ny,
                        const float *ky, float *tmp)
{
    const int px = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (px >= cw) return;
    const float *w = wy + (size_t)i * mt;
    const uint8_t *p = src + (size_t)sy[i] * stride + 4 * px;
    const float k = ky[i];
    float a0 = k, a1 = k, a2 = k, a3 = k;
    for (int j = 0, n = ny[i]; j < n; j++, p += stride) {
        const uint32_t v = *(const uint32_t *)p;
        const float wj = w[j];
        a0 = fmaf(wj, (float)(v & 255), a0);
        a1 = fmaf(wj, (float)((v >> 8) & 255), a1);
        a2 = fmaf(wj, (float)((v >> 16) & 255), a2);
        a3 = fmaf(wj, (float)(v >> 24), a3);
    }
    *(float4 *)(tmp + (size_t)i * cw * 4 + 4 * px) = make_float4(a0, a1, a2, a3);
}

__device__ __forceinline__ size_t op_index(int i, int j, int q)
{
    return ((size_t)(i / 14) * 32 + j / 14) * K0P + q * 196 + (i % 14) * 14 + j % 14;
}

// pad columns 588..591 of the 32 patches whose first pixel row is i (one thread per column)
__device__ __forceinline__ void zero_pad(int i, int j, uint16_t *out)
{
    if (i % 14 == 0 && j < 32 * 4) out[((size_t)(i / 14) * 32 + j / 4) * K0P + 588 + (j & 3)] = 0;
}

__device__ __forceinline__ uint16_t h_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

// Horizontal pass for output pixel (blockIdx.y, j): three channels over the taps of tmp's row, clamped to [-1, 1]
__global__ void k_hpass(const float *tmp, int cw, int mt, const float *wx, const int *sx, const int *nx, const float *kx,
                        uint16_t *out)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (j >= PREP_S) return;
    const float4 *t = (const float4 *)(tmp + (size_t)i * cw * 4) + sx[j];
    const float *w = wx + (size_t)j * mt;
    float r = kx[j], g = r, b = r;
    for (int q = 0, n = nx[j]; q < n; q++) {
        const float4 v = t[q];
        const float wq = w[q];
        r = fmaf(wq, v.x, r);
        g = fmaf(wq, v.y, g);
        b = fmaf(wq, v.z, b);
    }
    r = fminf(fmaxf(r, -1.0f), 1.0f);
    g = fminf(fmaxf(g, -1.0f), 1.0f);
    b = fminf(fmaxf(b, -1.0f), 1.0f);
    out[op_index(i, j, 0)] = h_bits(b);
    out[op_index(i, j, 1)] = h_bits(g);
    out[op_index(i, j, 2)] = h_bits(r);
    zero_pad(i, j, out);
}

// Scale 1: content pixels v / 127.5 - 1 (one FMA), the rest white (1.0)
__global__ void k_ident(const uint8_t *src, int stride, int cw, int ch, int ox, int oy, uint16_t *out)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (j >= PREP_S) return;
    const int r = i - oy, c = j - ox;
    uint16_t hb = 0x3C00, hg = 0x3C00, hr = 0x3C00;
    if (r >= 0 && r < ch && c >= 0 && c < cw) {
        const uint32_t v = *(const uint32_t *)(src + (size_t)r * stride + 4 * c);
        const float sc = 1.0f / 127.5f;
        hr = h_bits(fmaf((float)(v & 255), sc, -1.0f));
        hg = h_bits(fmaf((float)((v >> 8) & 255), sc, -1.0f));
        hb = h_bits(fmaf((float)((v >> 16) & 255), sc, -1.0f));
    }
    out[op_index(i, j, 0)] = hb;
    out[op_index(i, j, 1)] = hg;
    out[op_index(i, j, 2)] = hr;
    zero_pad(i, j, out);
}

// ---- host side ----
struct Pyr {
    int n, lw[PREP_LV], lh[PREP_LV];
    size_t off[PREP_LV];  // levels 1..: byte offset in the scratch (rows lw * 4 bytes apart)
    size_t bytes;         // of all levels 1..
};

static Pyr pyr_dims(int w, int h)
{
    Pyr p;
    p.lw[0] = w;
    p.lh[0] = h;
    p.off[0] = 0;
    p.bytes = 0;
    int n = 1;
    for (; n < PREP_LV; n++) {
        const int m = std::max(p.lw[n - 1], p.lh[n - 1]);
        if ((m >> 1) < PREP_PYRMIN || p.lw[n - 1] < 2 || p.lh[n - 1] < 2) break;
        p.lw[n] = p.lw[n - 1] >> 1;
        p.lh[n] = p.lh[n - 1] >> 1;
        p.off[n] = p.bytes;
        p.bytes += ((size_t)p.lw[n] * 4 * p.lh[n] + 255) & ~(size_t)255;
    }
    p.n = n;
    return p;
}

static int max_taps(int side)
{
    return 2 * (int)(2.0f * (side > PREP_S ? (float)side / (float)PREP_S : 1.0f) + 1.0f) + 2;
}

// scratch: [levels 1..][axis tables: 2 x (w [S][mt], k [S], s [S], n [S])][tmp: S rows x w * 4 floats]
static size_t tables_bytes(int mt) { return 2 * (((size_t)PREP_S * mt * 4 + 3 * PREP_S * 4 + 255) & ~(size_t)255); }

static size_t scratch_bytes(int w, int h)
{
    const Pyr p = pyr_dims(w, h);
    return p.bytes + tables_bytes(max_taps(std::max(w, h))) + (size_t)PREP_S * w * 16;
}

static bool image_ok(const void *img, int w, int h, int stride, const char *what)
{
    if (!img || w <= 0 || h <= 0 || stride < 4 * w || (stride & 3) || ((uintptr_t)img & 3)) {
        fprintf(stderr, "eva: %s: bad image (%p, %d x %d, stride %d: 4-byte aligned RGBA rows of at least 4 w bytes)\n",
                what, img, w, h, stride);
        return false;
    }
    return true;
}

int prep_ingest(uint8_t *img, int w, int h, int stride, int alpha, uint8_t *scratch, cudaStream_t st)
{
    k_over_white<<<dim3((w + 255) / 256, h), 256, 0, st>>>(img, w, stride, alpha);
    XTB_CK(cudaGetLastError());
    const Pyr p = pyr_dims(w, h);
    for (int L = 1; L < p.n; L++) {
        const uint8_t *s = L == 1 ? img : scratch + p.off[L - 1];
        const int ss = L == 1 ? stride : p.lw[L - 1] * 4;
        k_half<<<dim3((p.lw[L] + 255) / 256, p.lh[L]), 256, 0, st>>>(s, ss, scratch + p.off[L], p.lw[L], p.lw[L] * 4);
        XTB_CK(cudaGetLastError());
    }
    return 0;
}

// The pyramid level a crop reads and the rect on it (clipped, at least one pixel); returns the level.
static int crop_level(const Pyr &p, int &x0, int &y0, int &cw, int &ch)
{
    const int side0 = std::max(cw, ch);
    int L = 0;
    while (L + 1 < p.n && (side0 >> (L + 1)) >= 2 * PREP_S) L++;
    int x1 = std::min((x0 + cw) >> L, p.lw[L]), y1 = std::min((y0 + ch) >> L, p.lh[L]);
    x0 = std::min(x0 >> L, p.lw[L] - 1);
    y0 = std::min(y0 >> L, p.lh[L] - 1);
    cw = x1 > x0 ? x1 - x0 : 1;
    ch = y1 > y0 ? y1 - y0 : 1;
    return L;
}

int prep_crop(const uint8_t *img, int w, int h, int stride, int x0, int y0, int cw, int ch, uint8_t *scratch,
              uint16_t *out, cudaStream_t st)
{
    const Pyr p = pyr_dims(w, h);
    const int L = crop_level(p, x0, y0, cw, ch);
    const int ls = L == 0 ? stride : p.lw[L] * 4;
    const uint8_t *src = (L == 0 ? img : scratch + p.off[L]) + (size_t)y0 * ls + (size_t)x0 * 4;
    const int side = std::max(cw, ch);
    const dim3 grid((PREP_S + 127) / 128, PREP_S);
    if (side == PREP_S) {
        k_ident<<<grid, 128, 0, st>>>(src, ls, cw, ch, (PREP_S - cw) >> 1, (PREP_S - ch) >> 1, out);
        XTB_CK(cudaGetLastError());
        return 0;
    }
    const int mt = max_taps(side);
    uint8_t *tb = scratch + p.bytes;
    const size_t half = tables_bytes(mt) / 2;
    auto axis = [&](uint8_t *base, int off, int len, float sc, float add) {
        AxisArgs a;
        a.side = side;
        a.off = off;
        a.len = len;
        a.mt = mt;
        a.sc = sc;
        a.add = add;
        a.w = (float *)base;
        a.k = a.w + (size_t)PREP_S * mt;
        a.s = (int *)(a.k + PREP_S);
        a.n = a.s + PREP_S;
        return a;
    };
    const AxisArgs ax = axis(tb, (side - cw) >> 1, cw, 1.0f / 127.5f, -1.0f);
    const AxisArgs ay = axis(tb + half, (side - ch) >> 1, ch, 1.0f, 0.0f);
    float *tmp = (float *)(tb + 2 * half);
    k_axis<<<dim3((PREP_S + 127) / 128, 2), 128, 0, st>>>(ax, ay);
    XTB_CK(cudaGetLastError());
    k_vpass<<<dim3((cw + 127) / 128, PREP_S), 128, 0, st>>>(src, ls, cw, mt, ay.w, ay.s, ay.n, ay.k, tmp);
    XTB_CK(cudaGetLastError());
    k_hpass<<<grid, 128, 0, st>>>(tmp, cw, mt, ax.w, ax.s, ax.n, ax.k, out);
    XTB_CK(cudaGetLastError());
    return 0;
}

}  // namespace xtb

using namespace xtb;

extern "C" {

size_t xtb_prep_scratch_bytes(int w, int h)
{
    if (w <= 0 || h <= 0) return 0;
    return scratch_bytes(w, h);
}

int xtb_prep_ingest(uint8_t *rgba, int w, int h, int stride, int alpha, void *scratch, void *stream)
{
    if (!image_ok(rgba, w, h, stride, "xtb_prep_ingest") || !scratch) return -1;
    return prep_ingest(rgba, w, h, stride, alpha, (uint8_t *)scratch, (cudaStream_t)stream);
}

int xtb_prep_crop(const uint8_t *rgba, int w, int h, int stride, int x0, int y0, int cw, int ch, void *scratch,
                  uint16_t *out, void *stream)
{
    if (!image_ok(rgba, w, h, stride, "xtb_prep_crop") || !scratch || !out) return -1;
    if (x0 < 0 || y0 < 0 || cw <= 0 || ch <= 0 || x0 + cw > w || y0 + ch > h) {
        fprintf(stderr, "eva: xtb_prep_crop: rect (%d, %d, %d x %d) outside the %d x %d image\n", x0, y0, cw, ch, w, h);
        return -1;
    }
    return prep_crop(rgba, w, h, stride, x0, y0, cw, ch, (uint8_t *)scratch, out, (cudaStream_t)stream);
}

int xtb_prep_kernels(int w, int h, int x0, int y0, int cw, int ch)
{
    if (w <= 0 || h <= 0) return -1;
    const Pyr p = pyr_dims(w, h);
    if (cw <= 0) return p.n;  // xtb_prep_ingest: alpha over white, then one box-halving kernel per level
    if (x0 < 0 || y0 < 0 || ch <= 0 || x0 + cw > w || y0 + ch > h) return -1;
    crop_level(p, x0, y0, cw, ch);
    return std::max(cw, ch) == PREP_S ? 1 : 3;  // normalise only, or weight tables + vertical + horizontal pass
}

}  // extern "C"

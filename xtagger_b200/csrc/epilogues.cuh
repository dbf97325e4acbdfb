// Fused GEMM epilogues of the EVA02-L forward (calling convention in gemm.cuh). Each one replaces a reference
// kernel's epilogue, written for the tcgen05 GEMM's one-row-per-thread accumulator layout:
//   EpiQKV    <- k_qkv   (eva_kernels.cu:41-114):  RoPE on q / k of patch tokens, E4M3, attention layouts
//   EpiResid  <- k_oproj (eva_kernels.cu:134-162): fp16 residual += acc
//   EpiFC1    <- k_fc1   (eva_kernels.cu:211-279): SwiGLU, per-row LN statistics partials, E4M3 h
//   EpiFC2    <- k_fc2   (eva_kernels.cu:286-334): inner MLP LayerNorm folded in, fp16 residual += ...
//   EpiPatch  <- k_pe + k_embed (eva_kernels.cu:21-33, 126-130): patch embedding + position / cls rows
//   EpiHead   <- k_headmv (kern_common.cuh:695-727): logits + bias -> sigmoid, weights as the M operand
#pragma once
#include "gemm.cuh"
#include "ops.h"

namespace xtb {

// ---- QKV projection: acc = x W_qkv^T (dequantised); columns [0,1024) q, [1024,2048) k, [2048,3072) v ----
// q, k: scaled by cq / ck, interleaved RoPE (pair (2j, 2j+1) of a head shares angle j, table cs[t - 1][j] =
// (cos, sin)) for patch tokens t >= 1, E4M3 -> q8 / k8 [img][head][TP][64] (row t of 64 dims).
// v: scaled by cv, E4M3 -> vt8 [img][head][64 dims][TP] (V transposed: keys contiguous per dim).
// Padded key rows / columns t >= 1025 are zeroed once at allocation and never written.
struct EpiQKV {
    struct Params {
        uint8_t *q8, *k8, *vt8;
        const float2 *cs;
        float cq, ck, cv;
        int M;
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
        const int which = cx.col0 >> 10;           // 0 q, 1 k, 2 v (a thread's 128 columns never straddle)
        const int head0 = (cx.col0 & 1023) >> 6;   // two heads per thread
        const int row = cx.row0 + cx.lane;
        const int b = row / T, t = row - b * T;
        if (which < 2) {
            const float sc = which ? p.ck : p.cq;
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                uint32_t w[16];
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    float f[4];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        float f0 = acc[hh * 64 + 2 * (j + e)] * sc, f1 = acc[hh * 64 + 2 * (j + e) + 1] * sc;
                        if (t > 0 && row < p.M) {
                            const float2 a = p.cs[(t - 1) * 32 + j + e];
                            const float g0 = f0 * a.x - f1 * a.y;
                            f1 = f1 * a.x + f0 * a.y;
                            f0 = g0;
                        }
                        f[2 * e] = f0;
                        f[2 * e + 1] = f1;
                    }
                    w[j >> 1] = e4m3x2(f[0], f[1]) | (e4m3x2(f[2], f[3]) << 16);
                }
#pragma unroll
                for (int c = 0; c < 4; c++)
                    *(uint4 *)stage_chunk(cx.stage, cx.lane, 4 * hh + c) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
            }
            __syncwarp();
            uint8_t *dst = which ? p.k8 : p.q8;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int pc = i * 32 + cx.lane;          // piece: head hh, row r, 16-byte chunk ch
                const int hh = pc >> 7, r = (pc >> 2) & 31, ch = pc & 3;
                const int rw = cx.row0 + r;
                if (rw < p.M) {
                    const int bb = rw / T, tt = rw - bb * T;
                    *(uint4 *)(dst + (((size_t)(bb * NH + head0 + hh) * TP + tt) << 6) + ch * 16) =
                        *(const uint4 *)stage_chunk(cx.stage, r, 4 * hh + ch);
                }
            }
            __syncwarp();
        } else if (row < p.M) {
            // V^T: for each dim, the 32 lanes (consecutive tokens) write consecutive key bytes
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                uint8_t *col = p.vt8 + ((size_t)(b * NH + head0 + hh) * HD) * TP + t;
#pragma unroll
                for (int d = 0; d < 64; d += 2) {
                    const uint32_t pr = e4m3x2(acc[hh * 64 + d] * p.cv, acc[hh * 64 + d + 1] * p.cv);
                    col[(size_t)d * TP] = (uint8_t)pr;
                    col[(size_t)(d + 1) * TP] = (uint8_t)(pr >> 8);
                }
            }
        }
    }
};

// ---- fp16 residual update: x[row][col] = fp16(x + acc) (attention out-projection) ----
struct EpiResid {
    struct Params {
        __half *x;
        int M;
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            __syncwarp();
            stage_row_f32(cx.stage, cx.lane, acc + 32 * c);
            __syncwarp();
            const int w = (cx.lane & 15) * 2;
#pragma unroll 4
            for (int i = 0; i < 16; i++) {
                const int r = 2 * i + (cx.lane >> 4), row = cx.row0 + r;
                if (row < p.M) {
                    __half2 *xp = (__half2 *)(p.x + (size_t)row * D + cx.col0 + 32 * c + w);
                    const float2 a = stage_f32x2(cx.stage, r, w);
                    const float2 xf = __half22float2(*xp);
                    *xp = __floats2half2_rn(xf.x + a.x, xf.y + a.y);
                }
            }
        }
        __syncwarp();
    }
};

// ---- fc1 + SwiGLU: W12 rows interleave g / x in 16-unit chunks (32 columns = units 16c .. 16c + 15) ----
// u = x * g * sigmoid(g) (sigmoid(g) = 0.5 (1 + tanh(g / 2)), as the reference), h8 = E4M3(u * rs[unit]),
// stat[col0 / 128][row] = (sum u, sum u^2) over this thread's 64 units (each partial has exactly one writer).
struct EpiFC1 {
    struct Params {
        uint8_t *h8;
        float2 *stat;
        const float *rs;
        int M;
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
        const int row = cx.row0 + cx.lane;
        float s = 0.f, q = 0.f;
        int nch = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int n = cx.col0 + 32 * c;
            if (n >= N12) break;
            nch = c + 1;
            const int ub = n >> 1;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float hq[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float gg = acc[32 * c + i + e], xx = acc[32 * c + 16 + i + e];
                    const float u = xx * (0.5f * gg * (1.0f + tanh_fast(0.5f * gg)));
                    s += u;
                    q += u * u;
                    hq[e] = u * __ldg(p.rs + ub + i + e);
                }
                w[i >> 2] = e4m3x2(hq[0], hq[1]) | (e4m3x2(hq[2], hq[3]) << 16);
            }
            *(uint4 *)stage_chunk(cx.stage, cx.lane, c) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (nch && row < p.M) p.stat[(size_t)(cx.col0 >> 7) * p.M + row] = make_float2(s, q);
        __syncwarp();
        // 32 rows x nch 16-byte chunks; h8 is read once by fc2, so it leaves with an evict-first hint
        const int ub0 = cx.col0 >> 1;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int pc = i * 32 + cx.lane, r = pc >> 2, ch = pc & 3;
            const int rw = cx.row0 + r;
            if (ch < nch && rw < p.M)
                __stcs((uint4 *)(p.h8 + (size_t)rw * HIDP + ub0 + 16 * ch), *(const uint4 *)stage_chunk(cx.stage, r, ch));
        }
        __syncwarp();
    }
};

// ---- fc2 with the MLP LayerNorm folded in: x += rstd * (acc - mean * c) + d ----
// mean / rstd over the 2730 SwiGLU units from fc1's NSTAT partials of the row, summed in a fixed order.
struct EpiFC2 {
    struct Params {
        __half *x;
        const float2 *stat;
        const float *c, *d;
        int M;
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
        const int row = cx.row0 + cx.lane;
        float s = 0.f, q = 0.f;
        if (row < p.M) {
#pragma unroll 4
            for (int g = 0; g < NSTAT; g++) {
                const float2 v = p.stat[(size_t)g * p.M + row];
                s += v.x;
                q += v.y;
            }
        }
        const float mean = s * (1.0f / HID);
        const float rstd = rsqrtf(q * (1.0f / HID) - mean * mean + 1e-6f);
        const float nb = -mean * rstd;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            __syncwarp();
            stage_row_f32(cx.stage, cx.lane, acc + 32 * c);
            __syncwarp();
            const int w = (cx.lane & 15) * 2;
            const int col = cx.col0 + 32 * c + w;
            const float2 c2 = *(const float2 *)(p.c + col), d2 = *(const float2 *)(p.d + col);
#pragma unroll 4
            for (int i = 0; i < 16; i++) {
                const int r = 2 * i + (cx.lane >> 4), rw = cx.row0 + r;
                const float rs = __shfl_sync(0xffffffffu, rstd, r), bb = __shfl_sync(0xffffffffu, nb, r);
                if (rw < p.M) {
                    __half2 *xp = (__half2 *)(p.x + (size_t)rw * D + col);
                    const float2 a = stage_f32x2(cx.stage, r, w);
                    const float2 xf = __half22float2(*xp);
                    *xp = __floats2half2_rn(xf.x + rs * a.x + bb * c2.x + d2.x, xf.y + rs * a.y + bb * c2.y + d2.y);
                }
            }
        }
        __syncwarp();
    }
};

// ---- patch embedding (fp16 GEMM, no block scales): rows are patches (img * 1024 + p) ----
// x[img * 1025 + 1 + p][col] = fp16(fp16(acc) + pos[1 + p][col]); the image's cls row gets fp16(pos[0][col]).
struct EpiPatch {
    struct Params {
        __half *x;
        const float *pos;
        int M;  // patch rows = images * 1024
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            __syncwarp();
            stage_row_f32(cx.stage, cx.lane, acc + 32 * c);
            __syncwarp();
            const int w = (cx.lane & 15) * 2;
            const int col = cx.col0 + 32 * c + w;
#pragma unroll 4
            for (int i = 0; i < 16; i++) {
                const int r = 2 * i + (cx.lane >> 4), rw = cx.row0 + r;
                if (rw < p.M) {
                    const int b = rw >> 10, pp = rw & 1023;
                    const float2 a = stage_f32x2(cx.stage, r, w);
                    const float2 ps = *(const float2 *)(p.pos + (size_t)(1 + pp) * D + col);
                    const float2 ah = __half22float2(__floats2half2_rn(a.x, a.y));
                    *(__half2 *)(p.x + ((size_t)b * T + 1 + pp) * D + col) = __floats2half2_rn(ah.x + ps.x, ah.y + ps.y);
                    if (pp == 0) {
                        const float2 p0 = *(const float2 *)(p.pos + col);
                        *(__half2 *)(p.x + (size_t)b * T * D + col) = __floats2half2_rn(p0.x, p0.y);
                    }
                }
            }
        }
        __syncwarp();
    }
};

// ---- tag head with the weights as the M operand: thread row = tag, columns = images ----
// out[img][tag] = sigmoid(acc + bias[tag]) for tag < nt, img < nimg.
template <int COLS>
struct EpiHead {
    struct Params {
        float *out;
        const float *hb;
        int nt, nimg;
    };
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx)
    {
        const int tag = cx.row0 + cx.lane;
        if (tag >= p.nt) return;
        const float bias = p.hb[tag];
#pragma unroll
        for (int j = 0; j < COLS; j++) {
            const int b = cx.col0 + j;
            if (b < p.nimg) p.out[(size_t)b * p.nt + tag] = 1.0f / (1.0f + __expf(-(acc[j] + bias)));
        }
    }
};

}  // namespace xtb

// Fused GEMM epilogues of the EVA02-L forward (calling convention in gemm.cuh; the CTA-pair GEMM of gemm2.cuh
// calls them the same way). Each one replaces a reference kernel's epilogue, written for the tcgen05 GEMM's
// one-row-per-thread accumulator layout:
//   EpiQKV    <- k_qkv   (eva_kernels.cu:41-114):  RoPE on q / k of patch tokens, E4M3, attention layouts
//   EpiResid  <- k_oproj (eva_kernels.cu:134-162): fp16 residual += acc, as a TMA reduce-add into x
//   EpiFC1    <- k_fc1   (eva_kernels.cu:211-279): SwiGLU, per-row LN statistics partials, E4M3 h (TMA store)
//   EpiFC2    <- k_fc2   (eva_kernels.cu:286-334): inner MLP LayerNorm folded in, TMA reduce-add into x
//   EpiPatch  <- k_pe + k_embed (eva_kernels.cu:21-33, 126-130): patch embedding + position / cls rows
//   EpiHead   <- k_headmv (kern_common.cuh:695-727): logits + bias -> sigmoid, weights as the M operand
// The residual updates are asynchronous bulk reductions (cp.reduce.async.bulk.tensor .add on the fp16 residual):
// the epilogue writes fp16(delta) to shared memory and the TMA unit performs x = fp16(x + fp16(delta)) in L2, so
// no epilogue thread waits on a load of x. Against the reference's x = fp16(x + delta) this rounds delta to fp16
// first: at most half an fp16 ulp of delta, far below an ulp of x.
#pragma once
#include "gemm2.cuh"
#include "ops.h"

namespace xtb {

// (mean, rstd) over the 2730 SwiGLU units of a row from fc1's NSTAT partial (sum, sum of squares) pairs, four threads
// per row (lanes 4 i .. 4 i + 3 of a warp: `row`, part j = lane & 3): part j adds partials j, j + 4, ... in order, and
// the four part sums are combined as (t0 + t1) + (t2 + t3) by two butterfly shuffles. Addition commutes, so every lane
// of the four gets the same bits: a fixed order, whatever the schedule. All 32 lanes of the warp must call it.
// (mean, rstd) of a row from its sums of u and u^2 over the HID units, every operation rounded explicitly so that
// each place that computes it (k_rowstat, the fc2 epilogue, the allocation-free fc2) gets the same bits.
__device__ __forceinline__ float2 rowstat_final(float s, float q)
{
    const float mean = __fmul_rn(s, 1.0f / HID);
    return make_float2(mean, rsqrtf(__fadd_rn(__fsub_rn(__fmul_rn(q, 1.0f / HID), __fmul_rn(mean, mean)), 1e-6f)));
}
__device__ __forceinline__ float2 rowstat_of(const float2 *__restrict__ stat, int rows, int row, int j)
{
    float s = 0.f, q = 0.f;
    if (row < rows) {
#pragma unroll
        for (int g = j; g < NSTAT; g += 4) {
            const float2 v = stat[(size_t)g * rows + row];
            s += v.x;
            q += v.y;
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    q += __shfl_xor_sync(0xffffffffu, q, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    q += __shfl_xor_sync(0xffffffffu, q, 2);
    return rowstat_final(s, q);
}
constexpr int ROWSTAT_THREADS = 256;  // 64 rows per block
__host__ __device__ constexpr int rowstat_blocks(int rows) { return (rows * 4 + ROWSTAT_THREADS - 1) / ROWSTAT_THREADS; }


// ---- QKV projection: acc = x W_qkv^T (dequantised); columns [0,1024) q, [1024,2048) k, [2048,3072) v ----
// q, k: scaled by cq / ck, interleaved RoPE (pair (2j, 2j+1) of a head shares angle j, table cs[t - 1][j] =
// (cos, sin)) for patch tokens t >= 1; v: scaled by cv. E4M3 -> q8 / k8 / v8 [img][head][TP][64] (row t of 64
// dims; the attention reads V as an MN-major operand, so no transpose). Rows t >= 1025 stay zero.
struct EpiQKV {
    struct Params {
        uint8_t *q8, *k8, *v8;
        const float2 *cs;
        float cq, ck, cv;
        int M;
    };
    using State = NoState;
    // 8 KB of staging per warp on the pair GEMM: both halves of the RoPE angles (4 KB each) are brought in when the
    // tile starts, so no angle load waits in the apply phase; the first 4 KB are reused for the output rows
    static constexpr int STAGING_PER_WARP = 8192;
    // cq / ck / cv ride along with the block-scale promotion, so acc arrives already scaled
    __device__ __forceinline__ static float col_scale(const Params &p, const EpiCtx &cx)
    {
        const int which = cx.col0 >> 10;
        return which == 0 ? p.cq : which == 1 ? p.ck : p.cv;
    }
    // The RoPE angles of the warp's 32 rows (256 bytes each) are brought in through the staging buffer with
    // coalesced loads, half a row (16 pairs) at a time into 4 KB each: rows t of one warp are consecutive in the
    // table, so each load instruction covers 4 whole 128-byte lines instead of 32 lines touched by one lane each.
    __device__ __forceinline__ static void stage_angles(const Params &p, const EpiCtx &cx, int h)
    {
        uint8_t *st = cx.stage + h * 4096;
        const int t0 = cx.row0 % T;
        float4 vv[8];  // all loads first, then the staging stores
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = 4 * i + (cx.lane >> 3), c = cx.lane & 7;
            int tt = t0 + r;
            if (tt >= T) tt -= T;
            float4 v = make_float4(1.f, 0.f, 1.f, 0.f);  // cls rows and rows past M: identity
            if (tt > 0 && cx.row0 + r < p.M) v = __ldg((const float4 *)(p.cs + (size_t)(tt - 1) * 32 + 16 * h) + c);
            vv[i] = v;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) *(float4 *)stage_chunk(st, 4 * i + (cx.lane >> 3), cx.lane & 7) = vv[i];
    }
    // Both halves are staged before the accumulator is built (the staging buffer is free between tiles: the
    // previous tile's stores read it synchronously), so those loads overlap the main loop.
    __device__ __forceinline__ static void begin(const Params &p, const EpiCtx &cx, State &)
    {
        if ((cx.col0 >> 10) < 2) {
            stage_angles(p, cx, 0);
            stage_angles(p, cx, 1);
        }
    }
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
        const int which = cx.col0 >> 10;           // 0 q, 1 k, 2 v (a thread's 128 columns never straddle)
        const int head0 = (cx.col0 & 1023) >> 6;   // two heads per thread
        uint4 o[2][4];                             // E4M3 output: head hh, dims 16 q .. 16 q + 15
        if (which == 2) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float *a = acc + hh * 64 + 16 * q;
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) w[e] = e4m3x2(a[4 * e], a[4 * e + 1]) | (e4m3x2(a[4 * e + 2], a[4 * e + 3]) << 16);
                    o[hh][q] = make_uint4(w[0], w[1], w[2], w[3]);
                }
        } else {
            __syncwarp();
#pragma unroll
            for (int h = 0; h < 2; h++) {          // pairs 16 h .. 16 h + 15 (staged by begin)
#pragma unroll
                for (int q2 = 0; q2 < 2; q2++) {   // 8 pairs (16 dims of each head) per step
                    float4 a[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) a[e] = *(const float4 *)stage_chunk(cx.stage + h * 4096, cx.lane, 4 * q2 + e);
                    const int j = 16 * h + 8 * q2;
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            float2 f[2];
#pragma unroll
                            for (int u = 0; u < 2; u++) {
                                // (f0, f1) -> (f0 cos - f1 sin, f1 cos + f0 sin) as two packed ops
                                const float cosv = u ? a[e >> 1].z : a[e >> 1].x, sinv = u ? a[e >> 1].w : a[e >> 1].y;
                                const float f0 = acc[hh * 64 + 2 * (j + e + u)], f1 = acc[hh * 64 + 2 * (j + e + u) + 1];
                                f[u] = fma2(make_float2(f1, f0), make_float2(-sinv, sinv), mul2(make_float2(f0, f1), make_float2(cosv, cosv)));
                            }
                            w[e >> 1] = e4m3x2(f[0].x, f[0].y) | (e4m3x2(f[1].x, f[1].y) << 16);
                        }
                        o[hh][2 * h + q2] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
        __syncwarp();
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
#pragma unroll
            for (int q = 0; q < 4; q++) *(uint4 *)stage_chunk(cx.stage, cx.lane, 4 * hh + q) = o[hh][q];
        __syncwarp();
        uint8_t *dst = which == 0 ? p.q8 : which == 1 ? p.k8 : p.v8;
        uint4 pieces[8];  // all staged pieces first, then the stores (see EpiF32::apply)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int pc = i * 32 + cx.lane;          // piece: head hh, row r, 16-byte chunk ch
            pieces[i] = *(const uint4 *)stage_chunk(cx.stage, (pc >> 2) & 31, 4 * (pc >> 7) + (pc & 3));
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int pc = i * 32 + cx.lane;
            const int hh = pc >> 7, r = (pc >> 2) & 31, ch = pc & 3;
            const int rw = cx.row0 + r;
            if (rw < p.M) {
                const int bb = rw / T, tt = rw - bb * T;
                *(uint4 *)(dst + (((size_t)(bb * NH + head0 + hh) * TP + tt) << 6) + ch * 16) = pieces[i];
            }
        }
        __syncwarp();
    }
};

// ---- fp16 residual update (attention out-projection): x[row][col] += acc, by TMA reduce-add ----
// 64-column rounds: the warp's 32 rows x 64 fp16 deltas (4 KB, 128B-swizzled like the x tensor map's box) go out
// as one cp.reduce.async.bulk.tensor.
template <class F>
__device__ __forceinline__ void reduce_add_rows(const EpiCtx &cx, int M, int col, F delta)
{
    if (cx.lane == 0) bulk_wait_read0();  // the previous round's source has been read
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; c++) {
        __half2 h[4];
#pragma unroll
        for (int e = 0; e < 4; e++) h[e] = __floats2half2_rn(delta(8 * c + 2 * e), delta(8 * c + 2 * e + 1));
        *(uint4 *)stage_chunk(cx.stage, cx.lane, c) = *(const uint4 *)h;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (cx.lane == 0 && cx.row0 < M) {
        tma_reduce_add_2d(cx.tmC, cx.stage, col, cx.row0);
        bulk_commit();
    }
}

struct EpiResid {
    struct Params {
        int M;
    };
    using State = NoState;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
#pragma unroll
        for (int rd = 0; rd < 2; rd++) reduce_add_rows(cx, p.M, cx.col0 + 64 * rd, [&](int j) { return acc[64 * rd + j]; });
    }
};

// ---- fc1 + SwiGLU: W12 rows interleave g / x in 16-unit chunks (32 columns = units 16c .. 16c + 15) ----
// u = x * g * sigmoid(g) (sigmoid(g) = 0.5 (1 + tanh(g / 2)), as the reference), h8 = E4M3(u * rs[unit]),
// stat[col0 / 128][row] = (sum u, sum u^2) over this thread's 64 units (each partial has exactly one writer).
// h8 leaves through a TMA store of the warp's 32 rows x 64 units (64-byte rows, 64B swizzle).
struct EpiFC1 {
    struct Params {
        float2 *stat;
        const float *rs;
        int M;
    };
    using State = NoState;
    static constexpr int STAGING_PER_WARP = 2048;  // 32 rows x 64 units of E4M3
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
        const int row = cx.row0 + cx.lane;
        if (cx.col0 >= N12) return;  // warp-uniform: this half of the last tile is past the units
        float2 s2 = make_float2(0.f, 0.f), q2 = make_float2(0.f, 0.f);
        if (cx.lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int n = cx.col0 + 32 * c;
            if (n >= N12) break;
            const int ub = n >> 1;
            const float4 *rs4 = (const float4 *)(p.rs + ub);
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                const float4 r4 = __ldg(rs4 + (i >> 2));
                float2 hq[2];
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                    // u = x * (g/2) (1 + tanh(g/2)) on pairs of units
                    const float2 hg = mul2(make_float2(acc[32 * c + i + e], acc[32 * c + i + e + 1]), make_float2(0.5f, 0.5f));
                    const float2 th = make_float2(tanh_fast(hg.x), tanh_fast(hg.y));
                    const float2 u = mul2(make_float2(acc[32 * c + 16 + i + e], acc[32 * c + 16 + i + e + 1]), fma2(hg, th, hg));
                    s2 = add2(s2, u);
                    q2 = fma2(u, u, q2);
                    hq[e >> 1] = mul2(u, e ? make_float2(r4.z, r4.w) : make_float2(r4.x, r4.y));
                }
                w[i >> 2] = e4m3x2(hq[0].x, hq[0].y) | (e4m3x2(hq[1].x, hq[1].y) << 16);
            }
            *(uint4 *)(cx.stage + cx.lane * 64 + ((c ^ ((cx.lane >> 1) & 3)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (row < p.M) p.stat[(size_t)(cx.col0 >> 7) * p.M + row] = make_float2(s2.x + s2.y, q2.x + q2.y);
        fence_proxy_async_smem();
        __syncwarp();
        if (cx.lane == 0 && cx.row0 < p.M) {
            tma_store_2d(cx.tmC, cx.stage, cx.col0 >> 1, cx.row0);
            bulk_commit();
        }
    }
};

// ---- fc2 with the MLP LayerNorm folded in: x += rstd * (acc - mean * c) + d, by TMA reduce-add ----
// (mean, rstd) of the row over the 2730 SwiGLU units come from k_rowstat, which folds fc1's partials in a fixed
// order into stat[0][row]; the load is issued when the tile starts.
struct EpiFC2 {
    struct Params {
        const float2 *ms;    // per-row (mean, rstd), or
        const float2 *part;  // when not null: fc1's NSTAT partials [NSTAT][M], summed here
        const float *c, *d;
        int M;
    };
    struct State {
        float2 ms;
    };
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    // The thread's row statistics, before the accumulator is ready: either loaded, or summed from the partials in
    // the order of rowstat_of (partials j, j + 4, ... into sum j, then (s0 + s1) + (s2 + s3)), which gives the same
    // bits as k_rowstat without its launch. Each load covers 32 consecutive rows (256 bytes) across the warp.
    __device__ __forceinline__ static void begin(const Params &p, const EpiCtx &cx, State &st)
    {
        const int row = cx.row0 + cx.lane;
        if (row >= p.M) {
            st.ms = make_float2(0.f, 1.f);
        } else if (!p.part) {
            st.ms = p.ms[row];
        } else {
            float s[4] = {0.f, 0.f, 0.f, 0.f}, q[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 3
            for (int g0 = 0; g0 < NSTAT; g0 += 4) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (g0 + j < NSTAT) {
                        const float2 v = __ldg(p.part + (size_t)(g0 + j) * p.M + row);
                        s[j] += v.x;
                        q[j] += v.y;
                    }
                }
            }
            st.ms = rowstat_final((s[0] + s[1]) + (s[2] + s[3]), (q[0] + q[1]) + (q[2] + q[3]));
        }
    }
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &st)
    {
        const float rstd = st.ms.y, nb = -st.ms.x * st.ms.y;
#pragma unroll
        for (int rd = 0; rd < 2; rd++) {
            const int col = cx.col0 + 64 * rd;
            reduce_add_rows(cx, p.M, col, [&](int j) {
                return fmaf(rstd, acc[64 * rd + j], fmaf(nb, __ldg(p.c + col + j), __ldg(p.d + col + j)));
            });
        }
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
    using State = NoState;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            __syncwarp();
            stage_row_f32(cx.stage, cx.lane, acc + 32 * c);
            __syncwarp();
            const int w = (cx.lane & 15) * 2;
            const int col = cx.col0 + 32 * c + w;
            // two rounds of eight row pairs: each round's staged values and position rows are all loaded before its
            // stores, so eight position loads (L2) are in flight at a time and each round waits out one latency
#pragma unroll 1
            for (int h = 0; h < 2; h++) {
                float2 sv[8], ps[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int r = 2 * (8 * h + i) + (cx.lane >> 4), rw = cx.row0 + r;
                    sv[i] = stage_f32x2(cx.stage, r, w);
                    ps[i] = rw < p.M ? __ldg((const float2 *)(p.pos + (size_t)(1 + (rw & 1023)) * D + col))
                                     : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int r = 2 * (8 * h + i) + (cx.lane >> 4), rw = cx.row0 + r;
                    if (rw < p.M) {
                        const int b = rw >> 10, pp = rw & 1023;
                        const float2 ah = __half22float2(__floats2half2_rn(sv[i].x, sv[i].y));
                        *(__half2 *)(p.x + ((size_t)b * T + 1 + pp) * D + col) =
                            __floats2half2_rn(ah.x + ps[i].x, ah.y + ps[i].y);
                        if (pp == 0) {
                            const float2 p0 = __ldg((const float2 *)(p.pos + col));
                            *(__half2 *)(p.x + (size_t)b * T * D + col) = __floats2half2_rn(p0.x, p0.y);
                        }
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
    using State = NoState;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
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

// PixAI tagger (ViTDet-L at 1008^2) kernels: the GEMM epilogues of its block projections and its row / head
// kernels, for the tcgen05 GEMMs of gemm.cuh / gemm2.cuh and the attention of attention.cuh. Each replaces a
// reference kernel of src/engine/px_kernels.cu, written for this library's one-row-per-thread accumulators:
//   EpiPxPatch   <- k_ppe (patch_gemm<0>, kern_common.cuh:361-387): x = fp16(in . pe^T), window-major rows
//   k_px_embed   <- k_pembed (px_kernels.cu:16-52): x = LN_pre(x + pos[t]), eps 1e-5
//   EpiPxQKV     <- k_pqkv (px_kernels.cu:60-129): bias, cq / ck / cv, RoPE on every token (table row m % L), E4M3,
//                   q8 / k8 / v8 [sequence][16][L][64]
//   EpiPxResid   <- resgemm (px_kernels.cu:157-187): x += acc + bias, as a TMA reduce-add into the fp16 residual
//   EpiPxFC1     <- k_pfc1 (px_kernels.cu:203-239): bias, exact-erf GELU, * rs, E4M3 (TMA store)
//   k_px_head_*  <- k_phln / k_phscore / k_phsoft / k_phpool / k_phv (px_kernels.cu:347-503): attention-pool head
// Tokens are window-major throughout (9 windows of 576); windowed blocks attend within 576-token sequences, global
// blocks over all 5184 tokens of an image.
#pragma once
#include "attention.cuh"
#include "epilogues.cuh"
#include "ops.h"

namespace xtb {

constexpr int PX_T = 5184, PX_LW = 576, PX_HID = 4736, PX_QKV = 3 * D;
constexpr int PX_PCH = 144;                   // attention-pool token chunk
constexpr int PX_NCH = PX_T / PX_PCH;         // 36 chunks per image
constexpr float PX_EPS = 1e-5f;               // ln_pre and the head LayerNorm (px_kernels.cu:44, 376)

// ---- patch embedding (fp16 GEMM): x[row][col] = fp16(acc), rows = image * 5184 + window-major patch ----
struct EpiPxPatch {
    struct Params {
        __half *x;
        int M;
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
            float2 sv[16];  // all staged values first, then the stores (see EpiF32::apply)
#pragma unroll
            for (int i = 0; i < 16; i++) sv[i] = stage_f32x2(cx.stage, 2 * i + (cx.lane >> 4), w);
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int rw = cx.row0 + 2 * i + (cx.lane >> 4);
                if (rw < p.M) *(__half2 *)(p.x + (size_t)rw * D + col) = __floats2half2_rn(sv[i].x, sv[i].y);
            }
        }
        __syncwarp();
    }
};

// ---- QKV projection: acc = alpha h Wqkv^T; columns [0,1024) q, [1024,2048) k, [2048,3072) v ----
// f = (acc + bias) * cq / ck / cv; q, k: interleaved RoPE (pair (2j, 2j+1) of a head by angle j of cs[t][j]) with
// t = row % L on every token; E4M3 -> [s][head][L][64] with s = row / L.
struct EpiPxQKV {
    struct Params {
        uint8_t *q8, *k8, *v8;
        const float2 *cs;
        const float *bias;
        float cq, ck, cv;
        int M, L;
    };
    using State = NoState;
    static constexpr int STAGING_PER_WARP = 8192;  // both halves of the angles (4 KB each)
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    // The angles of the warp's 32 rows, half a row (16 pairs) at a time into 4 KB: consecutive rows are consecutive
    // table rows (wrapping at L), so each load instruction covers 4 whole 128-byte lines.
    __device__ __forceinline__ static void stage_angles(const Params &p, const EpiCtx &cx, int h)
    {
        uint8_t *st = cx.stage + h * 4096;
        const int t0 = cx.row0 % p.L;
        float4 vv[8];  // all loads first, then the staging stores
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = 4 * i + (cx.lane >> 3), c = cx.lane & 7;
            int tt = t0 + r;
            if (tt >= p.L) tt -= p.L;
            float4 v = make_float4(1.f, 0.f, 1.f, 0.f);  // rows past M: identity
            if (cx.row0 + r < p.M) v = __ldg((const float4 *)(p.cs + (size_t)tt * 32 + 16 * h) + c);
            vv[i] = v;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) *(float4 *)stage_chunk(st, 4 * i + (cx.lane >> 3), cx.lane & 7) = vv[i];
    }
    __device__ __forceinline__ static void begin(const Params &p, const EpiCtx &cx, State &)
    {
        if ((cx.col0 >> 10) < 2) {
            stage_angles(p, cx, 0);
            stage_angles(p, cx, 1);
        }
    }
    // A streaming epilogue: chunk c (32 columns) is dims 32 (c & 1) .. + 31 of head head0 + (c >> 1); its 32 E4M3
    // bytes go straight to the row's 64-byte line of q8 / k8 / v8 (consecutive lanes are consecutive tokens, so a
    // warp's stores cover whole lines of one head), and the angle rows stay staged for every chunk.
    static constexpr bool STREAM = true;
    __device__ __forceinline__ static void apply_chunk(const Params &p, const float *v, float s, int c,
                                                       const EpiCtx &cx, State &)
    {
        const int which = cx.col0 >> 10;           // 0 q, 1 k, 2 v (a thread's 128 columns never straddle)
        const int hh = c >> 1, h = c & 1;          // head within the thread's two, half of its 64 dims
        const int n0 = hh * 64 + 32 * h;           // first column of the chunk within the thread's 128
        const float sc = which == 0 ? p.cq : which == 1 ? p.ck : p.cv;
        const float2 s2 = make_float2(s, s), sc2 = make_float2(sc, sc);
        const float4 *bq = (const float4 *)(p.bias + cx.col0 + n0);
        uint32_t w[8];
        if (which == 2) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float4 b4 = __ldg(bq + e);
                const float2 f0 = mul2(fma2(make_float2(v[4 * e], v[4 * e + 1]), s2, make_float2(b4.x, b4.y)), sc2);
                const float2 f1 = mul2(fma2(make_float2(v[4 * e + 2], v[4 * e + 3]), s2, make_float2(b4.z, b4.w)), sc2);
                w[e] = e4m3x2(f0.x, f0.y) | (e4m3x2(f1.x, f1.y) << 16);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {           // pairs 16 h + 2 e, 16 h + 2 e + 1 (dims 4 e .. 4 e + 3)
                const float4 b4 = __ldg(bq + e);
                const float4 a = *(const float4 *)stage_chunk(cx.stage + h * 4096, cx.lane, e);  // (cos, sin) x 2
                float2 f[2];
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const float cosv = u ? a.z : a.x, sinv = u ? a.w : a.y;
                    const float2 fb = mul2(fma2(make_float2(v[4 * e + 2 * u], v[4 * e + 2 * u + 1]), s2,
                                                u ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y)), sc2);
                    // (f0, f1) -> (f0 cos - f1 sin, f1 cos + f0 sin)
                    f[u] = fma2(make_float2(fb.y, fb.x), make_float2(-sinv, sinv), mul2(fb, make_float2(cosv, cosv)));
                }
                w[e] = e4m3x2(f[0].x, f[0].y) | (e4m3x2(f[1].x, f[1].y) << 16);
            }
        }
        const int rw = cx.row0 + cx.lane;
        if (rw < p.M) {
            uint8_t *dst = which == 0 ? p.q8 : which == 1 ? p.k8 : p.v8;
            const int sq = rw / p.L, tt = rw - sq * p.L;
            const int head = ((cx.col0 & 1023) >> 6) + hh;
            uint4 *o = (uint4 *)(dst + ((((size_t)sq * NH + head) * p.L + tt) << 6) + 32 * h);
            o[0] = make_uint4(w[0], w[1], w[2], w[3]);
            o[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
    __device__ __forceinline__ static void finish(const Params &, const EpiCtx &, State &) { __syncwarp(); }
    // the non-streaming call (a block-scaled weight): acc arrives dequantised, 128 columns
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &st)
    {
#pragma unroll
        for (int c = 0; c < 4; c++) apply_chunk(p, acc + 32 * c, 1.0f, c, cx, st);
    }
};

// ---- residual update with bias (attention out-projection, fc2): x += acc + bias, by TMA reduce-add ----
struct EpiPxResid {
    struct Params {
        const float *bias;
        int M;
    };
    using State = NoState;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
#pragma unroll
        for (int rd = 0; rd < 2; rd++) {
            const int col = cx.col0 + 64 * rd;
            reduce_add_rows(cx, p.M, col, [&](int j) { return acc[64 * rd + j] + __ldg(p.bias + col + j); });
        }
    }
};

// Exact-erf GELU, v (1 + erf(v / sqrt 2)) / 2, with erf from Abramowitz & Stegun 7.1.26 (Handbook of Mathematical
// Functions, 1964): erf(x) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^(-x^2), t = 1 / (1 + p x), x >= 0,
// absolute error below 1.5e-7. With hq = (1 - erf(|z|)) / 2 (the coefficients carry the 1/2), z = v / sqrt 2:
// gelu = v - v hq for v >= 0 and v hq for v < 0, so the small tail is computed without cancellation. The result
// feeds an E4M3 code (3 mantissa bits), so this matches the reference's erff-based value except where the two sit
// within ~1e-7 of a rounding boundary. Two elements at a time on packed f32x2 operations; two MUFU operations (rcp,
// ex2) per element.
__device__ __forceinline__ float2 gelu_erf2(float2 v)
{
    constexpr float P = 0.3275911f, A1 = 0.5f * 0.254829592f, A2 = 0.5f * -0.284496736f, A3 = 0.5f * 1.421413741f,
                    A4 = 0.5f * -1.453152027f, A5 = 0.5f * 1.061405429f;
    const float2 az = mul2(make_float2(fabsf(v.x), fabsf(v.y)), make_float2(0.70710678f, 0.70710678f));
    const float2 d = fma2(az, make_float2(P, P), make_float2(1.0f, 1.0f));
    float2 t;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.y) : "f"(d.y));
    float2 poly = fma2(t, make_float2(A5, A5), make_float2(A4, A4));
    poly = fma2(t, poly, make_float2(A3, A3));
    poly = fma2(t, poly, make_float2(A2, A2));
    poly = fma2(t, poly, make_float2(A1, A1));
    poly = mul2(t, poly);
    const float2 arg = mul2(mul2(az, make_float2(-1.44269504f, -1.44269504f)), az);
    const float2 e = make_float2(ex2(arg.x), ex2(arg.y));
    const float2 g = mul2(v, mul2(poly, e));   // v hq
    return make_float2(v.x >= 0.0f ? v.x - g.x : g.x, v.y >= 0.0f ? v.y - g.y : g.y);
}

// ---- fc1 + GELU: u8 = E4M3(rs * gelu(acc + b1)), gelu(v) = v (1 + erf(v / sqrt 2)) / 2 ----
// A streaming epilogue: each 32-column chunk of the accumulator is turned into 32 E4M3 bytes of the warp's staging
// rows as soon as its TMEM load lands; the warp's 32 rows x 128 units then leave through one TMA store (128-byte
// rows, 128B swizzle: the staging layout).
struct EpiPxFC1 {
    struct Params {
        const float *b1, *rs;
        int M;
    };
    using State = NoState;
    static constexpr bool STREAM = true;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &cx, State &)
    {
        if (cx.lane == 0) bulk_wait_read0();  // the previous tile's store has read the staging rows
        __syncwarp();
    }
    __device__ __forceinline__ static void apply_chunk(const Params &p, const float *v, float s, int c,
                                                       const EpiCtx &cx, State &)
    {
        if (cx.col0 >= PX_HID) return;  // warp-uniform: the half of the last tile past the units
        const float4 *b4p = (const float4 *)(p.b1 + cx.col0 + 32 * c), *r4p = (const float4 *)(p.rs + cx.col0 + 32 * c);
        const float2 s2 = make_float2(s, s);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float4 b4 = __ldg(b4p + 4 * h + e), r4 = __ldg(r4p + 4 * h + e);
                const float *a = v + 16 * h + 4 * e;
                const float2 g0 = mul2(gelu_erf2(fma2(make_float2(a[0], a[1]), s2, make_float2(b4.x, b4.y))),
                                       make_float2(r4.x, r4.y));
                const float2 g1 = mul2(gelu_erf2(fma2(make_float2(a[2], a[3]), s2, make_float2(b4.z, b4.w))),
                                       make_float2(r4.z, r4.w));
                w[e] = e4m3x2(g0.x, g0.y) | (e4m3x2(g1.x, g1.y) << 16);
            }
            *(uint4 *)stage_chunk(cx.stage, cx.lane, 2 * c + h) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    __device__ __forceinline__ static void finish(const Params &p, const EpiCtx &cx, State &)
    {
        if (cx.col0 >= PX_HID) return;
        fence_proxy_async_smem();
        __syncwarp();
        if (cx.lane == 0 && cx.row0 < p.M) {
            tma_store_2d(cx.tmC, cx.stage, cx.col0, cx.row0);
            bulk_commit();
        }
    }
    // the non-streaming call (a block-scaled weight): acc arrives dequantised, 128 columns
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &st)
    {
#pragma unroll
        for (int c = 0; c < 4; c++) apply_chunk(p, acc + 32 * c, 1.0f, c, cx, st);
        finish(p, cx, st);
    }
};

// ---- row kernels: one warp per row, 8 rows per 256-thread block; lane holds columns 4 (lane + 32 j), j < 8 ----
__device__ __forceinline__ void px_load_row(const __half *xr, int lane, float *v)
{
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint2 u = __ldg((const uint2 *)(xr + 4 * (lane + 32 * j)));
        const float2 a = __half22float2(*(const __half2 *)&u.x), b = __half22float2(*(const __half2 *)&u.y);
        v[4 * j] = a.x;
        v[4 * j + 1] = a.y;
        v[4 * j + 2] = b.x;
        v[4 * j + 3] = b.y;
    }
}

// mean and 1 / sqrt(var + eps) of a row held across the warp (two passes, as the reference's ln_row)
__device__ __forceinline__ void px_row_stats(const float *v, float eps, float *mean, float *rstd)
{
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) s += v[i];
    const float m = warp_sum(s) * (1.0f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const float d = v[i] - m;
        q = fmaf(d, d, q);
    }
    *mean = m;
    *rstd = rsqrtf(warp_sum(q) * (1.0f / D) + eps);
}

// x = fp16(LN_pre(x + pos[row % 5184]) * w + b), in place
__global__ void __launch_bounds__(256) k_px_embed(__half *__restrict__ x, const float *__restrict__ pos,
                                                  const float *__restrict__ w, const float *__restrict__ b, int rows)
{
    griddep_wait();  // the previous kernel of the stream has completed
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    __half *xr = x + (size_t)row * D;
    const float *pr = pos + (size_t)(row % PX_T) * D;
    float v[32], mean, rstd;
    px_load_row(xr, lane, v);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 p4 = __ldg((const float4 *)(pr + 4 * (lane + 32 * j)));
        v[4 * j] += p4.x;
        v[4 * j + 1] += p4.y;
        v[4 * j + 2] += p4.z;
        v[4 * j + 3] += p4.w;
    }
    px_row_stats(v, PX_EPS, &mean, &rstd);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int c = 4 * (lane + 32 * j);
        const float4 g = __ldg((const float4 *)(w + c)), bb = __ldg((const float4 *)(b + c));
        const __half2 h0 = __floats2half2_rn((v[4 * j] - mean) * rstd * g.x + bb.x, (v[4 * j + 1] - mean) * rstd * g.y + bb.y);
        const __half2 h1 = __floats2half2_rn((v[4 * j + 2] - mean) * rstd * g.z + bb.z, (v[4 * j + 3] - mean) * rstd * g.w + bb.w);
        uint2 u;
        u.x = *(const uint32_t *)&h0;
        u.y = *(const uint32_t *)&h1;
        *(uint2 *)(xr + c) = u;
    }
}

// Head LayerNorm + pool scores: y = fp16(LN(x) * w + b + hpos[t]) and s[row][h] = U[h] . y (the constant query
// folded into the key projection). U (64 KB fp32) sits in shared memory for the block's rows (grid-stride).
constexpr size_t PX_HEAD_SMEM = (size_t)NH * D * 4;
__global__ void __launch_bounds__(256) k_px_head_ln_score(const __half *__restrict__ x, const float *__restrict__ w,
                                                          const float *__restrict__ b, const __half *__restrict__ hpos,
                                                          const float *__restrict__ U, __half *__restrict__ y,
                                                          float *__restrict__ s, int rows)
{
    griddep_wait();  // the previous kernel of the stream has completed
    extern __shared__ float sU[];
    for (int i = threadIdx.x; i < NH * D / 4; i += 256) ((float4 *)sU)[i] = __ldg((const float4 *)U + i);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += gridDim.x * 8) {
        float v[32], mean, rstd;
        px_load_row(x + (size_t)row * D, lane, v);
        px_row_stats(v, PX_EPS, &mean, &rstd);
        const __half *hp = hpos + (size_t)(row % PX_T) * D;
        float hv[32];
        px_load_row(hp, lane, hv);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = 4 * (lane + 32 * j);
            const float4 g = __ldg((const float4 *)(w + c)), bb = __ldg((const float4 *)(b + c));
            const __half2 h0 = __floats2half2_rn((v[4 * j] - mean) * rstd * g.x + bb.x + hv[4 * j],
                                                 (v[4 * j + 1] - mean) * rstd * g.y + bb.y + hv[4 * j + 1]);
            const __half2 h1 = __floats2half2_rn((v[4 * j + 2] - mean) * rstd * g.z + bb.z + hv[4 * j + 2],
                                                 (v[4 * j + 3] - mean) * rstd * g.w + bb.w + hv[4 * j + 3]);
            uint2 u;
            u.x = *(const uint32_t *)&h0;
            u.y = *(const uint32_t *)&h1;
            *(uint2 *)(y + (size_t)row * D + c) = u;
            const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
            v[4 * j] = f0.x;
            v[4 * j + 1] = f0.y;
            v[4 * j + 2] = f1.x;
            v[4 * j + 3] = f1.y;
        }
        float part[NH];
#pragma unroll
        for (int h = 0; h < NH; h++) {
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 u4 = *(const float4 *)(sU + h * D + 4 * (lane + 32 * j));
                a = fmaf(v[4 * j], u4.x, a);
                a = fmaf(v[4 * j + 1], u4.y, a);
                a = fmaf(v[4 * j + 2], u4.z, a);
                a = fmaf(v[4 * j + 3], u4.w, a);
            }
            part[h] = a;
        }
        // 16 warp sums at once: halve the set of partials per butterfly step (lane bit k picks which half it keeps)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int n = NH >> (k + 1);
            const bool up = (lane >> k) & 1;
#pragma unroll
            for (int i = 0; i < n; i++) {
                const float send = up ? part[i] : part[i + n], keep = up ? part[i + n] : part[i];
                part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1 << k);
            }
        }
        // part[0] of lane l holds heads {bit-reversed low 4 bits of l} partial over lanes sharing bits 0..3
        float tot = part[0] + __shfl_xor_sync(0xffffffffu, part[0], 16);
        const int h = ((lane & 1) << 3) | ((lane & 2) << 1) | ((lane & 4) >> 1) | ((lane & 8) >> 3);
        if (lane < 16) s[(size_t)row * NH + h] = tot;
    }
}

// Pool weights: P[img][h][t] = fp16(exp2(s[t][h] - max) / sum), one block per (image, head)
__global__ void __launch_bounds__(256) k_px_head_softmax(const float *__restrict__ s, __half *__restrict__ P)
{
    griddep_wait();  // the previous kernel of the stream has completed
    __shared__ float red[8];
    const int img = blockIdx.x / NH, h = blockIdx.x % NH, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float *sb = s + (size_t)img * PX_T * NH + h;
    float m = -INFINITY;
    for (int t = threadIdx.x; t < PX_T; t += 256) m = fmaxf(m, sb[(size_t)t * NH]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wid] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < 8; i++) m = fmaxf(m, red[i]);
    __syncthreads();
    float l = 0.f;
    for (int t = threadIdx.x; t < PX_T; t += 256) l += exp2f(sb[(size_t)t * NH] - m);
    l = warp_sum(l);
    if (lane == 0) red[wid] = l;
    __syncthreads();
    l = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) l += red[i];
    const float li = 1.0f / l;
    for (int t = threadIdx.x; t < PX_T; t += 256)
        P[(size_t)blockIdx.x * PX_T + t] = __float2half_rn(exp2f(sb[(size_t)t * NH] - m) * li);
}

// Pool partial sums: part[img][c][h][n] = sum over the 144 tokens t of chunk c of P[img][h][t] y[t][n]. Grid
// (images, 36 chunks), 512 threads: one dimension pair each, all 16 heads at once, so y is read exactly once.
__global__ void __launch_bounds__(512) k_px_head_pool(const __half *__restrict__ P, const __half *__restrict__ y,
                                                      float *__restrict__ part)
{
    griddep_wait();  // the previous kernel of the stream has completed
    __shared__ __align__(16) float sp[PX_PCH][NH];
    const int img = blockIdx.x, c = blockIdx.y, t0 = c * PX_PCH;
    for (int i = threadIdx.x; i < PX_PCH * NH; i += 512) {
        const int h = i / PX_PCH, t = i % PX_PCH;
        sp[t][h] = __half2float(P[((size_t)img * NH + h) * PX_T + t0 + t]);
    }
    __syncthreads();
    float2 acc[NH];
#pragma unroll
    for (int h = 0; h < NH; h++) acc[h] = make_float2(0.f, 0.f);
    const __half2 *yr = (const __half2 *)(y + ((size_t)img * PX_T + t0) * D) + threadIdx.x;
    for (int t = 0; t < PX_PCH; t++) {
        const float2 v = __half22float2(yr[(size_t)t * (D / 2)]);
#pragma unroll
        for (int q = 0; q < NH / 4; q++) {
            const float4 p4 = *(const float4 *)&sp[t][4 * q];
            acc[4 * q] = fma2(make_float2(p4.x, p4.x), v, acc[4 * q]);
            acc[4 * q + 1] = fma2(make_float2(p4.y, p4.y), v, acc[4 * q + 1]);
            acc[4 * q + 2] = fma2(make_float2(p4.z, p4.z), v, acc[4 * q + 2]);
            acc[4 * q + 3] = fma2(make_float2(p4.w, p4.w), v, acc[4 * q + 3]);
        }
    }
    float *po = part + (((size_t)img * PX_NCH + c) * NH) * D + 2 * threadIdx.x;
#pragma unroll
    for (int h = 0; h < NH; h++) *(float2 *)(po + (size_t)h * D) = acc[h];
}

// o[img][n] = fp16(Wv[n] . pooled[img][n / 64]), pooled = the 36 chunk partials added in chunk order (the same sum
// every run). One block (256 threads) per (image, head): the 64 outputs of head h.
__global__ void __launch_bounds__(256) k_px_head_v(const float *__restrict__ part, const __half *__restrict__ wv,
                                                   __half *__restrict__ o)
{
    griddep_wait();  // the previous kernel of the stream has completed
    __shared__ __align__(16) float xs[D];
    const int img = blockIdx.x / NH, h = blockIdx.x % NH, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float *pv = part + ((size_t)img * PX_NCH * NH + h) * D;
    {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < PX_NCH; c++) {
            const float4 v = __ldg((const float4 *)(pv + (size_t)c * NH * D) + threadIdx.x);
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        }
        ((float4 *)xs)[threadIdx.x] = a;
    }
    __syncthreads();
    for (int k = 0; k < 8; k++) {
        const int n = 64 * h + 8 * wid + k;
        float a = 0.f;
        float v[32];
        px_load_row(wv + (size_t)n * D, lane, v);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 x4 = ((const float4 *)xs)[lane + 32 * j];
            a = fmaf(v[4 * j], x4.x, a);
            a = fmaf(v[4 * j + 1], x4.y, a);
            a = fmaf(v[4 * j + 2], x4.z, a);
            a = fmaf(v[4 * j + 3], x4.w, a);
        }
        a = warp_sum(a);
        if (lane == 0) o[(size_t)img * D + n] = __float2half_rn(a);
    }
}

}  // namespace xtb

// Memory-bound row kernels of the forward: LayerNorm + E4M3 quantisation of the GEMM inputs, mean pooling over
// patch tokens, and the fc_norm LayerNorm that produces the head input.
#pragma once
#include "ops.h"
#include "ptx.cuh"

namespace xtb {

// LayerNorm over 1024 fp16 values (eps 1e-6, two-pass mean / variance from registers), * gamma + beta, * qs,
// E4M3 with saturation. Replaces k_ln / ln_row<1> (kern_common.cuh:147-186), same arithmetic in the same order.
// Persistent warps: warp w of the grid takes rows w, w + W, ... and keeps LN_DEPTH of them in flight as 2 KB bulk
// copies (cp.async.bulk, completion on one mbarrier per slot) into its own shared-memory ring, so the HBM latency is
// covered by copies instead of by registers; gamma and beta of the lane's 32 columns stay in registers for all of
// the warp's rows. A lane reads the 16-byte chunks lane + 32 i of a row (conflict-free) and writes 8 bytes each.
constexpr int LN_WARPS = 8, LN_DEPTH = 4, LN_BLOCKS_PER_SM = 2;
constexpr int LN_SMEM = LN_WARPS * LN_DEPTH * D * 2 + LN_WARPS * LN_DEPTH * 8;

__global__ void __launch_bounds__(LN_WARPS * 32, LN_BLOCKS_PER_SM)
    k_ln_e4m3(const __half *__restrict__ x, const float *__restrict__ g, const float *__restrict__ bta,
              uint8_t *__restrict__ y, int rows, float qs, uint32_t *err)
{
    extern __shared__ __align__(128) uint8_t ln_smem[];
    const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *ring = ln_smem + wl * LN_DEPTH * D * 2;
    uint64_t *bar = (uint64_t *)(ln_smem + LN_WARPS * LN_DEPTH * D * 2) + wl * LN_DEPTH;
    const int W = gridDim.x * LN_WARPS;
    const int w0 = blockIdx.x * LN_WARPS + wl;
    if (lane == 0) {
        for (int s = 0; s < LN_DEPTH; s++) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    float gv[32], bv[32];  // gamma / beta are weights: loaded before the wait
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int c = 8 * (lane + 32 * i);
        *(float4 *)(gv + 8 * i) = __ldg((const float4 *)(g + c));
        *(float4 *)(gv + 8 * i + 4) = __ldg((const float4 *)(g + c + 4));
        *(float4 *)(bv + 8 * i) = __ldg((const float4 *)(bta + c));
        *(float4 *)(bv + 8 * i + 4) = __ldg((const float4 *)(bta + c + 4));
    }
    griddep_wait();  // the previous kernel of the stream has completed: x may be read, y written
    if (lane == 0) {
        for (int s = 0; s < LN_DEPTH; s++) {
            const int r = w0 + s * W;
            if (r < rows) {
                mbar_arrive_expect_tx(&bar[s], D * 2);
                bulk_load(ring + s * D * 2, x + (size_t)r * D, D * 2, &bar[s]);
            }
        }
    }
    __syncwarp();
    for (int k = 0, row = w0; row < rows; k++, row += W) {
        const int s = k % LN_DEPTH;
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], (k / LN_DEPTH) & 1, err, XTB_ERR_WAIT_TMA))) return;
        const uint4 *xr = (const uint4 *)(ring + s * D * 2);
        float v[32];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 u = xr[lane + 32 * i];
            const __half2 *hp = (const __half2 *)&u;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(hp[e]);
                v[8 * i + 2 * e] = f.x;
                v[8 * i + 2 * e + 1] = f.y;
                sum += f.x + f.y;
            }
        }
        // every lane has its row in registers: the slot goes back to the copy engine for row + LN_DEPTH * W
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row + LN_DEPTH * W < rows) {
            mbar_arrive_expect_tx(&bar[s], D * 2);
            bulk_load(ring + s * D * 2, x + (size_t)(row + LN_DEPTH * W) * D, D * 2, &bar[s]);
        }
        const float mean = warp_sum(sum) * (1.0f / D);
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const float dx = v[i] - mean;
            q += dx * dx;
        }
        const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + 1e-6f);
        uint2 *yr = (uint2 *)(y + (size_t)row * D);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = (v[8 * i + e] - mean) * rstd * gv[8 * i + e] + bv[8 * i + e];
            yr[lane + 32 * i] = make_uint2(e4m3x2(o[0] * qs, o[1] * qs) | (e4m3x2(o[2] * qs, o[3] * qs) << 16),
                                           e4m3x2(o[4] * qs, o[5] * qs) | (e4m3x2(o[6] * qs, o[7] * qs) << 16));
        }
    }
}

// Calibration: per-column max |x| over the rows of an fp16 [rows][K] tensor (K a multiple of 8), folded into amax
// (fp32 bit patterns, which order like the non-negative values they hold) with atomicMax. One thread per 8 columns,
// grid.y strides over the rows. The statistic of the reference's k_amax (kern_common.cuh:194-217).
__global__ void __launch_bounds__(128) k_amax(const __half *__restrict__ x, int K, int rows, unsigned *__restrict__ amax)
{
    const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
    if (c8 * 8 >= K) return;
    float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
        const uint4 v = __ldg((const uint4 *)(x + (size_t)r * K) + c8);
        const __half2 *hv = (const __half2 *)&v;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f = __half22float2(hv[j]);
            m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
            m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
        }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) atomicMax(amax + c8 * 8 + j, __float_as_uint(m[j]));
}

// Self-test of the failure path: one thread waits on an mbarrier of count 1 with a bound of `ns`. With arrive set
// it arrives first and the wait completes; without, nothing arrives, the wait runs out, XTB_ERR_SELFTEST is set in
// the error word and the kernel returns normally (no trap, no fault: the context stays usable).
__global__ void k_selftest_wait(uint64_t ns, int arrive, uint32_t *err)
{
    __shared__ uint64_t bar;
    if (threadIdx.x) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (arrive) mbar_arrive(&bar);
    mbar_wait_ns(&bar, 0, err, XTB_ERR_SELFTEST, ns);
}

// Row statistics of the SwiGLU output for the folded MLP LayerNorm: the NSTAT partials (sum u, sum u^2) that fc1
// wrote for a row are added in a fixed order (bit-identical run to run, as eva_kernels.cu:205-210) and turned into
// (mean, rstd) over the 2730 units (eps 1e-6, k_fc2's formula, eva_kernels.cu:318-320), written in place into
// partial 0 of the row.
// Each row's (mean, rstd) into partial 0 of stat, for the 2:4-sparse fc2 (the dense fc2's epilogue sums the
// partials itself, in the same order). Four threads per row so that small batches still spread the partial loads.
__global__ void __launch_bounds__(ROWSTAT_THREADS) k_rowstat(float2 *__restrict__ stat, int rows)
{
    griddep_wait();  // the previous kernel of the stream has completed
    const int t = blockIdx.x * ROWSTAT_THREADS + threadIdx.x, row = t >> 2;
    const float2 ms = rowstat_of(stat, rows, row, t & 3);
    __syncwarp();  // every part has read partial 0 of its row before part 0 overwrites it
    if ((t & 3) == 0 && row < rows) stat[row] = ms;
}

// Mean over patch tokens 1..1024 of each image: x [img][1025][1024] fp16 -> pool [img][1024] fp32.
// Grid (img, 16): 64 columns per block; thread (c, grp) sums 4 columns over a 64-token group; the 16 group
// partials are added in a fixed order. Replaces k_pool (eva_kernels.cu:404-431).
__global__ void __launch_bounds__(256) k_pool(const __half *__restrict__ x, float *__restrict__ pool)
{
    griddep_wait();  // the previous kernel of the stream has completed
    __shared__ float4 red[16][16];
    const int c = threadIdx.x & 15, grp = threadIdx.x >> 4;
    const __half *xr = x + ((size_t)blockIdx.x * T + 1 + grp * 64) * D + blockIdx.y * 64 + 4 * c;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int t = 0; t < 64; t++) {
        const uint2 u = *(const uint2 *)(xr + (size_t)t * D);
        const float2 p = __half22float2(*(const __half2 *)&u.x), q = __half22float2(*(const __half2 *)&u.y);
        a.x += p.x;
        a.y += p.y;
        a.z += q.x;
        a.w += q.y;
    }
    red[grp][c] = a;
    __syncthreads();
    if (grp) return;
    float4 v = red[0][c];
    for (int i = 1; i < 16; i++) {
        const float4 w = red[i][c];
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
    }
    const float k = 1.0f / (T - 1);
    *(float4 *)(pool + (size_t)blockIdx.x * D + blockIdx.y * 64 + 4 * c) = make_float4(v.x * k, v.y * k, v.z * k, v.w * k);
}

// fc_norm LayerNorm of the pooled features -> fp16 head input pn (and, for an FP8 head, E4M3(pn * qs)).
// One warp per image. Replaces k_lnh (kern_common.cuh:188-192).
__global__ void __launch_bounds__(256) k_ln_head(const float *__restrict__ pool, const float *__restrict__ g,
                                                 const float *__restrict__ bta, __half *__restrict__ pn,
                                                 uint8_t *__restrict__ pn8, int nimg, float qs)
{
    griddep_wait();  // the previous kernel of the stream has completed
    const int img = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (img >= nimg) return;
    const float4 *xr = (const float4 *)(pool + (size_t)img * D);
    float4 v[8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        v[i] = xr[lane + 32 * i];
        s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float dx;
        dx = v[i].x - mean; q += dx * dx;
        dx = v[i].y - mean; q += dx * dx;
        dx = v[i].z - mean; q += dx * dx;
        dx = v[i].w - mean; q += dx * dx;
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + 1e-6f);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int c = 4 * (lane + 32 * i);
        const float4 gg = *(const float4 *)(g + c), bb = *(const float4 *)(bta + c);
        const __half2 h0 = __floats2half2_rn((v[i].x - mean) * rstd * gg.x + bb.x, (v[i].y - mean) * rstd * gg.y + bb.y);
        const __half2 h1 = __floats2half2_rn((v[i].z - mean) * rstd * gg.z + bb.z, (v[i].w - mean) * rstd * gg.w + bb.w);
        *(uint2 *)(pn + (size_t)img * D + c) = make_uint2(*(const uint32_t *)&h0, *(const uint32_t *)&h1);
        if (pn8) {
            const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
            *(uint32_t *)(pn8 + (size_t)img * D + c) = e4m3x2(f0.x * qs, f0.y * qs) | (e4m3x2(f1.x * qs, f1.y * qs) << 16);
        }
    }
}

}  // namespace xtb

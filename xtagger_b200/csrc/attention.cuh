// FP8 flash attention on tcgen05 for the EVA02-L tagger: one CTA per (128-query tile, head, image), 1025 tokens.
// Replaces flash8<1025> (kern_common.cuh:403-543) with its arithmetic and decisions:
//   - keys in tiles of 64, as the reference; scores are raw E4M3 dot products and sinv = 1 / (cq ck) folds the
//     dequantisation (and the softmax scale times log2 e, which the weights carry in Wq) into the exp2 argument:
//     p = exp2(s sinv - m sinv) (one fma, ex2.approx as the reference's fast-math exp2f);
//   - lazy rescale, decided per 16-row slice of query rows (the rows of one reference warp, lanes 0..15 or
//     16..31 here): when some row of the slice has max(m, tm) > m + RESCALE / sinv, every row of the slice takes
//     m = max(m, tm) and rescales l and O; otherwise the running max stays stale (p <= 2^RESCALE);
//   - dead tile: when every row of the slice has tm < m - PSKIP / sinv, every p of the slice's tile rounds to zero
//     in E4M3; the slice's P is zero and l does not advance;
//   - P is quantised to E4M3 for the P V product; l sums the unquantised p; out = E4M3(fp16(O * vo / l)).
//
// Work split (320 threads, 2 CTAs per SM): one CTA per pair of 128-query tiles of one (head, image); the two tiles
// ("groups") share every K / V tile. Warp 0 TMA (both Q tiles once; K / V in tiles of 128 keys through a 3-deep
// ring), warp 1 TMEM allocation (256 columns: S_g at [64 g, 64 g + 64), O_g at [128 + 64 g, 192 + 64 g)) and the MMA
// issuer, warps 2..5 the softmax of group 0 and warps 6..9 that of group 1, one query row per thread (warp w reads
// TMEM lanes 32 (w % 4) ..). Per 64-key step u and group g: S_g,u = Q_g K_u^T (M 128, N 64 keys, K 64 dims); the
// softmax reads it in one pass with the running max (p, l and the tile max together) and re-passes a warp only when
// one of its slices rescales; it writes P_g,u (128 x 64 E4M3, 64B-swizzled K-major) to shared memory; O_g += P_g,u V_u
// (M 128, N 64 dims, K 64 keys) accumulates in TMEM with V read as an MN-major operand straight from its
// [token][64 dims] rows. While one group's softmax works, the tensor core computes the other group's scores, and 16
// softmax warps per SM (4 per sub-partition) keep the exp2 unit fed through each warp's latencies. Warps whose 32
// query rows are all padding (the last query tile holds one real row) skip the math.
#pragma once
#include "ops.h"
#include "ptx.cuh"

namespace xtb {

constexpr float ATT_RESCALE = 8.0f;
constexpr float ATT_PSKIP = 10.0f;
constexpr int ATT_SUB = 64;                       // keys per softmax step (the reference's key tile)
constexpr int ATT_NSUB = (T + ATT_SUB - 1) / ATT_SUB;  // 17 steps; the last holds 1 key
constexpr int ATT_NK = (ATT_NSUB + 1) / 2;        // 9 K / V tiles of 128 keys
constexpr int ATT_KS = 3;                         // K / V ring depth (128-key tiles)
constexpr int ATT_G = 2;                          // query tiles (groups) per CTA
constexpr int ATT_QPAIRS = (QT + ATT_G - 1) / ATT_G;  // CTAs per (head, image)
constexpr int ATT_PB = 2;                         // P buffers per group in shared memory
constexpr int ATT_THREADS = 64 + 32 * 4 * ATT_G;
constexpr int ATT_Q_BYTES = 128 * 64;
constexpr int ATT_K_BYTES = 128 * 64;
constexpr int ATT_V_BYTES = 128 * 64;
constexpr int ATT_P_BYTES = 128 * 64;             // 128 rows x 64 keys
constexpr size_t ATT_SMEM =
    1024 + ATT_G * ATT_Q_BYTES + ATT_KS * (ATT_K_BYTES + ATT_V_BYTES) + ATT_G * ATT_PB * ATT_P_BYTES + 512;

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte chunk q (0..3) of row r of a P buffer: 64-byte rows, 64B swizzle (the layout the MMA descriptor reads)
__device__ __forceinline__ uint8_t *p_chunk(uint8_t *prow, int r, int q) { return prow + ((q ^ ((r >> 1) & 3)) << 4); }

// Max of a row's valid scores in an S buffer (TMEM, 64 columns at sS).
__device__ __forceinline__ float tile_max(uint32_t sS, int nvalid)
{
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < 2; c++) {
        if (c * 32 < nvalid) {  // warp-uniform
            float v[32];
            tmem_ld32(sS + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (nvalid == 64 || c * 32 + i < nvalid) t4[i & 3] = fmaxf(t4[i & 3], v[i]);
        }
    }
    return fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
}

// One pass over a row of an S buffer with max m: tile max, p = exp2(s sinv - m sinv), sum of p, E4M3(p) -> the
// row of P. Masked keys give p = 0.
__device__ __forceinline__ void exp_pass(uint32_t sS, uint8_t *prow, int r, int nvalid, float2 sv2, float m, float *tm_out,
                                         float *l_out)
{
    const float2 nm2 = make_float2(-m * sv2.x, -m * sv2.x);
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    float2 l2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c = 0; c < 2; c++) {
        uint32_t w[8];
        if (c * 32 < nvalid) {  // warp-uniform
            float v[32];
            tmem_ld32(sS + c * 32, v);
            tmem_wait_ld();
            if (nvalid < 64) {
#pragma unroll
                for (int i = 0; i < 32; i++)
                    if (c * 32 + i >= nvalid) v[i] = -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                float pp[4];
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                    t4[e] = fmaxf(t4[e], v[i + e]);
                    t4[e + 1] = fmaxf(t4[e + 1], v[i + e + 1]);
                    const float2 a = fma2(make_float2(v[i + e], v[i + e + 1]), sv2, nm2);
                    pp[e] = ex2(a.x);
                    pp[e + 1] = ex2(a.y);
                    l2[e >> 1] = add2(l2[e >> 1], make_float2(pp[e], pp[e + 1]));
                }
                w[i >> 2] = e4m3x2(pp[0], pp[1]) | (e4m3x2(pp[2], pp[3]) << 16);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) w[i] = 0;
        }
        *(uint4 *)p_chunk(prow, r, 2 * c) = make_uint4(w[0], w[1], w[2], w[3]);
        *(uint4 *)p_chunk(prow, r, 2 * c + 1) = make_uint4(w[4], w[5], w[6], w[7]);
    }
    *tm_out = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
    *l_out = (l2[0].x + l2[0].y) + (l2[1].x + l2[1].y);
}

__device__ __forceinline__ void zero_prow(uint8_t *prow)
{
#pragma unroll
    for (int q = 0; q < 4; q++) *(uint4 *)(prow + 16 * q) = make_uint4(0, 0, 0, 0);
}

// fp32 -> fp16 (round to nearest) -> E4M3, as the reference's output staging (kern_common.cuh:527-541)
__device__ __forceinline__ uint32_t e4m3x2_via_f16(float a, float b)
{
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    return e4m3x2(f.x, f.y);
}

__global__ void __launch_bounds__(ATT_THREADS, 2)
    k_attention(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, uint8_t *__restrict__ out, float sinv, float vo, uint32_t *err)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem;                                  // [ATT_G]
    uint8_t *sK = sQ + ATT_G * ATT_Q_BYTES;              // [ATT_KS]
    uint8_t *sV = sK + ATT_KS * ATT_K_BYTES;             // [ATT_KS]
    uint8_t *sP = sV + ATT_KS * ATT_V_BYTES;             // [ATT_G][ATT_PB]
    uint64_t *bar = (uint64_t *)(sP + ATT_G * ATT_PB * ATT_P_BYTES);
    uint64_t *q_full = bar;
    uint64_t *kv_full = q_full + 1;                      // [ATT_KS]
    uint64_t *kv_empty = kv_full + ATT_KS;               // [ATT_KS]
    uint64_t *s_full = kv_empty + ATT_KS;                // [ATT_G]
    uint64_t *s_free = s_full + ATT_G;                   // [ATT_G]
    uint64_t *p_full = s_free + ATT_G;                   // [ATT_G][ATT_PB]
    uint64_t *pv_done = p_full + ATT_G * ATT_PB;         // [ATT_G][ATT_PB]
    uint32_t *tslot = (uint32_t *)(pv_done + ATT_G * ATT_PB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt0 = blockIdx.x * ATT_G, h = blockIdx.y, b = blockIdx.z;
    const int ng = min(ATT_G, QT - qt0);                 // query tiles this CTA holds
    const int bh = b * NH + h;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ATT_KS; s++) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int g = 0; g < ATT_G; g++) {
            mbar_init(&s_full[g], 1);
            mbar_init(&s_free[g], 4);
            for (int s = 0; s < ATT_PB; s++) {
                mbar_init(&p_full[g * ATT_PB + s], 4);
                mbar_init(&pv_done[g * ATT_PB + s], 1);
            }
        }
        fence_mbar_init();
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        tma_prefetch_desc(&tv);
    }
    if (warp == 1) {
        tmem_alloc(tslot, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, ng * ATT_Q_BYTES);
            for (int g = 0; g < ng; g++) tma_load_2d(sQ + g * ATT_Q_BYTES, &tq, q_full, 0, bh * TP + (qt0 + g) * 128);
            uint32_t ph = 0;
            int st = 0;
            for (int j = 0; j < ATT_NK; j++) {
                if (!mbar_wait(&kv_empty[st], ph ^ 1, err, XTB_ERR_WAIT_ATTN)) break;
                mbar_arrive_expect_tx(&kv_full[st], ATT_K_BYTES + ATT_V_BYTES);
                tma_load_2d(sK + st * ATT_K_BYTES, &tk, &kv_full[st], 0, bh * TP + j * 128);
                tma_load_2d(sV + st * ATT_V_BYTES, &tv, &kv_full[st], 0, bh * TP + j * 128);
                if (++st == ATT_KS) {
                    st = 0;
                    ph ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            // S: N = 64 keys. PV: B = V, MN-major (bit 16): its N (dims) run contiguous within each key's 64-byte row
            constexpr uint32_t ID_S = idesc_m128(64), ID_PV = idesc_m128(64) | (1u << 16);
            bool ok = mbar_wait(q_full, 0, err, XTB_ERR_WAIT_ATTN);
            for (int u = 0; u <= ATT_NSUB && ok; u++) {
                if (u < ATT_NSUB) {  // S_g,u = Q_g K_u^T, each group once its softmax has read S_g,u-1
                    const int j = u >> 1, st = j % ATT_KS;
                    if (!(u & 1) && !(ok = mbar_wait(&kv_full[st], (j / ATT_KS) & 1, err, XTB_ERR_WAIT_ATTN))) break;
                    const uint32_t k0 = smem_u32(sK + st * ATT_K_BYTES) + (u & 1) * 4096;  // 64 keys x 64 bytes in
                    for (int g = 0; g < ng && ok; g++) {
                        if (u > 0 && !(ok = mbar_wait(&s_free[g], (u - 1) & 1, err, XTB_ERR_WAIT_ATTN))) break;
                        tc_fence_after();
                        const uint32_t q0 = smem_u32(sQ + g * ATT_Q_BYTES);
#pragma unroll
                        for (int kk = 0; kk < 2; kk++)
                            umma<false>(tbase + g * 64, sdesc(q0 + kk * 32, 512, SWZ_64B), sdesc(k0 + kk * 32, 512, SWZ_64B),
                                        ID_S, kk);
                        umma_commit(&s_full[g]);
                    }
                    if (!ok) break;
                }
                if (u > 0) {  // O_g += P_g,w V_w for the previous step
                    const int w = u - 1, pb = w & 1, st = (w >> 1) % ATT_KS;
                    const uint32_t v0 = smem_u32(sV + st * ATT_V_BYTES) + (w & 1) * 4096;
                    for (int g = 0; g < ng && ok; g++) {
                        if (!(ok = mbar_wait(&p_full[g * ATT_PB + pb], (w >> 1) & 1, err, XTB_ERR_WAIT_ATTN))) break;
                        tc_fence_after();
                        const uint32_t p0 = smem_u32(sP + (g * ATT_PB + pb) * ATT_P_BYTES);
#pragma unroll
                        for (int kk = 0; kk < 2; kk++)
                            umma<false>(tbase + 128 + g * 64, sdesc(p0 + kk * 32, 512, SWZ_64B),
                                        sdesc_mn(v0 + kk * 2048, 512, SWZ_64B), ID_PV, (w > 0 || kk > 0));
                        umma_commit(&pv_done[g * ATT_PB + pb]);
                    }
                    if (!ok) break;
                    if ((w & 1) || w == ATT_NSUB - 1) umma_commit(&kv_empty[st]);  // the K / V tile is used up
                }
            }
        }
    } else if ((warp - 2) / 4 < ng) {
        const int g = (warp - 2) / 4;                    // query tile (group) of this warp
        const int quad = warp & 3;
        const int r = quad * 32 + lane;                  // query row within the tile = TMEM lane
        const uint32_t lrow = (uint32_t)(quad * 32) << 16;
        const uint32_t sS = tbase + g * 64 + lrow, sO = tbase + 128 + g * 64 + lrow;
        uint64_t *gp_full = p_full + g * ATT_PB, *gpv_done = pv_done + g * ATT_PB;
        const float thr = ATT_RESCALE / sinv, dthr = ATT_PSKIP / sinv;
        const bool idle = (qt0 + g) * 128 + quad * 32 >= T;   // warp-uniform: every row of the warp is padding
        const uint32_t half = lane < 16 ? 0x0000FFFFu : 0xFFFF0000u;  // this row's 16-row slice
        const float2 sv2 = make_float2(sinv, sinv);
        float m = -1e30f, l = 0.f;
        bool ok = true;
        for (int u = 0; u < ATT_NSUB && ok; u++) {
            const int pb = u & 1;
            const int nvalid = min(ATT_SUB, T - u * ATT_SUB);
            uint8_t *prow = sP + (g * ATT_PB + pb) * ATT_P_BYTES + r * 64;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[g], u & 1, err, XTB_ERR_WAIT_ATTN)))) break;
            // P buffer pb was last read by PV_{u-2}
            if (u >= ATT_PB &&
                !(ok = __all_sync(0xffffffffu, mbar_wait(&gpv_done[pb], ((u >> 1) - 1) & 1, err, XTB_ERR_WAIT_ATTN))))
                break;
            tc_fence_after();
            if (idle) {
                zero_prow(prow);
            } else {
                // one pass with the running max: tile max, p = exp2(s sinv - m sinv), l_tile, P
                float tm = -INFINITY, lt = 0.f;
                if (u > 0) exp_pass(sS, prow, r, nvalid, sv2, m, &tm, &lt);
                else tm = tile_max(sS, nvalid);
                const float mn = fmaxf(m, tm);
                const bool resc = (__ballot_sync(0xffffffffu, mn > m + thr) & half) != 0;
                if (__any_sync(0xffffffffu, resc)) {
                    float sc = 1.0f;
                    if (resc) {  // every row of a rescaling slice takes its max
                        sc = ex2((m - mn) * sinv);
                        l *= sc;
                        m = mn;
                    }
                    if (u > 0) {
                        // O holds P V of the earlier steps: rescale it in TMEM once PV_{u-1} has landed (TMEM access
                        // is warp-collective: factor 1 for the slice that keeps its max)
                        const int w = u - 1;
                        if (!(ok = __all_sync(0xffffffffu,
                                              mbar_wait(&gpv_done[w & 1], (w >> 1) & 1, err, XTB_ERR_WAIT_ATTN))))
                            break;
                        tc_fence_after();
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            float v[16];
                            tmem_ld16(sO + c * 16, v);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; i++) v[i] *= sc;
                            tmem_st16(sO + c * 16, v);
                        }
                        tmem_wait_st();
                    }
                    // (re)compute P with the refreshed max; the other slice recomputes the same values
                    float tm2;
                    exp_pass(sS, prow, r, nvalid, sv2, m, &tm2, &lt);
                }
                if ((__ballot_sync(0xffffffffu, tm < m - dthr) & half) == half) {  // dead slice: P zero, l unchanged
                    zero_prow(prow);
                    lt = 0.f;
                }
                l += lt;
            }
            // S_g,u fully read: the tensor core may overwrite it with S_g,u+1
            tc_fence_before();
            fence_proxy_async_smem();  // P (generic-proxy stores) -> visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_free[g]);
                mbar_arrive(&gp_full[pb]);
            }
        }
        if (ok) {
            const int wl = ATT_NSUB - 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&gpv_done[wl & 1], (wl >> 1) & 1, err, XTB_ERR_WAIT_ATTN));
        }
        if (ok && !idle) {
            tc_fence_after();
            const float f = vo / l;
            uint32_t w[16];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                float v[32];
                tmem_ld32(sO + c * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    w[c * 8 + (i >> 2)] = e4m3x2_via_f16(v[i] * f, v[i + 1] * f) | (e4m3x2_via_f16(v[i + 2] * f, v[i + 3] * f) << 16);
            }
            const int t = (qt0 + g) * 128 + r;
            if (t < T) {
                uint4 *o = (uint4 *)(out + ((size_t)b * T + t) * D + h * HD);
#pragma unroll
                for (int c = 0; c < 4; c++) o[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, 256);
    }
}

}  // namespace xtb

// FP8 flash attention on tcgen05 for the EVA02-L tagger: one CTA per (128-query tile, head, image), 1025 tokens.
// Replaces flash8<1025> (kern_common.cuh:403-543) with the same arithmetic contract:
//   - scores are raw E4M3 dot products; sinv = 1 / (cq ck) folds the dequantisation (and the softmax scale
//     times log2 e, which the weights carry in Wq) into the exp2 argument: p = exp2((s - m) * sinv);
//   - lazy rescale: the running max m of a row is only refreshed when a tile's max exceeds it by more than
//     RESCALE / sinv (p stays <= 2^RESCALE, inside E4M3), which also rescales l and O;
//   - dead tile: when a row's tile max is below m - PSKIP / sinv every p of the tile rounds to zero in E4M3,
//     so the row's P is zero and l is not advanced;
//   - P is quantised to E4M3 for the P V product; l sums the unquantised p; out = O * vo / l -> E4M3.
// Decisions are per query row here (one row per thread), where the reference takes them per 16-row warp slice.
//
// Warp roles (192 threads, 2 CTAs per SM): warp 0 TMA (Q once; K / V tiles through a 3-deep ring), warp 1 TMEM
// allocation (256 columns: S at [0,128), O at [128,192)) and the MMA issuer, warps 2..5 softmax, one query row per
// thread. After the first tile the softmax makes a single pass over S with the running max (p, l and P computed
// while the tile max is tracked) and only re-passes a warp when one of its rows crossed the lazy-rescale
// threshold; warps whose 32 query rows are all padding (the last query tile holds one real row) skip the math.
// S_j = Q K_j^T (M 128, N 128 keys, K 64 dims) -> TMEM; softmax reads it (two passes: max, then exp2 / quantise),
// writes P_j (128 x 128 E4M3, 128B-swizzled K-major) to shared memory; O += P_j V_j (M 128, N 64 dims, K 128 keys)
// accumulates in TMEM, with V read as an MN-major operand straight from its [token][64 dims] rows (64B swizzle,
// 8-key groups 512 bytes apart). S_{j+1} is issued as soon as the softmax has read S_j, ahead of PV_j.
#pragma once
#include "ops.h"
#include "ptx.cuh"

namespace xtb {

constexpr float ATT_RESCALE = 8.0f;
constexpr float ATT_PSKIP = 10.0f;
constexpr int ATT_KS = 3;                 // K / V ring depth
constexpr int ATT_NK = TP / 128;          // key tiles (9; the last holds 1 key)
constexpr int ATT_THREADS = 192;
constexpr int ATT_Q_BYTES = 128 * 64;
constexpr int ATT_K_BYTES = 128 * 64;
constexpr int ATT_V_BYTES = 128 * 64;
constexpr int ATT_P_BYTES = 128 * 128;
constexpr size_t ATT_SMEM = 1024 + ATT_Q_BYTES + ATT_KS * (ATT_K_BYTES + ATT_V_BYTES) + 2 * ATT_P_BYTES + 256;

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Max of a row's valid scores in the S tile (TMEM, 128 columns at sS).
__device__ __forceinline__ float tile_max(uint32_t sS, int nvalid)
{
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        if (c * 32 < nvalid) {  // warp-uniform
            float v[32];
            tmem_ld32(sS + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (nvalid == 128 || c * 32 + i < nvalid) t4[i & 3] = fmaxf(t4[i & 3], v[i]);
        }
    }
    return fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
}

// One pass over a row of the S tile with max m: tile max, p = exp2((s - m) sinv), sum of p, E4M3(p) -> the row of P
// (128B-swizzled). Masked keys give p = 0.
__device__ __forceinline__ void exp_pass(uint32_t sS, uint8_t *prow, int r, int nvalid, float2 sv2, float m, float *tm_out,
                                         float *l_out)
{
    const float2 nm2 = make_float2(-m * sv2.x, -m * sv2.x);
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    float2 l2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t w[8];
        if (c * 32 < nvalid) {  // warp-uniform
            float v[32];
            tmem_ld32(sS + c * 32, v);
            tmem_wait_ld();
            if (nvalid < 128) {
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
        *(uint4 *)(prow + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *(uint4 *)(prow + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
    *tm_out = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
    *l_out = (l2[0].x + l2[0].y) + (l2[1].x + l2[1].y);
}

__global__ void __launch_bounds__(ATT_THREADS, 2)
    k_attention(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, uint8_t *__restrict__ out, float sinv, float vo, uint32_t *err)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + ATT_Q_BYTES;
    uint8_t *sV = sK + ATT_KS * ATT_K_BYTES;
    uint8_t *sP = sV + ATT_KS * ATT_V_BYTES;
    uint64_t *bar = (uint64_t *)(sP + 2 * ATT_P_BYTES);
    uint64_t *q_full = bar;
    uint64_t *kv_full = bar + 1;              // [ATT_KS]
    uint64_t *kv_empty = kv_full + ATT_KS;    // [ATT_KS]
    uint64_t *s_full = kv_empty + ATT_KS;
    uint64_t *s_free = s_full + 1;
    uint64_t *p_full = s_free + 1;            // [2]
    uint64_t *pv_done = p_full + 2;           // [2]
    uint32_t *tslot = (uint32_t *)(pv_done + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int bh = b * NH + h;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ATT_KS; s++) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        for (int i = 0; i < 2; i++) {
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_done[i], 1);
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
    const uint32_t tS = tbase, tO = tbase + 128;

    if (warp == 0) {
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, ATT_Q_BYTES);
            tma_load_2d(sQ, &tq, q_full, 0, bh * TP + qt * 128);
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
            // PV: B = V, MN-major (bit 16): its N (dims) run contiguous within each key's 64-byte row
            constexpr uint32_t ID_S = idesc_m128(128), ID_PV = idesc_m128(64) | (1u << 16);
            const uint32_t q0 = smem_u32(sQ);
            bool ok = mbar_wait(q_full, 0, err, XTB_ERR_WAIT_ATTN);
            int st = 0, pst = 0;
            uint32_t ph = 0;
            for (int j = 0; j <= ATT_NK && ok; j++) {
                if (j < ATT_NK) {
                    if (!(ok = mbar_wait(&kv_full[st], ph, err, XTB_ERR_WAIT_ATTN))) break;
                    if (j > 0 && !(ok = mbar_wait(s_free, (j - 1) & 1, err, XTB_ERR_WAIT_ATTN))) break;
                    tc_fence_after();
                    const uint32_t k0 = smem_u32(sK + st * ATT_K_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 2; kk++)
                        umma<false>(tS, sdesc(q0 + kk * 32, 512, SWZ_64B), sdesc(k0 + kk * 32, 512, SWZ_64B), ID_S, kk);
                    umma_commit(s_full);
                }
                if (j > 0) {
                    const int jp = j - 1;
                    if (!(ok = mbar_wait(&p_full[jp & 1], (jp >> 1) & 1, err, XTB_ERR_WAIT_ATTN))) break;
                    tc_fence_after();
                    const uint32_t p0 = smem_u32(sP + (jp & 1) * ATT_P_BYTES);
                    const uint32_t v0 = smem_u32(sV + pst * ATT_V_BYTES);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma<false>(tO, sdesc(p0 + kk * 32, 1024, SWZ_128B), sdesc_mn(v0 + kk * 2048, 512, SWZ_64B),
                                    ID_PV, (jp > 0 || kk > 0));
                    umma_commit(&pv_done[jp & 1]);
                    umma_commit(&kv_empty[pst]);
                    if (++pst == ATT_KS) pst = 0;
                }
                if (j < ATT_NK && ++st == ATT_KS) {
                    st = 0;
                    ph ^= 1;
                }
            }
        }
    } else {
        const int quad = warp & 3;
        const int r = quad * 32 + lane;                 // query row within the tile = TMEM lane
        const uint32_t lrow = (uint32_t)(quad * 32) << 16;
        const uint32_t sS = tS + lrow, sO = tO + lrow;
        const float thr = ATT_RESCALE / sinv, dthr = ATT_PSKIP / sinv;
        const bool idle = qt * 128 + quad * 32 >= T;     // warp-uniform: every row of the warp is padding
        const float2 sv2 = make_float2(sinv, sinv);
        float m = -1e30f, l = 0.f;
        bool ok = true;
        for (int j = 0; j < ATT_NK && ok; j++) {
            const int nvalid = min(128, T - j * 128);
            uint8_t *prow = sP + (j & 1) * ATT_P_BYTES + r * 128;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, err, XTB_ERR_WAIT_ATTN)))) break;
            // P buffer j & 1 was last read by PV_{j-2}
            if (j >= 2) {
                const int jq = j - 2;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[jq & 1], (jq >> 1) & 1, err, XTB_ERR_WAIT_ATTN))))
                    break;
            }
            tc_fence_after();
            if (idle) {
#pragma unroll
                for (int c = 0; c < 8; c++) *(uint4 *)(prow + ((c ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
            } else {
                // one pass with the running max: tile max, p = exp2((s - m) sinv), l_tile, P
                float tm = -INFINITY, lt = 0.f;
                if (j > 0) exp_pass(sS, prow, r, nvalid, sv2, m, &tm, &lt);
                else tm = tile_max(sS, nvalid);
                const bool resc = tm > m + thr;
                if (__any_sync(0xffffffffu, resc)) {
                    float sc = 1.0f;
                    if (resc) {
                        sc = ex2((m - tm) * sinv);
                        l *= sc;
                        m = tm;
                    }
                    if (j > 0) {
                        // O holds P V of the earlier tiles: rescale it in TMEM once PV_{j-1} has landed (TMEM
                        // access is warp-collective: factor 1 for the rows that keep their max)
                        const int jp = j - 1;
                        if (!(ok = __all_sync(0xffffffffu,
                                              mbar_wait(&pv_done[jp & 1], (jp >> 1) & 1, err, XTB_ERR_WAIT_ATTN))))
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
                    // (re)compute P with the refreshed max; rows that kept theirs recompute the same values
                    float tm2, lt2;
                    exp_pass(sS, prow, r, nvalid, sv2, m, &tm2, &lt2);
                    lt = lt2;
                }
                if (tm < m - dthr) {   // dead row: every p of the tile rounds to zero in E4M3, l unchanged
#pragma unroll
                    for (int c = 0; c < 8; c++) *(uint4 *)(prow + ((c ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                    lt = 0.f;
                }
                l += lt;
            }
            // S_j fully read: the tensor core may overwrite it with S_{j+1}
            tc_fence_before();
            fence_proxy_async_smem();  // P (generic-proxy stores) -> visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(s_free);
                mbar_arrive(&p_full[j & 1]);
            }
        }
        if (ok) {
            const int jl = ATT_NK - 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, err, XTB_ERR_WAIT_ATTN));
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
                    w[c * 8 + (i >> 2)] = e4m3x2(v[i] * f, v[i + 1] * f) | (e4m3x2(v[i + 2] * f, v[i + 3] * f) << 16);
            }
            const int t = qt * 128 + r;
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

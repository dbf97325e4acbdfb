// Block-scaled FP8 GEMM on CTA pairs with the tensor core's own block scaling (tcgen05.mma.cta_group::2
// kind::mxf8f6f4.block_scale), for weights whose 128 x 128 block scales are powers of two.
//
// A pair computes 256 x 128 output tiles: rank r loads A rows 128 r .. 128 r + 127 of the tile and B rows 64 r ..
// 64 r + 63, rank 0 issues M = 256, N = 128 MMAs for both (gemm2.cuh's operand split, which halves each SM's B
// traffic). A tile's 128 B rows are exactly one 128-row weight block, so one scale record per 128-byte K slice covers
// the whole MMA: both ranks load the same 512-byte record (every byte the block's UE8M0 exponent, gemm_mx.cuh's
// image) into the same shared-memory offset, and rank 0 copies it into both CTAs' tensor memory with
// tcgen05.cp.cta_group::2 — uniform records make the result independent of how the pair splits the scale factors
// between the two CTAs. A's scale factors are 2^0.
//
// The whole K range accumulates in one TMEM buffer per tile (128 columns). Two epilogue groups of four warps (one
// per lane quadrant, 128 columns per thread, gemm2.cuh's GROUPS layout) take the pair's tiles in turn, each with
// its own buffer, so one group's drain and fused apply overlap the MMA of the other group's tile; TMEM: buffers at
// columns 0 / 128, A scale factors at 256, B scale factors at 288.
//
// NB2 = 2 (wide tiles): a pair computes 256 x 256 tiles as two M = 256, N = 128 MMAs per 128-byte K slice, one per
// 128-row weight block, each with that block's own uniform scale record (B scale factors at columns 288 and 296), so
// each A slice brought into shared memory serves 256 output columns instead of 128: half the A traffic per FLOP,
// which bounds fc2 (K = 2736, A streamed from DRAM) and speeds up QKV and fc1 as well; N need not be a multiple
// of 256 when the epilogue skips a half tile past N (the B rows there read as the TMA fill value, and the scale
// image's block count is even, so the second record exists). The tile's accumulator fills columns 0 .. 255,
// so there is one buffer: epilogue group g drains columns 128 g .. 128 g + 127 of every tile, and the next tile's
// MMAs start once both groups of both CTAs have read it.
#pragma once
#include "gemm2.cuh"
#include "gemm_mx.cuh"

namespace xtb {

template <int SPW, int NB2 = 1>
struct Gemm2MxCfg {
    static_assert(NB2 == 1 || NB2 == 2, "one or two weight blocks per tile");
    static constexpr int BN = 128 * NB2;                    // tile columns
    static constexpr int EW = 8;                            // two groups of four epilogue warps
    static constexpr int COLS = 128;                        // accumulator columns per epilogue thread
    static constexpr int NBUF = 3 - NB2;                    // accumulator buffers (one per group, or one shared)
    static constexpr int TEMPTY = NB2 * 2 * 4;              // the buffer's readers: one or both groups, both CTAs
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = NB2 * 64 * 128;          // per weight block: 64 rows per CTA
    static constexpr int SF_BYTES = NB2 * 512;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGING = EW * SPW;
    static constexpr int STAGES_FIT = (232448 - 1024 - 1024 - 1024 - 512 - STAGING) / (STAGE_BYTES + SF_BYTES);
    static constexpr int STAGES = STAGES_FIT < 8 ? STAGES_FIT : 8;
    static constexpr int SF_AREA = (STAGES * SF_BYTES + 1023) & ~1023;   // keeps the staging 1024-aligned
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + SF_AREA + STAGING + 512 + 1024;
    static constexpr int THREADS = 64 + 32 * EW;
    static constexpr uint32_t SFA_COL = 256, SFB_COL = 288;  // weight block j's B scale factors at SFB_COL + 8 j
    static_assert(STAGES >= 4 && SMEM <= 232448, "shared memory budget");
};

// XTB_PREFETCH_W=0 at build time: no weight loads before the grid-dependency wait.
#ifndef XTB_PREFETCH_W
#define XTB_PREFETCH_W 1
#endif

template <class Epi, int NB2 = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    k_gemm2_mx(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmSF, const __grid_constant__ CUtensorMap tmC, const GemmArgs g,
               const GemmMxArgs mx, const typename Epi::Params ep)
{
    using C = Gemm2MxCfg<StagingOf<Epi>::v, NB2>;
    constexpr int STAGES = C::STAGES, COLS = C::COLS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = sA + STAGES * C::A_BYTES;
    uint8_t *sSF = sB + STAGES * C::B_BYTES;            // [STAGES][512]
    uint8_t *sStage = sSF + C::SF_AREA;
    uint8_t *sSFA = sStage + C::STAGING;                // 512 bytes of 2^0 scale factors
    uint64_t *full = (uint64_t *)(sSFA + 512);          // rank 0: both producers' bytes
    uint64_t *empty = full + STAGES;                    // every rank: stage consumed by the pair MMA
    uint64_t *tfull = empty + STAGES;                   // every rank: [buffer] tile accumulated
    uint64_t *tempty = tfull + 2;                       // rank 0: [buffer] buffer read by its readers in both CTAs
    uint32_t *tslot = (uint32_t *)(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    for (int i = threadIdx.x; i < 512 / 16; i += blockDim.x) ((uint4 *)sSFA)[i] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 2);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], C::TEMPTY);
        }
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmSF);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tslot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers and scale factors are ready before anyone uses them
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const int total = g.m_tiles * g.n_tiles;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int KI = g.kiters;
    if (warp != 0) griddep_wait();  // the previous kernel of the stream has completed: activations may be touched

    if (warp == 0) {
        if (elect_one()) {
            const uint32_t full0 = mapa_shared(smem_u32(full), 0);
            // Weights (B rows and scale records) are not written by earlier kernels: the first tile's first ring
            // slots get theirs before the wait, so that their load latency overlaps the previous kernel's tail.
            // These slots are in their first round (no consumer to wait for); the expected bytes include A's.
            const int pre = (XTB_PREFETCH_W && pair < total) ? min(STAGES, KI) : 0;
            for (int k = 0; k < pre; k++) {
                const int nb = pair % g.n_tiles;
                const uint32_t fb = full0 + k * 8;
                mbar_arrive_expect_tx_cluster(fb, C::STAGE_BYTES + C::SF_BYTES);
#pragma unroll
                for (int j = 0; j < NB2; j++) {
                    const int wb = nb * NB2 + j;
                    tma_load_2d_pair(sB + k * C::B_BYTES + j * 8192, &tmB, fb, k * 128, wb * 128 + rank * 64);
                    tma_load_2d_pair(sSF + k * C::SF_BYTES + j * 512, &tmSF, fb, 0, 2 * (k * mx.nbp + wb));
                }
            }
            griddep_wait();
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                const int nb = t % g.n_tiles, mb = t / g.n_tiles;
                for (int k = 0; k < KI; k++) {
                    const bool early = t == pair && k < pre;  // B and scales already on their way
                    const uint32_t fb = full0 + stage * 8;
                    if (!early) {
                        if (!(ok = mbar_wait(&empty[stage], ph ^ 1, g.err, XTB_ERR_WAIT_TMA))) break;
                        mbar_arrive_expect_tx_cluster(fb, C::STAGE_BYTES + C::SF_BYTES);
                    }
                    tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, fb, k * 128, mb * 256 + rank * 128);
                    if (!early) {
#pragma unroll
                        for (int j = 0; j < NB2; j++) {  // weight block nb NB2 + j: B rows and its scale record
                            const int wb = nb * NB2 + j;
                            tma_load_2d_pair(sB + stage * C::B_BYTES + j * 8192, &tmB, fb, k * 128, wb * 128 + rank * 64);
                            tma_load_2d_pair(sSF + stage * C::SF_BYTES + j * 512, &tmSF, fb, 0, 2 * (k * mx.nbp + wb));
                        }
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (rank == 0 && elect_one()) {
            const uint32_t sfa = tbase + C::SFA_COL, sfb = tbase + C::SFB_COL;
            tmem_cp_pair_32x128b_x4(sfa, sdesc_rows16(smem_u32(sSFA)));
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair, i = 0; t < total && ok; t += npairs, i++) {
                // NB2 = 1: group i & 1's buffer and its use count's parity; NB2 = 2: the one buffer
                const uint32_t buf = NB2 == 1 ? (i & 1) : 0, tph = NB2 == 1 ? (i >> 1) & 1 : i & 1;
                for (int k = 0; k < KI; k++) {
                    if (k == 0) {
                        if (!(ok = mbar_wait(&tempty[buf], tph ^ 1, g.err, XTB_ERR_WAIT_TMEM))) break;
                        tc_fence_after();
                    }
                    if (!(ok = mbar_wait(&full[stage], ph, g.err, XTB_ERR_WAIT_TMA))) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
                    // in issue order after the previous slice's MMAs (the tensor core keeps its order)
#pragma unroll
                    for (int j = 0; j < NB2; j++)
                        tmem_cp_pair_32x128b_x4(sfb + 8 * j, sdesc_rows16(smem_u32(sSF + stage * C::SF_BYTES + j * 512)));
#pragma unroll
                    for (int j = 0; j < NB2; j++)
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_pair_mx(tbase + buf * 128 + j * 128, sdesc(a0 + kk * 32, 1024, SWZ_128B),
                                         sdesc(b0 + j * 8192 + kk * 32, 1024, SWZ_128B), idesc_mx_m256(128, kk, kk), sfa,
                                         sfb + 8 * j, (k > 0 || kk > 0));
                    umma_commit_pair(&empty[stage], 0x3);
                    if (k == KI - 1) umma_commit_pair(&tfull[buf], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1;
                    }
                }
            }
        }
    } else {
        const int ew = warp - 2;
        const int quad = warp & 3;
        const int grp = ew >> 2;
        const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
        EpiCtx cx;
        cx.lane = lane;
        cx.stage = sStage + ew * StagingOf<Epi>::v;
        cx.tmC = &tmC;
        uint32_t tph = 0;
        bool ok = true;
        // NB2 = 1: the groups take the pair's tiles in turn, each in its own buffer; NB2 = 2: both take every tile,
        // group g its columns 128 g .. 128 g + 127 (in TMEM and in the output), from the one buffer
        const int bufi = NB2 == 1 ? grp : 0;
        for (int t = pair + (NB2 == 1 ? grp * npairs : 0); t < total && ok; t += (NB2 == 1 ? 2 : 1) * npairs) {
            const int nb = t % g.n_tiles, mb = t / g.n_tiles;
            cx.row0 = mb * 256 + rank * 128 + quad * 32;
            cx.col0 = nb * C::BN + (NB2 == 1 ? 0 : grp * 128);
            typename Epi::State es;
            Epi::begin(ep, cx, es);
            const float s = g.ascale * Epi::col_scale(ep, cx);
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[bufi], tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
            tph ^= 1;
            tc_fence_after();
            const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + grp * 128;  // either layout
            if constexpr (StreamOf<Epi>::v) {
                float v[2][32];
                tmem_ld16(taddr, v[0]);
                tmem_ld16(taddr + 16, v[0] + 16);
#pragma unroll
                for (int c = 0; c < COLS / 32; c++) {
                    tmem_wait_ld_regs(v[c & 1]);
                    if (c + 1 < COLS / 32) {
                        tmem_ld16(taddr + 32 * (c + 1), v[(c + 1) & 1]);
                        tmem_ld16(taddr + 32 * (c + 1) + 16, v[(c + 1) & 1] + 16);
                    } else {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(tempty0 + bufi * 8);
                    }
                    Epi::apply_chunk(ep, v[c & 1], s, c, cx, es);
                }
                Epi::finish(ep, cx, es);
            } else {
                float2 acc[COLS / 2];
                const float2 s2 = make_float2(s, s);
#pragma unroll
                for (int c0 = 0; c0 < COLS; c0 += 32) {
                    float v[32];
                    tmem_ld16(taddr + c0, v);
                    tmem_ld16(taddr + c0 + 16, v + 16);
                    tmem_wait_ld_regs(v);
#pragma unroll
                    for (int j = 0; j < 16; j++) acc[c0 / 2 + j] = mul2(s2, make_float2(v[2 * j], v[2 * j + 1]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty0 + bufi * 8);
                Epi::apply(ep, (float *)acc, cx, es);
            }
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still arrive on its barriers or read its shared memory
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tbase, 512);
    }
}

}  // namespace xtb

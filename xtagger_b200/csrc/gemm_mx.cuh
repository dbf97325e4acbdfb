// Block-scaled FP8 GEMM on the tensor core's own block scaling (tcgen05.mma kind::mxf8f6f4.block_scale), for
// weights whose 128 x 128 block scales are powers of two: D[M][N] = epilogue(ascale x sum_k A[m][k] B[n][k] w[n/128][k/128]).
//
// A power-of-two block scale is exact as an UE8M0 scale factor, so the tensor core applies it inside the MMA and
// the whole K range accumulates in one TMEM buffer: no per-K-block promotion through the epilogue warps (gemm.cuh's
// PROMOTE path), the same dequantize-then-matmul values up to the fp32 summation order.
//
// Layout (one persistent CTA per SM, 128 x 256 output tiles, 320 threads as gemm.cuh):
//   warp 0   TMA producer: per 128-byte K slice the A box (128 rows), the B box (256 rows) and, by a bulk copy, the
//            slice's 1 KB scale-factor image: two 512-byte records, one per 128-row N block of the tile, every byte
//            the block scale's UE8M0 exponent (so the scale-factor layout inside a record does not matter);
//   warp 1   TMEM (512 columns: accumulator [0, 256), A scale factors at 256, B scale factors at 288 / 296), MMA:
//            per K slice tcgen05.cp of the two records into the B scale-factor columns, then for each 32-byte K step
//            two N = 128 MMAs (one per N block, each with its own scale factors); A's scale factors are 2^0;
//   warps 2..9 the epilogue of gemm.cuh (streaming or not) on the single accumulator, handed back to the MMA as soon
//            as it is in registers.
#pragma once
#include "gemm.cuh"

namespace xtb {

template <int SPW>
struct GemmMxCfg {
    static constexpr int BN = 256;
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int SF_BYTES = 1024;               // two 512-byte records per K slice
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EW = 8;
    static constexpr int COLS = BN / (EW / 4);          // 128 accumulator columns per epilogue thread
    static constexpr int STAGING = EW * SPW;
    // as many stages (at most 4) as fit beside the epilogue's staging: 4 with 2 KB per warp, 3 with 4 or 8 KB
    static constexpr int STAGES_FIT = (232448 - 2048 - STAGING) / (STAGE_BYTES + SF_BYTES);
    static constexpr int STAGES = STAGES_FIT < 4 ? STAGES_FIT : 4;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * (STAGE_BYTES + SF_BYTES) + STAGING + 512 + 512;
    static constexpr int THREADS = 64 + 32 * EW;
    static constexpr uint32_t SFA_COL = 256, SFB_COL = 288;
    static_assert(STAGES >= 3 && SMEM <= 232448, "shared memory budget");
};

// Scale-factor image of a weight: [kiters][nbp][512] bytes, nbp = N blocks rounded up to even.
struct GemmMxArgs {
    const uint8_t *sf;
    int nbp;
};

template <class Epi>
__global__ void __launch_bounds__(320, 1)
    k_gemm_mx(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, const GemmArgs g, const GemmMxArgs mx,
              const typename Epi::Params ep)
{
    using C = GemmMxCfg<StagingOf<Epi>::v>;
    constexpr int STAGES = C::STAGES, COLS = C::COLS, BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * C::A_BYTES;
    uint8_t *sSF = sB + STAGES * C::B_BYTES;            // [STAGES][1024]
    uint8_t *sStage = sSF + STAGES * C::SF_BYTES;       // 1024-aligned: the epilogues' swizzled TMA boxes
    uint8_t *sSFA = sStage + C::STAGING;                // 512 bytes of 2^0 scale factors
    uint64_t *full = (uint64_t *)(sSFA + 512);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 1;
    uint32_t *tslot = (uint32_t *)(tempty + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < 512 / 16; i += blockDim.x) ((uint4 *)sSFA)[i] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    fence_proxy_async_smem();  // the tensor core's copy reads them through the async proxy
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, C::EW);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    griddep_wait();  // the previous kernel of the stream has completed: activations may be touched
    const int total = g.m_tiles * g.n_tiles;
    const int KI = g.kiters;

    if (warp == 0) {
        if (elect_one()) {
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const int nb = t % g.n_tiles, mb = t / g.n_tiles;
                for (int k = 0; k < KI; k++) {
                    if (!(ok = mbar_wait(&empty[stage], ph ^ 1, g.err, XTB_ERR_WAIT_TMA))) break;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES + C::SF_BYTES);
                    tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], k * 128, mb * 128);
                    tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], k * 128, nb * BN);
                    bulk_load(sSF + stage * C::SF_BYTES, mx.sf + ((size_t)k * mx.nbp + 2 * nb) * 512, C::SF_BYTES,
                              &full[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            const uint32_t sfa = tbase + C::SFA_COL;
            tmem_cp_32x128b_x4(sfa, sdesc_rows16(smem_u32(sSFA)));
            int stage = 0;
            uint32_t ph = 0, tph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int k = 0; k < KI; k++) {
                    if (k == 0) {
                        if (!(ok = mbar_wait(tempty, tph ^ 1, g.err, XTB_ERR_WAIT_TMEM))) break;
                        tc_fence_after();
                    }
                    if (!(ok = mbar_wait(&full[stage], ph, g.err, XTB_ERR_WAIT_TMA))) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t f0 = smem_u32(sSF + stage * C::SF_BYTES);
                    // the tensor core runs its copies and MMAs in issue order: this slice's MMAs read these scale
                    // factors after the previous slice's MMAs have read theirs
                    tmem_cp_32x128b_x4(tbase + C::SFB_COL, sdesc_rows16(f0));
                    tmem_cp_32x128b_x4(tbase + C::SFB_COL + 8, sdesc_rows16(f0 + 512));
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
#pragma unroll
                        for (int h = 0; h < 2; h++)
                            umma_mx(tbase + h * 128, sdesc(a0 + kk * 32, 1024, SWZ_128B),
                                    sdesc(b0 + h * 128 * 128 + kk * 32, 1024, SWZ_128B), idesc_mx_m128(128, kk, kk), sfa,
                                    tbase + C::SFB_COL + 8 * h, (k > 0 || kk > 0));
                    umma_commit(&empty[stage]);
                    if (k == KI - 1) {
                        umma_commit(tfull);
                        tph ^= 1;
                    }
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
        const int half = ew >> 2;
        EpiCtx cx;
        cx.lane = lane;
        cx.stage = sStage + ew * StagingOf<Epi>::v;
        cx.tmC = &tmC;
        uint32_t tph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            const int nb = t % g.n_tiles, mb = t / g.n_tiles;
            cx.row0 = mb * 128 + quad * 32;
            cx.col0 = nb * BN + half * COLS;
            typename Epi::State es;
            Epi::begin(ep, cx, es);
            const float s = g.ascale * Epi::col_scale(ep, cx);
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(tfull, tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
            tph ^= 1;
            tc_fence_after();
            const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + half * COLS;
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
                        if (lane == 0) mbar_arrive(tempty);
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
                if (lane == 0) mbar_arrive(tempty);
                Epi::apply(ep, (float *)acc, cx, es);
            }
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

}  // namespace xtb

// Block-scaled FP8 GEMM on CTA pairs (tcgen05 .cta_group::2) for sm_100a:  D[M][N] = epilogue( sum_k A[m][k] B[n][k] ).
//
// A cluster of two CTAs, placed by the hardware on the two SMs of one TPC, computes one 256 x 256 output tile. Rank r
// keeps rows 128 r .. 128 r + 127 of the tile's A rows and rows 128 r .. 128 r + 127 of its B rows in its own shared
// memory. Rank 0 issues one M = 256, N = 256 MMA for both: each SM's tensor core multiplies its own A rows by all
// 256 B rows (half of them read from the peer) and leaves its 128 x 256 block of the tile in its own TMEM. Against
// the single-CTA GEMM (gemm.cuh) each SM loads half as many B bytes per MMA through L2 and TMA (A 16 KB + B 16 KB
// per 128-deep K block instead of 16 + 32 KB): the GEMM whose operands stream from DRAM (fc2, K = 2736, A = the
// 180 MB SwiGLU output) is bound by that feed and runs a third faster this way. The epilogue side is that of the
// single-CTA GEMM: two TMEM buffers of 256 columns, 8 epilogue warps with 128 accumulator columns per thread.
// An MMA with N = 128 per SM would leave room for four TMEM buffers but reads shared memory faster than it can
// supply (about 20 % below the N = 256 rate, measured both with one CTA and with pairs).
// GROUPS (BN = 128): the four TMEM buffers go to two epilogue groups of four warps (one per lane quadrant, 128
// columns per thread) that take the pair's tiles in turn, each promoting into its own two buffers. While one group
// runs the fused apply phase of a tile from registers, the MMA keeps filling the other group's buffers, so the apply
// no longer stalls the main loop (with two buffers the MMA can run at most two K blocks ahead of the epilogue).
//
// Roles (320 threads per CTA):
//   warp 0      TMA producer of this CTA's A and B slices into a 6-stage ring. Completion is counted on rank 0's
//               `full` barrier (both producers arrive on it with their own byte counts).
//   warp 1      allocates TMEM (512 columns, both CTAs together); on rank 0 one lane issues the pair MMAs and
//               commits to `empty` (stage free) and `tfull` (K block done) in both CTAs at once.
//   warps 2..9  epilogue of this CTA's 128 rows: promotion of each K block's partial into fp32 registers
//               (acc += a_scale * w_scale[block] * partial), then the fused epilogue; each warp tells rank 0's
//               `tempty` barrier when it has read a TMEM buffer.
// Every wait is bounded (XTB_WAIT_NS); a wait that runs out sets the error word and the CTA winds down.
#pragma once
#include "gemm.cuh"

namespace xtb {

template <int BN_, bool GROUPS_ = false, int SPW_ = 4096>
struct Gemm2CfgT {
    static constexpr int BN = BN_;                          // output columns per tile
    static constexpr bool GROUPS = GROUPS_;
    static constexpr int EW = 8;                            // epilogue warps: 2 per TMEM lane quadrant
    static constexpr int COLS = GROUPS ? BN : BN / 2;       // accumulator columns per epilogue thread
    static constexpr int TEMPTY = GROUPS ? 2 * 4 : 2 * EW;  // arrivals that free a TMEM buffer (both CTAs)
    static constexpr int A_BYTES = 128 * 128;               // this CTA's 128 A rows x one 128-byte K slice
    static constexpr int B_BYTES = (BN / 2) * 128;          // this CTA's BN / 2 B rows
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE_PER_WARP = SPW_;             // epilogue staging per warp
    static constexpr int STAGING = EW * SPW_;
    static constexpr int STAGES = (7 * 32768 - STAGING) / STAGE_BYTES;  // the rest of 224 KB as ring (6 stages at 4 KB)
    static constexpr int TBUF = 512 / BN;                   // TMEM accumulator buffers
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + STAGING + 1024;  // + barriers
    static constexpr int THREADS = 64 + 32 * EW;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(!GROUPS || BN == 128, "grouped epilogue: four 128-column buffers");
};
using Gemm2Cfg = Gemm2CfgT<256>;
using Gemm2GCfg = Gemm2CfgT<128, true>;

template <class Epi, bool PROMOTE, int BN = 256, bool GROUPS = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2CfgT<BN, GROUPS>::THREADS, 1)
    k_gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmC, const GemmArgs g, const typename Epi::Params ep)
{
    using C = Gemm2CfgT<BN, GROUPS, StagingOf<Epi>::v>;
    static_assert(!GROUPS || PROMOTE, "the grouped epilogue promotes every K block");
    constexpr int STAGES = C::STAGES, TBUF = C::TBUF, COLS = C::COLS;
    constexpr uint32_t IDESC = idesc_m256(C::BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * C::A_BYTES;
    uint8_t *sStage = smem + STAGES * C::STAGE_BYTES;
    uint64_t *full = (uint64_t *)(sStage + C::STAGING);  // rank 0: both producers' bytes
    uint64_t *empty = full + STAGES;                     // every rank: stage consumed by the pair MMA
    uint64_t *tfull = empty + STAGES;                    // every rank: K block (or tile) accumulated in TMEM
    uint64_t *tempty = tfull + TBUF;                     // rank 0: TMEM buffer read by all 16 epilogue warps
    uint32_t *tslot = (uint32_t *)(tempty + TBUF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 2);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < TBUF; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], C::TEMPTY);
        }
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tslot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers are initialised before anyone arrives on them
    tc_fence_after();
    const uint32_t tbase = *tslot;
    const int total = g.m_tiles * g.n_tiles;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int KI = g.kiters;
    if (warp != 0) griddep_wait();  // the previous kernel of the stream has completed: activations may be touched

    if (warp == 0) {
        if (elect_one()) {
            const uint32_t full0 = mapa_shared(smem_u32(full), 0);
            // B is a weight (every launch passes one), never written by an earlier kernel: the first tile's first
            // ring slots get their B rows before the wait (first round: no consumer to wait for; the expected bytes
            // include A's), so their load latency overlaps the previous kernel's tail.
            const int pre = pair < total ? min(STAGES, KI) : 0;
            for (int k = 0; k < pre; k++) {
                const uint32_t fb = full0 + k * 8;
                mbar_arrive_expect_tx_cluster(fb, C::STAGE_BYTES);
                tma_load_2d_pair(sB + k * C::B_BYTES, &tmB, fb, k * 128, (pair % g.n_tiles) * C::BN + rank * (C::BN / 2));
            }
            griddep_wait();
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair; t < total && ok; t += npairs) {
                const int nb = t % g.n_tiles, mb = t / g.n_tiles;  // N fastest: an A tile is read by neighbours
                for (int k = 0; k < KI; k++) {
                    const bool early = t == pair && k < pre;  // B already on its way
                    const uint32_t fb = full0 + stage * 8;
                    if (!early) {
                        if (!(ok = mbar_wait(&empty[stage], ph ^ 1, g.err, XTB_ERR_WAIT_TMA))) break;
                        mbar_arrive_expect_tx_cluster(fb, C::STAGE_BYTES);
                    }
                    tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, fb, k * 128, mb * 256 + rank * 128);
                    if (!early)
                        tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, fb, k * 128, nb * C::BN + rank * (C::BN / 2));
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (rank == 0 && elect_one()) {
            int stage = 0;
            uint32_t ph = 0, tb = 0, tph = 0, cnt[2] = {0, 0};
            bool ok = true;
            for (int t = pair, i = 0; t < total && ok; t += npairs, i++) {
                for (int k = 0; k < KI; k++) {
                    if (GROUPS) {  // group i & 1 owns buffers 2 (i & 1) and 2 (i & 1) + 1, used in turn per K block
                        const uint32_t c = cnt[i & 1]++;
                        tb = 2 * (i & 1) + (c & 1);
                        tph = (c >> 1) & 1;
                    }
                    if (PROMOTE || k == 0) {
                        if (!(ok = mbar_wait(&tempty[tb], tph ^ 1, g.err, XTB_ERR_WAIT_TMEM))) break;
                        tc_fence_after();
                    }
                    if (!(ok = mbar_wait(&full[stage], ph, g.err, XTB_ERR_WAIT_TMA))) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t d = tbase + tb * C::BN;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma_pair_e4m3(d, sdesc(a0 + kk * 32, 1024, SWZ_128B), sdesc(b0 + kk * 32, 1024, SWZ_128B), IDESC,
                                       PROMOTE ? (kk > 0) : (k > 0 || kk > 0));
                    umma_commit_pair(&empty[stage], 0x3);
                    if (PROMOTE || k == KI - 1) {
                        umma_commit_pair(&tfull[tb], 0x3);
                        if (!GROUPS && ++tb == TBUF) {
                            tb = 0;
                            tph ^= 1;
                        }
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
        const int half = ew >> 2;  // which COLS-wide half of the tile (GROUPS: which epilogue group)
        const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
        EpiCtx cx;
        cx.lane = lane;
        cx.stage = sStage + ew * C::STAGE_PER_WARP;
        cx.tmC = &tmC;
        uint32_t tb = 0, tph = 0, c = 0;
        bool ok = true;
        for (int t = pair + (GROUPS ? half * npairs : 0); t < total && ok; t += (GROUPS ? 2 : 1) * npairs) {
            const int nb = t % g.n_tiles, mb = t / g.n_tiles;
            cx.row0 = mb * 256 + rank * 128 + quad * 32;
            cx.col0 = nb * C::BN + (GROUPS ? 0 : half * COLS);
            typename Epi::State es;
            Epi::begin(ep, cx, es);  // per-tile loads issued before the accumulator is ready
            if constexpr (!PROMOTE && !GROUPS && StreamOf<Epi>::v) {  // streaming epilogue (gemm.cuh)
                static_assert(COLS % 32 == 0, "streaming epilogues take 32-column chunks");
                const float s = g.ascale * Epi::col_scale(ep, cx) * g.wsu;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[tb], tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
                tc_fence_after();
                const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + tb * C::BN + half * COLS;
                float v[2][32];
                tmem_ld16(taddr, v[0]);
                tmem_ld16(taddr + 16, v[0] + 16);
#pragma unroll
                for (int c = 0; c < COLS / 32; c++) {
                    tmem_wait_ld_regs(v[c & 1]);
                    if (c + 1 < COLS / 32) {
                        tmem_ld16(taddr + 32 * (c + 1), v[(c + 1) & 1]);
                        tmem_ld16(taddr + 32 * (c + 1) + 16, v[(c + 1) & 1] + 16);
                    } else {  // the whole buffer is in registers: hand it back to the MMA
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(tempty0 + tb * 8);
                    }
                    Epi::apply_chunk(ep, v[c & 1], s, c, cx, es);
                }
                if (++tb == TBUF) {
                    tb = 0;
                    tph ^= 1;
                }
                Epi::finish(ep, cx, es);
                continue;
            }
            float2 acc[COLS / 2];
#pragma unroll
            for (int j = 0; j < COLS / 2; j++) acc[j] = make_float2(0.f, 0.f);
            const int units = PROMOTE ? KI : 1;
            const float *wsr = nullptr;
            if (PROMOTE) wsr = g.ws + (size_t)min(cx.col0 >> 7, g.ws_rows - 1) * g.ws_ld;
            float snext = PROMOTE ? __ldg(wsr) : 1.0f;
            const float amul = g.ascale * Epi::col_scale(ep, cx);
            for (int u = 0; u < units; u++) {
                const float s = PROMOTE ? amul * snext : amul * g.wsu;
                if (PROMOTE && u + 1 < units) snext = __ldg(wsr + u + 1);
                if (GROUPS) {
                    tb = 2 * half + (c & 1);
                    tph = (c >> 1) & 1;
                    c++;
                }
                // warp-uniform outcome: the tcgen05.ld below is a .sync.aligned warp instruction
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[tb], tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
                tc_fence_after();
                const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + tb * C::BN + (GROUPS ? 0 : half * COLS);
                const float2 s2 = make_float2(s, s);
                constexpr int CH = COLS <= 64 ? COLS : 32;  // columns per tcgen05.wait::ld
#pragma unroll
                for (int c0 = 0; c0 < COLS; c0 += CH) {
                    float v[CH];
#pragma unroll
                    for (int c = 0; c < CH / 16; c++) tmem_ld16(taddr + c0 + c * 16, v + 16 * c);
                    tmem_wait_ld();
                    if (c0 + CH == COLS) {  // the whole buffer is in registers: hand it back to the MMA
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(tempty0 + tb * 8);
                    }
#pragma unroll
                    for (int j = 0; j < CH / 2; j++) {
                        const float2 vv = make_float2(v[2 * j], v[2 * j + 1]);
                        if (PROMOTE) acc[c0 / 2 + j] = ffma2(s2, vv, acc[c0 / 2 + j]);
                        else acc[c0 / 2 + j] = mul2(s2, vv);
                    }
                }
                if (!GROUPS && ++tb == TBUF) {
                    tb = 0;
                    tph ^= 1;
                }
            }
            if (!ok) break;
            Epi::apply(ep, (float *)acc, cx, es);
        }
        if (lane == 0) bulk_wait0();  // the epilogue's TMA stores / reductions have completed
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

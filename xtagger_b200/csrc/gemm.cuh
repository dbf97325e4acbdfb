// Block-scaled FP8 (and fp16) GEMM on tcgen05 for sm_100a:  D[M][N] = epilogue( sum_k A[m][k] * B[n][k] ).
//
// One persistent CTA per SM walks output tiles of 128 x BN. Warp roles (320 threads):
//   warp 0      TMA producer: 128-byte-wide K slices of A (128 rows) and B (BN rows), 128B-swizzled, into a
//               STAGES-deep shared-memory ring guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (512 columns) and one elected lane issues tcgen05.mma (M = 128, N = BN, K = 32 bytes
//               per instruction, 4 instructions per 128-byte slice).
//   warps 2..9  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes 32 (w % 4) ..; two warps per lane
//               quadrant split the BN columns), apply the fused epilogue, store through a per-warp 4 KB staging
//               buffer so that global stores are whole 128-byte rows (or 32-byte sectors) per warp instruction.
//
// PROMOTE (FP8 weights with one fp32 scale per 128 x 128 block): every 128-element K block is accumulated into its
// own TMEM buffer (two buffers of BN columns, ping-pong), and the epilogue warps fold it into fp32 registers with
// acc += (a_scale * w_scale[block]) * partial (packed fma.rn.f32x2). This keeps the dequantize-then-matmul
// semantics exactly (scales are arbitrary fp32, not powers of two) while the tensor core runs the next K block into
// the other buffer. Without PROMOTE the whole K range accumulates in one TMEM buffer and is scaled once by
// a_scale * wsu (a weight with one scale for the whole tensor, as the reference's v3 format, or 1 for fp16); the
// buffers ping-pong across tiles so that the epilogue of one tile overlaps the main loop of the next.
#pragma once
#include "ptx.cuh"

namespace xtb {

struct GemmArgs {
    int M, N;            // output rows / columns (rows of A / rows of B)
    int kiters;          // 128-byte K slices (ceil(K bytes / 128))
    int m_tiles, n_tiles;
    const float *ws;     // PROMOTE: block scales [ws_rows][ws_ld]; row = N block (or M block when WS_ON_M)
    int ws_ld, ws_rows;
    float ascale;        // activation dequant scale, folded into every block scale (or into wsu)
    float wsu;           // without PROMOTE: the one weight scale of the tensor (1 for unscaled fp16 operands)
    uint32_t *err;       // library error word
    int b_weight;        // single-CTA kernel: B is a weight (never written by an earlier kernel), prefetchable
};

template <int BN, int EW = 8>
struct GemmCfg {
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (6 * 32768) / STAGE_BYTES;  // 192 KB of ring: 4 stages at BN 256 / 192, 6 at 128
    static constexpr int EPI_WARPS = EW;   // epilogue warps: EW / 4 per TMEM lane quadrant
    static constexpr int COLS = BN / (EW / 4);  // accumulator columns per epilogue thread
    static constexpr int TBUF = 512 / BN;  // TMEM accumulator buffers (512 columns in all)
    static constexpr int STAGE_PER_WARP = 4096;  // staging bytes per epilogue warp
    static constexpr int STAGING = EW * STAGE_PER_WARP;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + STAGING + 512;  // + barriers
    static constexpr int THREADS = 64 + 32 * EW;
    static_assert(SMEM <= 232448, "shared memory budget");
};

// Staging bytes per epilogue warp an epilogue asks for (Epi::STAGING_PER_WARP), 4 KB by default. The CTA-pair GEMM
// sizes its staging from it; this kernel has 4 KB per warp and accepts only epilogues that fit.
template <class E, class = void>
struct StagingOf {
    static constexpr int v = 4096;
};
template <class E>
struct StagingOf<E, decltype((void)E::STAGING_PER_WARP)> {
    static constexpr int v = E::STAGING_PER_WARP;
};

// Streaming epilogues (Epi::STREAM, per-tensor weights only): the accumulator is handed over 32 columns at a time,
// apply_chunk(params, raw[32], scale, chunk, ctx, state), as soon as each chunk's TMEM load has landed, with the
// next chunk's load already in flight; finish(params, ctx, state) after the last chunk. No COLS-wide register copy
// of the accumulator, and the TMEM load latency hides behind the previous chunk's math.
template <class E, class = void>
struct StreamOf {
    static constexpr bool v = false;
};
template <class E>
struct StreamOf<E, decltype((void)E::STREAM)> {
    static constexpr bool v = E::STREAM;
};

// Epilogues with apply_last(params, acc[COLS], ctx, state, wide) (Epi::LAST_WIDE): on a CTA's last tile the
// operand ring is idle once the final accumulator is ready, and each epilogue warp gets 32 x COLS x 4 bytes of it
// (`wide`) to stage its whole slice at once. The accumulator registers are then free for the stores, which no
// longer run one latency-bound iteration at a time.
template <class E, class = void>
struct LastWideOf {
    static constexpr bool v = false;
};
template <class E>
struct LastWideOf<E, decltype((void)E::LAST_WIDE)> {
    static constexpr bool v = E::LAST_WIDE;
};

// Epilogue context of one thread: output row row0 + lane, columns col0 .. col0 + COLS - 1.
struct EpiCtx {
    int row0;        // first row of this warp's 32 rows
    int col0;
    int lane;
    uint8_t *stage;  // this warp's 4 KB staging buffer: 32 rows x 128 bytes, 16-byte chunks XOR-swizzled by row
    const CUtensorMap *tmC;  // the epilogue's output tensor map (TMA stores / reductions), when it has one
};

// Epilogues without per-tile state use this.
struct NoState {};

// Staging helpers. Row r's 16-byte chunk c sits at r * 128 + ((c ^ (r & 7)) * 16): a warp writing one row per lane
// and a warp reading one row across lanes are both free of bank conflicts.
__device__ __forceinline__ uint8_t *stage_chunk(uint8_t *st, int r, int c) { return st + r * 128 + (((c ^ (r & 7)) & 7) << 4); }
__device__ __forceinline__ void stage_row_f32(uint8_t *st, int lane, const float *v)
{
#pragma unroll
    for (int c = 0; c < 8; c++)
        *(float4 *)stage_chunk(st, lane, c) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
__device__ __forceinline__ float stage_f32(uint8_t *st, int r, int w) { return *(const float *)(stage_chunk(st, r, w >> 2) + ((w & 3) << 2)); }
__device__ __forceinline__ float2 stage_f32x2(uint8_t *st, int r, int w) { return *(const float2 *)(stage_chunk(st, r, w >> 2) + ((w & 3) << 2)); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
{
    uint64_t d = *reinterpret_cast<uint64_t *>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)));
    return *reinterpret_cast<float2 *>(&d);
}

// With 8 epilogue warps (320 threads) three warps share two of the SM's four sub-partitions (16K registers
// each): at most 168 registers per thread; with 16 (576 threads) five share one: at most 96.
template <class Epi, int BN, bool F16, bool PROMOTE, bool WS_ON_M, int EW = 8>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmC, const GemmArgs g, const typename Epi::Params ep)
{
    using C = GemmCfg<BN, EW>;
    static_assert(StagingOf<Epi>::v <= C::STAGE_PER_WARP, "epilogue staging larger than this kernel provides");
    constexpr int STAGES = C::STAGES;
    constexpr int COLS = C::COLS;
    constexpr uint32_t IDESC = idesc_m128(BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * C::A_BYTES;
    uint8_t *sStage = smem + STAGES * C::STAGE_BYTES;
    uint64_t *full = (uint64_t *)(sStage + C::STAGING);
    uint64_t *empty = full + STAGES;
    constexpr int TBUF = C::TBUF;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + TBUF;
    uint32_t *tslot = (uint32_t *)(tempty + TBUF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < TBUF; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EW);
        }
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
    const int total = g.m_tiles * g.n_tiles;
    const int KI = g.kiters;
    if (warp != 0) griddep_wait();  // the previous kernel of the stream has completed: activations may be touched

    if (warp == 0) {
        if (elect_one()) {
            // When B is a weight (g.b_weight), the first tile's first ring slots get their B rows before the wait
            // (first round: no consumer to wait for; the expected bytes include A's), so that their load latency
            // overlaps the previous kernel's tail.
            const int pre = (g.b_weight && (int)blockIdx.x < total) ? min(STAGES, KI) : 0;
            for (int k = 0; k < pre; k++) {
                mbar_arrive_expect_tx(&full[k], C::STAGE_BYTES);
                tma_load_2d(sB + k * C::B_BYTES, &tmB, &full[k], k * 128, ((int)blockIdx.x % g.n_tiles) * BN);
            }
            griddep_wait();
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const int nb = t % g.n_tiles, mb = t / g.n_tiles;  // N fastest: an A tile is read by neighbours
                for (int k = 0; k < KI; k++) {
                    const bool early = t == (int)blockIdx.x && k < pre;  // B already on its way
                    if (!early) {
                        if (!(ok = mbar_wait(&empty[stage], ph ^ 1, g.err, XTB_ERR_WAIT_TMA))) break;
                        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    }
                    tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], k * 128, mb * 128);
                    if (!early) tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], k * 128, nb * BN);
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            int stage = 0;
            uint32_t ph = 0, tb = 0, tph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int k = 0; k < KI; k++) {
                    if (PROMOTE || k == 0) {
                        if (!(ok = mbar_wait(&tempty[tb], tph ^ 1, g.err, XTB_ERR_WAIT_TMEM))) break;
                        tc_fence_after();
                    }
                    if (!(ok = mbar_wait(&full[stage], ph, g.err, XTB_ERR_WAIT_TMA))) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t d = tbase + tb * BN;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma<F16>(d, sdesc(a0 + kk * 32, 1024, SWZ_128B), sdesc(b0 + kk * 32, 1024, SWZ_128B), IDESC,
                                  PROMOTE ? (kk > 0) : (k > 0 || kk > 0));
                    umma_commit(&empty[stage]);
                    if (PROMOTE || k == KI - 1) {
                        umma_commit(&tfull[tb]);
                        if (++tb == TBUF) {
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
        const int half = ew >> 2;  // which COLS-wide column slice of the tile
        EpiCtx cx;
        cx.lane = lane;
        cx.stage = sStage + ew * C::STAGE_PER_WARP;
        cx.tmC = &tmC;
        uint32_t tb = 0, tph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            const int nb = t % g.n_tiles, mb = t / g.n_tiles;  // N fastest: an A tile is read by neighbours
            cx.row0 = mb * 128 + quad * 32;
            cx.col0 = nb * BN + half * COLS;
            typename Epi::State es;
            Epi::begin(ep, cx, es);  // per-tile loads issued before the accumulator is ready
            if constexpr (!PROMOTE && StreamOf<Epi>::v) {
                static_assert(COLS % 32 == 0, "streaming epilogues take 32-column chunks");
                const float s = g.ascale * Epi::col_scale(ep, cx) * g.wsu;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[tb], tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
                tc_fence_after();
                const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + tb * BN + half * COLS;
                float v[2][32];
                tmem_ld16(taddr, v[0]);
                tmem_ld16(taddr + 16, v[0] + 16);
#pragma unroll
                for (int c = 0; c < COLS / 32; c++) {
                    tmem_wait_ld_regs(v[c & 1]);
                    if (c + 1 < COLS / 32) {
                        tmem_ld16(taddr + 32 * (c + 1), v[(c + 1) & 1]);
                        tmem_ld16(taddr + 32 * (c + 1) + 16, v[(c + 1) & 1] + 16);
                    } else {  // every chunk is in registers: the buffer goes back to the MMA warp
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[tb]);
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
            if (PROMOTE) wsr = g.ws + (size_t)min(WS_ON_M ? mb : (cx.col0 >> 7), g.ws_rows - 1) * g.ws_ld;
            float snext = PROMOTE ? __ldg(wsr) : 1.0f;
            const float amul = g.ascale * Epi::col_scale(ep, cx);  // activation dequant x the epilogue's own factor
            for (int u = 0; u < units; u++) {
                const float s = PROMOTE ? amul * snext : amul * g.wsu;
                if (PROMOTE && u + 1 < units) snext = __ldg(wsr + u + 1);
                // warp-uniform outcome: the tcgen05.ld below is a .sync.aligned warp instruction
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[tb], tph, g.err, XTB_ERR_WAIT_TMEM)))) break;
                tc_fence_after();
                const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + tb * BN + half * COLS;
                const float2 s2 = make_float2(s, s);
                constexpr int CH = COLS >= 32 ? 32 : COLS;  // columns per tcgen05.wait::ld
#pragma unroll
                for (int c0 = 0; c0 < COLS; c0 += CH) {
                    float v[CH];
#pragma unroll
                    for (int c = 0; c < CH / 16; c++) tmem_ld16(taddr + c0 + c * 16, v + 16 * c);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < CH / 2; j++) {
                        const float2 vv = make_float2(v[2 * j], v[2 * j + 1]);
                        if (PROMOTE) acc[c0 / 2 + j] = ffma2(s2, vv, acc[c0 / 2 + j]);
                        else acc[c0 / 2 + j] = mul2(s2, vv);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[tb]);
                if (++tb == TBUF) {
                    tb = 0;
                    tph ^= 1;
                }
            }
            if (!ok) break;
            if constexpr (LastWideOf<Epi>::v) {
                static_assert((size_t)STAGES * C::STAGE_BYTES >= (size_t)EW * 32 * COLS * 4, "ring too small to stage");
                if (t + (int)gridDim.x >= total) {  // last tile: every MMA has read its operands, no load follows
                    Epi::apply_last(ep, (float *)acc, cx, es, smem + (size_t)ew * 32 * COLS * 4);
                    continue;
                }
            }
            Epi::apply(ep, (float *)acc, cx, es);
        }
        if (lane == 0) bulk_wait0();  // the epilogue's TMA stores / reductions have completed
        __syncwarp();
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Epilogues: apply(params, acc[COLS], ctx). acc holds output row ctx.row0 + lane, columns ctx.col0 .. + COLS - 1
// (already dequantised when the GEMM promotes block scales). Rows / columns past the problem are skipped.
// ---------------------------------------------------------------------------------------------------------------

// Plain fp32 store: out[row][col] (row stride ld floats). Used for the stand-alone block-scaled GEMM.
template <int COLS>
struct EpiF32 {
    struct Params {
        float *out;
        int ld, M, N;
    };
    using State = NoState;
    __device__ __forceinline__ static float col_scale(const Params &, const EpiCtx &) { return 1.0f; }
    __device__ __forceinline__ static void begin(const Params &, const EpiCtx &, State &) {}
    // Each 32 x 32 chunk goes out through the staging buffer, a warp store covering two rows (half a warp per row,
    // two columns per lane): with an even row stride and an 8-byte aligned output (the usual case: N = 2730 gives
    // 10,920-byte rows, 8- but not 16-byte aligned) one float2 store per lane, half as many store instructions as
    // one float per lane; otherwise two float stores.
    __device__ __forceinline__ static void apply(const Params &p, const float *acc, const EpiCtx &cx, State &)
    {
        const bool pairs = (p.ld & 1) == 0 && ((uintptr_t)p.out & 7) == 0;
        const int rr = cx.lane >> 4, cc = (cx.lane & 15) * 2;
#pragma unroll
        for (int c = 0; c < COLS / 32; c++) {
            __syncwarp();
            stage_row_f32(cx.stage, cx.lane, acc + 32 * c);
            __syncwarp();
            const int col = cx.col0 + 32 * c + cc;
            if (col < p.N) {
#pragma unroll 4
                for (int i = 0; i < 16; i++) {
                    const int row = cx.row0 + 2 * i + rr;
                    if (row < p.M) {
                        const float2 v = stage_f32x2(cx.stage, 2 * i + rr, cc);
                        float *o = p.out + (size_t)row * p.ld + col;
                        if (pairs && col + 1 < p.N) {
                            *(float2 *)o = v;
                        } else {
                            o[0] = v.x;
                            if (col + 1 < p.N) o[1] = v.y;
                        }
                    }
                }
            }
        }
        __syncwarp();
    }

    // Last tile: the warp's 32 x COLS slice goes to `wide` (row r at r * COLS * 4 bytes, its 16-byte chunks
    // XOR-swizzled by r & 7: conflict-free both for one row per lane and for whole rows across the warp), then out
    // with 32 / (COLS / 4) rows per warp instruction, four columns per lane: a float4 where the row's first column is
    // 16-byte aligned, else two float2 or, for an odd row stride or an unaligned output, floats. Eight instructions'
    // loads are in flight before their stores.
    static constexpr bool LAST_WIDE = true;
    __device__ __forceinline__ static uint8_t *wide_chunk(uint8_t *w, int r, int c)
    {
        return w + r * (COLS * 4) + ((c ^ (r & 7)) << 4);  // the XOR stays inside c's aligned group of 8 chunks
    }
    __device__ __forceinline__ static void apply_last(const Params &p, const float *acc, const EpiCtx &cx, State &,
                                                      uint8_t *wide)
    {
        static_assert(COLS % 32 == 0, "whole 32-column groups");
        constexpr int GC = (COLS == 64 || COLS == 128) ? COLS : 32;  // columns a lane group covers in one row
        constexpr int LPR = GC / 4;     // lanes per row
        constexpr int RPI = 32 / LPR;   // rows per instruction
        __syncwarp();
#pragma unroll
        for (int c = 0; c < COLS / 4; c++)
            *(float4 *)wide_chunk(wide, cx.lane, c) = make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
        __syncwarp();
        const bool al8 = (p.ld & 1) == 0 && ((uintptr_t)p.out & 7) == 0;
        const bool out16 = ((uintptr_t)p.out & 15) == 0;
        const int sub = cx.lane / LPR;
#pragma unroll 1
        for (int q = 0; q < COLS / GC; q++) {
        const int ch = q * LPR + cx.lane % LPR;  // the lane's 16-byte chunk of the row
        const int col = cx.col0 + 4 * ch;
#pragma unroll 1
        for (int i0 = 0; i0 < 32; i0 += 8 * RPI) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = *(const float4 *)wide_chunk(wide, i0 + i * RPI + sub, ch);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int row = cx.row0 + i0 + i * RPI + sub;
                if (row >= p.M || col >= p.N) continue;
                float *o = p.out + (size_t)row * p.ld + col;
                const uint32_t e = (uint32_t)row * (uint32_t)p.ld + (uint32_t)cx.col0;  // low bits of the row's first element offset
                if (col + 3 < p.N && out16 && (e & 3) == 0) {
                    *(float4 *)o = v[i];
                } else if (col + 3 < p.N && al8) {
                    *(float2 *)o = make_float2(v[i].x, v[i].y);
                    *(float2 *)(o + 2) = make_float2(v[i].z, v[i].w);
                } else {
                    o[0] = v[i].x;
                    if (col + 1 < p.N) o[1] = v[i].y;
                    if (col + 2 < p.N) o[2] = v[i].z;
                    if (col + 3 < p.N) o[3] = v[i].w;
                }
            }
        }
        }
        __syncwarp();
    }
};

}  // namespace xtb

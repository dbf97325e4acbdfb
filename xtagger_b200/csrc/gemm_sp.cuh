// 2:4-sparse block-scaled FP8 GEMM on tcgen05.mma.sp (sm_100a), the weights as the sparse operand:
//     D[n][t] = epilogue( sum_k W[n][k] * X[t][k] )        n: weight row (output feature), t: token
// tcgen05 takes sparsity on the A operand only, so the weights are A (128 rows per tile, one per TMEM lane) and the
// activations are B (SP_BT = 112 tokens per tile, TMEM columns): the accumulator holds the transposed output. The
// epilogues below are the transposed forms of those in epilogues.cuh, with the same arithmetic per (token,
// feature), so that on pruned weights this path reproduces the dense one (the reference runs pruned weights,
// prune24.py's output, through its dense kernels: this is the same product on the sparse tensor-core path).
//
// Weight format (sparse24_compress, sparse24.cu): values [Np][Kp / 2] = the two kept bytes of every group of four
// consecutive k, in k order; metadata [Np][Kp / 8] = per group the in-group index of the first kept byte in bits
// 0-1 and of the second in bits 2-3 (first < second), groups in k order, two per byte, low nibble first. Np and Kp
// are padded to multiples of 128 (padding groups: zero values, indices 0 and 1). This is the layout
// tcgen05.mma.sp reads for kind::f8f6f4 at M = 128: metadata row n in TMEM lane n, 16 bytes (4 columns) per
// 128 k, 2 columns per K = 64 instruction.
//
// Pipeline stage = one 128-element K block (one block scale): 128 weight rows x 64 value bytes (64B swizzle),
// 128 x 16 metadata bytes (unswizzled), 112 tokens x 128 activation bytes (128B swizzle).
// Warps (320 threads): 0 TMA producer; 1 TMEM allocation and MMA issue (tcgen05.cp of the stage's metadata into
// TMEM, then two K = 64 sparse MMAs); 2..9 epilogue, as two groups of four warps (one per TMEM lane quadrant,
// warp w reads lanes 32 (w % 4) ..) that take the CTA's tiles in turn: while one group runs a tile's epilogue (the
// fused apply phase, from registers), the MMA fills the other group's accumulators, so the apply overlaps the main
// loop instead of stalling it. Block scales are promoted per K block as gemm.cuh does.
// TMEM: four accumulators of 112 columns (group g: 2g and 2g + 1, ping-pong per K block) at [0, 448), metadata at
// 448 and 452 (ping-pong per K block; a metadata column must be even).
// Without PROMOTE (a weight with one scale for the whole tensor, as prune24.py writes the reference's v3 files) a
// tile accumulates its whole K range in one of its group's two buffers, which then ping-pong per tile: the group
// drains and scales the tile once, and its apply overlaps both the other group's tile and its own next tile.
#pragma once
#include "gemm.cuh"
#include "ops.h"

namespace xtb {

constexpr int SP_BT = 112;          // tokens per tile (MMA N)
constexpr int SP_COLS = SP_BT;      // token columns per epilogue thread (a group's four warps cover a tile)

struct SpCfg {
    static constexpr int A_BYTES = 128 * 64;
    static constexpr int E_BYTES = 128 * 16;
    static constexpr int B_BYTES = SP_BT * 128;
    static constexpr int STAGE_BYTES = A_BYTES + E_BYTES + B_BYTES;
    static constexpr int STAGES = 6;
    static constexpr int EW = 8;
    static constexpr int STAGE_PER_WARP = SP_COLS * 64;      // epilogue scratch per warp: 112 tokens x 64 bytes
    static constexpr int XRED_FLOAT2 = 2 * 2 * 4 * SP_COLS;  // fc1 statistics exchange [group][buffer][quad][token]
    static constexpr int E_COL = 4 * SP_BT;                  // metadata TMEM columns (two buffers of 4)
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + EW * STAGE_PER_WARP + XRED_FLOAT2 * 8 + 256;
    static constexpr int THREADS = 64 + 32 * EW;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(E_COL + 8 <= 512, "TMEM budget");
    static_assert(SP_COLS % 16 == 0, "epilogue drains 16 columns at a time");
    static_assert(B_BYTES % 1024 == 0, "128B-swizzled stages stay 1024-byte aligned");
};

struct SpArgs {
    int M;            // tokens
    int kiters;       // 128-element K blocks
    int n_tiles, t_tiles;
    const float *ws;  // block scales [ws_rows][ws_ld] (row = 128-row weight block)
    int ws_ld, ws_rows;
    float ascale;     // activation dequant scale
    float wsu;        // without PROMOTE: the weight's one scale
    uint32_t *err;
};

// Epilogue context of one thread: weight row (feature) f0 + lane, tokens t0 .. t0 + SP_COLS - 1.
struct SpCtx {
    int f0, t0, nb, lane, quad;
    uint8_t *stage;            // this warp's scratch (STAGE_PER_WARP bytes)
    uint8_t *gscratch;         // this group's scratch (its four warps' slices, contiguous)
    float2 *xred;              // this group's exchange buffers [2][4][SP_COLS]
    uint64_t *ebar;            // this group's four epilogue barriers (meaning set by the epilogue)
    uint32_t use;              // epilogue-defined counter (exchanges / prefetches done by this warp)
    const CUtensorMap *tmC;
    uint32_t *err;
};

// Epilogues without barriers or per-tile prefetch.
struct SpNoBars {
    __device__ __forceinline__ static void init_bars(uint64_t *) {}
};

template <class Epi, bool PROMOTE = true>
__global__ void __launch_bounds__(SpCfg::THREADS, 1)
    k_gemm_sp(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmE,
              const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC, const SpArgs g,
              const typename Epi::Params ep)
{
    using C = SpCfg;
    constexpr int STAGES = C::STAGES;
    constexpr uint32_t IDESC = idesc_sp_m128(SP_BT);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sA = smem;                       // weight values: 64B-swizzle atoms (512 bytes) need 512-byte alignment
    uint8_t *sB = sA + STAGES * C::A_BYTES;   // activations: 128B swizzle, 1024-byte aligned (14 KB per stage)
    uint8_t *sE = sB + STAGES * C::B_BYTES;   // metadata
    uint8_t *sEpi = sE + STAGES * C::E_BYTES;
    float2 *xred = (float2 *)(sEpi + C::EW * C::STAGE_PER_WARP);
    uint64_t *full = (uint64_t *)(xred + C::XRED_FLOAT2);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;         // [4] accumulators
    uint64_t *tempty = tfull + 4;
    uint64_t *ebar = tempty + 4;              // [group][4]
    uint32_t *tslot = (uint32_t *)(ebar + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 4; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);  // the four warps of the group that owns the accumulator
        }
        Epi::init_bars(ebar);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmE);
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
    const int total = g.n_tiles * g.t_tiles;
    const int KI = g.kiters;

    if (warp == 0) {
        if (elect_one()) {
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                // weight tiles fastest: the CTAs working at one time share a few token tiles (read from DRAM once,
                // then from L2), and every layer's weights fit in L2
                const int nb = t % g.n_tiles, tt = t / g.n_tiles;
                for (int k = 0; k < KI; k++) {
                    if (!(ok = mbar_wait(&empty[stage], ph ^ 1, g.err, XTB_ERR_WAIT_TMA))) break;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], k * 64, nb * 128);
                    tma_load_2d(sE + stage * C::E_BYTES, &tmE, &full[stage], k * 16, nb * 128);
                    tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], k * 128, tt * SP_BT);
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
            uint32_t ph = 0, eb = 0, cnt[2] = {0, 0};  // K blocks issued into each group's accumulators
            bool ok = true;
            for (int t = blockIdx.x, i = 0; t < total && ok; t += gridDim.x, i++) {
                const int grp = i & 1;
                for (int k = 0; k < KI; k++) {
                    const uint32_t c = cnt[grp];
                    const int buf = 2 * grp + (int)(c & 1);
                    if (PROMOTE || k == 0) {
                        if (!(ok = mbar_wait(&tempty[buf], ((c >> 1) & 1) ^ 1, g.err, XTB_ERR_WAIT_TMEM))) break;
                        tc_fence_after();
                    }
                    if (!(ok = mbar_wait(&full[stage], ph, g.err, XTB_ERR_WAIT_TMA))) break;
                    tc_fence_after();
                    const uint32_t ecol = tbase + C::E_COL + 4 * eb;
                    tmem_cp_128x128b(ecol, sdesc_rows16(smem_u32(sE + stage * C::E_BYTES)));
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t d = tbase + buf * SP_BT;
#pragma unroll
                    for (int kk = 0; kk < 2; kk++)
                        umma_sp(d, sdesc(a0 + kk * 32, 512, SWZ_64B), sdesc(b0 + kk * 64, 1024, SWZ_128B), ecol + 2 * kk,
                                IDESC, PROMOTE ? (kk > 0) : (k > 0 || kk > 0));
                    umma_commit(&empty[stage]);
                    eb ^= 1;
                    if (PROMOTE || k == KI - 1) {
                        umma_commit(&tfull[buf]);
                        cnt[grp] = c + 1;
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
        const int grp = ew >> 2;  // epilogue group: tiles grp, grp + 2, ... of this CTA
        SpCtx cx;
        cx.lane = lane;
        cx.quad = quad;
        cx.stage = sEpi + ew * C::STAGE_PER_WARP;
        cx.gscratch = sEpi + grp * 4 * C::STAGE_PER_WARP;
        cx.xred = xred + grp * (2 * 4 * SP_COLS);
        cx.ebar = ebar + 4 * grp;
        cx.use = 0;
        cx.tmC = &tmC;
        cx.err = g.err;
        uint32_t c = 0;  // K blocks drained by this group
        bool ok = true;
        for (int t = blockIdx.x + grp * gridDim.x; t < total && ok; t += 2 * gridDim.x) {
            const int nb = t % g.n_tiles, tt = t / g.n_tiles;
            cx.nb = nb;
            cx.f0 = nb * 128 + quad * 32;
            cx.t0 = tt * SP_BT;
            if (!(ok = Epi::begin(ep, cx))) break;  // per-tile loads issued before the accumulator is ready
            float2 acc[SP_COLS / 2];
#pragma unroll
            for (int j = 0; j < SP_COLS / 2; j++) acc[j] = make_float2(0.f, 0.f);
            const float *wsr = PROMOTE ? g.ws + (size_t)min(nb, g.ws_rows - 1) * g.ws_ld : nullptr;
            float snext = PROMOTE ? __ldg(wsr) : g.wsu;
            const float amul = g.ascale * Epi::row_scale(ep, cx.f0);
            const int units = PROMOTE ? KI : 1;
            for (int u = 0; u < units; u++, c++) {
                const float s = amul * snext;
                if (PROMOTE && u + 1 < units) snext = __ldg(wsr + u + 1);
                const int buf = 2 * grp + (int)(c & 1);
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&tfull[buf], (c >> 1) & 1, g.err, XTB_ERR_WAIT_TMEM)))) break;
                tc_fence_after();
                const uint32_t taddr = tbase + ((uint32_t)(quad * 32) << 16) + buf * SP_BT;
                const float2 s2 = make_float2(s, s);
#pragma unroll
                for (int cc = 0; cc < SP_COLS / 16; cc++) {
                    float v[16];
                    tmem_ld16(taddr + cc * 16, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        acc[cc * 8 + j] = PROMOTE ? ffma2(s2, make_float2(v[2 * j], v[2 * j + 1]), acc[cc * 8 + j])
                                                  : mul2(s2, make_float2(v[2 * j], v[2 * j + 1]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            if (!ok) break;
            ok = Epi::apply(ep, (const float *)acc, cx);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // no copy of an abandoned prefetch outlives the CTA
        if (lane == 0) bulk_wait0();                        // the epilogue's TMA stores / reductions have completed
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
// Transposed epilogues: begin(params, ctx) when a tile starts (before its accumulator is ready), apply(params,
// acc[SP_COLS], ctx) when it is complete: acc[j] = output (token ctx.t0 + j, feature ctx.f0 + lane), already
// dequantised. init_bars sets up the epilogue's barriers (four per group). Tokens past M and features past the
// problem are skipped. begin / apply return false only when a bounded wait ran out.
// ---------------------------------------------------------------------------------------------------------------

// Plain fp32 store out[t][f] (row stride ld floats): the stand-alone sparse GEMM.
struct SpF32 : SpNoBars {
    struct Params {
        float *out;
        int ld, M, N;
    };
    __device__ __forceinline__ static float row_scale(const Params &, int) { return 1.0f; }
    __device__ __forceinline__ static bool begin(const Params &, SpCtx &) { return true; }
    __device__ __forceinline__ static bool apply(const Params &p, const float *acc, SpCtx &cx)
    {
        const int f = cx.f0 + cx.lane;
        if (f < p.N) {
#pragma unroll
            for (int j = 0; j < SP_COLS; j++)
                if (cx.t0 + j < p.M) p.out[(size_t)(cx.t0 + j) * p.ld + f] = acc[j];
        }
        return true;
    }
};

// QKV (k_qkv, eva_kernels.cu:41-114), as EpiQKV: q / k rows get the interleaved RoPE of patch tokens (dims 2j and
// 2j + 1 are neighbouring lanes), v rows are only scaled (cq / ck / cv ride on the block-scale promotion); E4M3 into
// q8 / k8 / v8 [img][head][TP][64], one byte per lane (32 consecutive bytes per warp store).
// The RoPE angles of the tile's 112 tokens for a warp's 16 dim pairs (14 KB, [token][16 pairs]) are copied into the
// group's scratch by cp.async when the tile starts, so their latency hides behind the main loop. The two warps of
// a group that hold the same dims of the two heads (quads q and q ^ 2) share one buffer, each copying half of the
// tokens; group barriers 0 / 1 (64 arrivals: the copies of both warps' lanes have landed) and 2 / 3 (2 arrivals:
// both warps have read the buffer) order each use of the buffer of dim half 0 / 1.
struct SpQKV {
    struct Params {
        uint8_t *q8, *k8, *v8;
        const float2 *cs;
        float cq, ck, cv;
        int M;
    };
    __device__ __forceinline__ static void init_bars(uint64_t *eb)
    {
        for (int g = 0; g < 2; g++)
            for (int h = 0; h < 2; h++) {
                mbar_init(&eb[4 * g + h], 64);
                mbar_init(&eb[4 * g + 2 + h], 2);
            }
    }
    __device__ __forceinline__ static float row_scale(const Params &p, int f0)
    {
        const int which = f0 >> 10;
        return which == 0 ? p.cq : which == 1 ? p.ck : p.cv;
    }
    __device__ __forceinline__ static uint8_t *angles(const SpCtx &cx) { return cx.gscratch + (cx.quad & 1) * (SP_COLS * 128); }
    __device__ __forceinline__ static bool begin(const Params &p, SpCtx &cx)
    {
        if ((cx.f0 >> 10) == 2) return true;  // v rows: no RoPE
        const int h = cx.quad & 1;
        // the previous use of the buffer has been read by both warps
        if (cx.use > 0 &&
            !__all_sync(0xffffffffu, mbar_wait(&cx.ebar[2 + h], (cx.use - 1) & 1, cx.err, XTB_ERR_WAIT_TMEM)))
            return false;
        uint8_t *buf = angles(cx);
        const int r0 = (cx.quad >> 1) * (SP_COLS / 2);  // quads 0 / 1 copy tokens 0..55, quads 2 / 3 tokens 56..111
        const float2 *src = p.cs + ((cx.f0 & 63) >> 1);  // this warp's first pair (0 or 16)
        for (int i = cx.lane; i < (SP_COLS / 2) * 8; i += 32) {
            const int r = r0 + (i >> 3), ch = i & 7;
            const int t = cx.t0 + r, tt = t % T;
            if (t < p.M && tt > 0) cp_async16(buf + r * 128 + ch * 16, src + (size_t)(tt - 1) * 32 + ch * 2);
        }
        cp_async_mbar_arrive(&cx.ebar[h]);
        return true;
    }
    __device__ __forceinline__ static bool apply(const Params &p, const float *acc, SpCtx &cx)
    {
        const int which = cx.f0 >> 10, head = (cx.f0 & 1023) >> 6, dbase = cx.f0 & 63;
        const int h = cx.quad & 1;
        const bool odd = cx.lane & 1;
        const uint8_t *ang = angles(cx) + (cx.lane >> 1) * 8;
        if (which < 2 && !__all_sync(0xffffffffu, mbar_wait(&cx.ebar[h], cx.use & 1, cx.err, XTB_ERR_WAIT_TMEM)))
            return false;
        uint8_t *dst = which == 0 ? p.q8 : which == 1 ? p.k8 : p.v8;
        // E4M3 bytes of 56 tokens x 32 dims are staged per warp in its slice of the (otherwise unused) exchange area,
        // then leave as 16-byte pieces
        uint8_t *ob = (uint8_t *)cx.xred + (cx.quad & 3) * (SP_COLS / 2) * 32;
        int tt = cx.t0 % T;
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            __syncwarp();
#pragma unroll
            for (int jj = 0; jj < SP_COLS / 2; jj++) {
                const int j = hf * (SP_COLS / 2) + jj;
                float v = acc[j];
                if (which < 2) {
                    // (f0, f1) -> (f0 cos - f1 sin, f1 cos + f0 sin); cls rows and rows past M: cos 1, sin 0
                    const float pv = __shfl_xor_sync(0xffffffffu, v, 1);
                    float2 c = make_float2(1.f, 0.f);
                    if (tt > 0 && cx.t0 + j < p.M) c = *(const float2 *)(ang + j * 128);
                    v = fmaf(pv, odd ? c.y : -c.y, v * c.x);
                }
                ob[jj * 32 + cx.lane] = (uint8_t)e4m3x2(v, 0.f);
                if (++tt == T) tt = 0;
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < (SP_COLS + 31) / 32; i++) {  // 56 tokens x 2 pieces of 16 bytes: 112 of 128 lanes
                const int pc = i * 32 + cx.lane;
                const int r = pc >> 1, ch = pc & 1;
                const int t = cx.t0 + hf * (SP_COLS / 2) + r;
                if (r < SP_COLS / 2 && t < p.M) {
                    const int b = t / T, tq = t - b * T;
                    *(uint4 *)(dst + (((size_t)(b * NH + head) * TP + tq) << 6) + dbase + 16 * ch) =
                        *(const uint4 *)(ob + r * 32 + 16 * ch);
                }
            }
        }
        if (which < 2) {
            __syncwarp();
            if (cx.lane == 0) mbar_arrive(&cx.ebar[2 + h]);
            cx.use++;
        }
        return true;
    }
};

// fp16 residual update x[t][f] += delta by TMA reduce-add of the warp's 112 tokens x 32 features (the tensor map
// has boxes of 32 halves x 112 rows, unswizzled): the out-projection (EpiResid, LN = false) and fc2 with the MLP
// LayerNorm folded in (EpiFC2, LN = true: delta = rstd * (acc - mean * c[f]) + d[f] with (mean, rstd) of the token
// from k_rowstat).
template <bool LN>
struct SpResid : SpNoBars {
    struct Params {
        const float2 *ms;
        const float *c, *d;
        int M;
    };
    __device__ __forceinline__ static float row_scale(const Params &, int) { return 1.0f; }
    __device__ __forceinline__ static bool begin(const Params &, SpCtx &) { return true; }
    __device__ __forceinline__ static bool apply(const Params &p, const float *acc, SpCtx &cx)
    {
        if (cx.lane == 0) bulk_wait_read0();  // the previous tile's reduction has read the staging buffer
        __syncwarp();
        float cf = 0.f, df = 0.f;
        if (LN) {
            cf = __ldg(p.c + cx.f0 + cx.lane);
            df = __ldg(p.d + cx.f0 + cx.lane);
        }
        __half *srow = (__half *)cx.stage + cx.lane;
#pragma unroll
        for (int j = 0; j < SP_COLS; j++) {
            float v = acc[j];
            if (LN) {
                const float2 ms = __ldg(p.ms + min(cx.t0 + j, p.M - 1));
                v = fmaf(ms.y, v, fmaf(-ms.x * ms.y, cf, df));
            }
            srow[j * 32] = __float2half_rn(v);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (cx.lane == 0 && cx.t0 < p.M) {
            tma_reduce_add_2d(cx.tmC, cx.stage, cx.f0, cx.t0);
            bulk_commit();
        }
        return true;
    }
};

// Sum of v[8] (8 tokens) over the 16 lanes of each half-warp, in a fixed order: on return v[0] of lane l holds the
// total of token (l >> 1) & 7 (lanes l and l ^ 1 hold the same).
__device__ __forceinline__ void halfwarp_sum8(float (&v)[8], int lane)
{
    const bool b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float send = b3 ? v[i] : v[i + 4];
        const float keep = b3 ? v[i + 4] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float send = b2 ? v[i] : v[i + 2];
        const float keep = b2 ? v[i + 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const float send = b1 ? v[0] : v[1];
        const float keep = b1 ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// fc1 + SwiGLU (k_fc1, eva_kernels.cu:211-279), as EpiFC1. The W12 rows interleave g and x in 16-unit chunks, so a
// warp's lanes 0-15 hold g and lanes 16-31 x of the same 16 units: one exchange gives lanes 0-15 tokens 0..55 and
// lanes 16-31 tokens 56..111 of (g, x). u = x g sigmoid(g), h8 = E4M3(u rs[unit]) stored by TMA (boxes of 16 units x
// 112 tokens); the row statistics partial stat[nb][t] (sum u, sum u^2 over the tile's 64 units) is summed across
// the 16 lanes, then across the group's four warps through shared memory (group barriers 0 / 1, one per exchange
// buffer, four arrivals).
struct SpFC1 {
    struct Params {
        float2 *stat;
        const float *rs;
        int M;
    };
    __device__ __forceinline__ static void init_bars(uint64_t *eb)
    {
        for (int g = 0; g < 2; g++)
            for (int b = 0; b < 2; b++) mbar_init(&eb[4 * g + b], 4);
    }
    __device__ __forceinline__ static float row_scale(const Params &, int) { return 1.0f; }
    __device__ __forceinline__ static bool begin(const Params &, SpCtx &) { return true; }
    __device__ __forceinline__ static bool apply(const Params &p, const float *acc, SpCtx &cx)
    {
        constexpr int H = SP_COLS / 2;  // tokens per lane after the exchange
        const int lane = cx.lane;
        const bool hi = lane >= 16;
        const int unit = (cx.f0 >> 1) + (lane & 15);
        const bool live = cx.f0 < N12;  // warp-uniform: false for the padding rows of the last weight tile
        const float r = (live && unit < HIDP) ? __ldg(p.rs + unit) : 0.0f;
        const uint32_t buf = cx.use & 1;
        float2 *xr = cx.xred + buf * 4 * SP_COLS;
        if (lane == 0) bulk_wait_read0();  // the previous tile's h8 store has read the staging buffer
        __syncwarp();
        uint8_t *srow = cx.stage + (hi ? H : 0) * 16 + (lane & 15);
#pragma unroll
        for (int c = 0; c < H / 8; c++) {
            float s[8], q[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int j = 8 * c + i;
                const float send = hi ? acc[j] : acc[H + j];
                const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
                const float gv = hi ? recv : acc[j];
                const float xv = hi ? acc[H + j] : recv;
                const float hg = 0.5f * gv;  // u = x (g/2) (1 + tanh(g/2))
                const float u = xv * fmaf(hg, tanh_fast(hg), hg);
                srow[j * 16] = (uint8_t)e4m3x2(u * r, 0.f);
                s[i] = u;
                q[i] = u * u;
            }
            halfwarp_sum8(s, lane);
            halfwarp_sum8(q, lane);
            if (!(lane & 1)) xr[cx.quad * SP_COLS + (hi ? H : 0) + 8 * c + ((lane >> 1) & 7)] = make_float2(s[0], q[0]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && live && cx.t0 < p.M) {
            tma_store_2d(cx.tmC, cx.stage, cx.f0 >> 1, cx.t0);
            bulk_commit();
        }
        if (lane == 0) mbar_arrive(&cx.ebar[buf]);
        const bool ok = __all_sync(0xffffffffu, mbar_wait(&cx.ebar[buf], (cx.use >> 1) & 1, cx.err, XTB_ERR_WAIT_TMEM));
        if (ok && lane < SP_COLS / 4) {
            const int tk = (SP_COLS / 4) * cx.quad + lane;
            float2 a = xr[tk];
#pragma unroll
            for (int w = 1; w < 4; w++) {
                const float2 b = xr[w * SP_COLS + tk];
                a.x += b.x;
                a.y += b.y;
            }
            const int t = cx.t0 + tk;
            if (t < p.M) p.stat[(size_t)cx.nb * p.M + t] = a;
        }
        cx.use++;
        return ok;
    }
};

}  // namespace xtb

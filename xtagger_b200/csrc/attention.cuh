// FP8 flash attention on tcgen05 for the EVA02-L tagger (1025 tokens) and the PixAI tagger (sequences of 576 or
// 5184 tokens, AttSeq below): one CTA per pair of 128-query tiles of one (sequence, head).
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
// Work split (320 threads, 2 CTAs per SM): one CTA per pair of 128-query tiles of one (head, image) covering rows
// 0 .. 1023; the two tiles ("groups") share every K / V tile. Warp 0 TMA (both Q tiles once; K / V in tiles of 128
// keys through a 3-deep ring), warp 1 TMEM allocation (256 columns: S_g at [64 g, 64 g + 64), O_g at
// [128 + 64 g, 192 + 64 g)) and the MMA issuer, warps 2..5 the softmax of group 0 and warps 6..9 that of group 1, one
// query row per thread (warp w reads TMEM lanes 32 (w % 4) ..). Per 64-key step u and group g: S_g,u = Q_g K_u^T
// (M 128, N 64 keys, K 64 dims); the softmax reads it in one pass with the running max (p, l and the tile max
// together) and re-passes a warp only when one of its slices rescales; it writes P_g,u (the row's 64 E4M3 values)
// with one tcgen05.st into the first 16 columns of S_g, where O_g += P_g,u V_u (M 128, N 64 dims, K 64 keys) reads it
// as a TMEM A operand, V being an MN-major operand straight from its [token][64 dims] rows. The MMA issues PV_g,u
// before S_g,u+1, which overwrites those columns; the tensor core keeps the order, so the commit that signals
// S_g,u+1 also means PV_g,u is done. While one group's softmax works, the tensor core computes the other group's
// scores, and 16 softmax warps per SM (4 per sub-partition) keep the exp2 unit fed through each warp's latencies.
//
// Query row 1024 (the last token) is the only real row of its 128-row tile; a CTA for it would run all 17 steps for
// one row. k_attention_last computes it instead, one warp per (head, image). Its reference slice (rows 1024 .. 1039)
// holds 15 zero query rows of the padding, whose scores are all 0: they never ask for a rescale after the first
// tile and never let the slice go dead, so the row follows the per-row rule (rescale when its own tile max exceeds
// m + RESCALE / sinv; no dead tiles), which the warp applies exactly.
#pragma once
#include "ops.h"
#include "ptx.cuh"

namespace xtb {

constexpr float ATT_RESCALE = 8.0f;
constexpr float ATT_PSKIP = 10.0f;
constexpr int ATT_SUB = 64;                       // keys per softmax step (the reference's key tile)
constexpr int ATT_NSUB = (T + ATT_SUB - 1) / ATT_SUB;  // EVA02-L: 17 steps; the last holds 1 key
constexpr int ATT_KS = 3;                         // K / V ring depth (128-key tiles)
constexpr int ATT_G = 2;                          // query tiles (groups) per CTA
constexpr int ATT_QTF = (T - 1) / 128;               // EVA02-L: full query tiles (8): rows 0 .. 1023
constexpr int ATT_THREADS = 64 + 32 * 4 * ATT_G;

// Sequence shape of one attention instance: L tokens per (sequence, head), RS rows between consecutive
// (sequence, head) blocks of q8 / k8 / v8, NQT query tiles of 128 rows. Tile i starts at row min(128 i, L - 128):
// when L is not a multiple of 128 the last tile overlaps its neighbour and writes only its own rows; the rows it
// shares are computed identically in both (the lazy-rescale and dead-tile decisions are per 16-row slice, and a
// tile start is a multiple of 64). EVA02-L: <1025, 1152, 8> (rows 0 .. 1023; row 1024 by k_attention_last);
// PixAI windows <576, 576, 5>, global blocks <5184, 5184, 41>.
template <int L_, int RS_, int NQT_>
struct AttSeq {
    static constexpr int L = L_, RS = RS_, NQT = NQT_;
    static constexpr int NSUB = (L + ATT_SUB - 1) / ATT_SUB;  // 64-key softmax steps
    static constexpr int NK = (NSUB + 1) / 2;                 // K / V tiles of 128 keys
    static constexpr int PAIRS = (NQT + ATT_G - 1) / ATT_G;   // CTAs per (sequence, head)
    static constexpr bool RAGGED = (L % ATT_SUB) != 0;        // the last step holds fewer than 64 keys
    __device__ __forceinline__ static int qstart(int i) { return min(i * 128, L - 128); }
    static_assert(L >= 128 && NQT >= 1 && (NQT - 1) * 128 < L, "query tiles");
};
using AttEva = AttSeq<T, TP, ATT_QTF>;
constexpr int ATT_Q_BYTES = 128 * 64;
constexpr int ATT_K_BYTES = 128 * 64;
constexpr int ATT_V_BYTES = 128 * 64;
constexpr size_t ATT_SMEM = 1024 + ATT_G * ATT_Q_BYTES + ATT_KS * (ATT_K_BYTES + ATT_V_BYTES) + 512;

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


// 2^x on the FMA and ALU pipes, for the share of the softmax's exponentials taken off the MUFU unit (the kernel's
// limiter): Cody-Waite style reduction x = n + f with n = round(x) by the 1.5 x 2^23 shifter (no conversion
// instruction), f in [-0.5, 0.5]; 2^f by a degree-5 polynomial fitted for this library to 2^f on [-0.5, 0.5]
// (relative error 2.0e-7 in fp32 Horner form, the order of ex2.approx's own); 2^n added into the exponent field.
// Arguments below -126 are clamped there (2^-126 rounds to E4M3 zero and adds nothing measurable to a row sum);
// arguments stay below RESCALE = 8 by the softmax's construction.
constexpr int ATT_POLY_GROUPS = 2;  // of the 8 four-column groups of a 32-column score chunk
__device__ __forceinline__ float2 ex2_poly2(float2 x)
{
    constexpr float SH = 12582912.0f;  // 1.5 x 2^23: x + SH holds round(x) in its low mantissa bits
    constexpr float C0 = 1.0000001192092896f, C1 = 0.6931469440460205f, C2 = 0.24022121727466583f,
                    C3 = 0.05550742521882057f, C4 = 0.00967546459287405f, C5 = 0.0013266978785395622f;
    x = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
    const float2 t = add2(x, make_float2(SH, SH));
    const float2 f = add2(x, add2(make_float2(SH, SH), make_float2(-t.x, -t.y)));  // x - round(x)
    float2 p = fma2(f, make_float2(C5, C5), make_float2(C4, C4));
    p = fma2(f, p, make_float2(C3, C3));
    p = fma2(f, p, make_float2(C2, C2));
    p = fma2(f, p, make_float2(C1, C1));
    p = fma2(f, p, make_float2(C0, C0));
    const int nx = __float_as_int(t.x) - __float_as_int(SH), ny = __float_as_int(t.y) - __float_as_int(SH);
    return make_float2(__int_as_float(__float_as_int(p.x) + (nx << 23)), __int_as_float(__float_as_int(p.y) + (ny << 23)));
}

// Max of a row's scores in a full S buffer (TMEM, 64 columns at sS).
__device__ __forceinline__ float tile_max(uint32_t sS)
{
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < 2; c++) {
        float v[32];
        tmem_ld32(sS + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 8)
#pragma unroll
            for (int e = 0; e < 4; e++) t4[e] = fmax3(t4[e], v[i + 2 * e], v[i + 2 * e + 1]);
    }
    return fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
}

// Columns [16 cc, 16 cc + 16) of a full score row (v, 16 values) into the pass's accumulators: the same operations
// in the same order as the 32-column loop of exp_pass below (tile max per 4-column half, exponent, l, E4M3 pairs).
__device__ __forceinline__ void exp_cols16(const float *v, int cc, float2 sv2, float2 nm2, float *t4, float2 *l2,
                                           uint32_t *w)
{
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
        const int g = (cc & 1) * 16 + i;  // column within the 32-column chunk
        t4[(i >> 2) & 1] = fmax3(t4[(i >> 2) & 1], v[i], v[i + 1]);
        t4[2 + ((i >> 2) & 1)] = fmax3(t4[2 + ((i >> 2) & 1)], v[i + 2], v[i + 3]);
        float pp[4];
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
            const float2 a = fma2(make_float2(v[i + e], v[i + e + 1]), sv2, nm2);
            if ((g >> 2) < ATT_POLY_GROUPS) {
                const float2 q = ex2_poly2(a);
                pp[e] = q.x;
                pp[e + 1] = q.y;
            } else {
                pp[e] = ex2(a.x);
                pp[e + 1] = ex2(a.y);
            }
            l2[e >> 1] = add2(l2[e >> 1], make_float2(pp[e], pp[e + 1]));
        }
        w[cc * 4 + (i >> 2)] = e4m3x2(pp[0], pp[1]) | (e4m3x2(pp[2], pp[3]) << 16);
    }
}

// One pass over a row of an S buffer with max m: tile max, p = exp2(s sinv - m sinv), sum of p, E4M3(p) -> the
// row of P. FULL: all 64 keys are valid (every step but the last); otherwise keys >= nvalid are masked (p = 0).
// The full pass reads the row in four 16-column loads, each issued before the math on the previous one, so that
// only the first load's latency is exposed; the results are those of the 32-column loop (same order of operations).
template <bool FULL>
__device__ __forceinline__ void exp_pass(uint32_t sS, uint32_t *w, int nvalid, float2 sv2, float m, float *tm_out,
                                         float *l_out)
{
    const float2 nm2 = make_float2(-m * sv2.x, -m * sv2.x);
    float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    float2 l2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    if constexpr (FULL) {
        float va[16], vb[16];
        tmem_ld16(sS, va);
        tmem_wait_ld_regs16(va);
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
            float *cur = (cc & 1) ? vb : va;
            float *nxt = (cc & 1) ? va : vb;
            if (cc < 3) tmem_ld16(sS + (cc + 1) * 16, nxt);
            exp_cols16(cur, cc, sv2, nm2, t4, l2, w);
            if (cc < 3) tmem_wait_ld_regs16(nxt);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (c * 32 < nvalid) {  // warp-uniform
                float v[32];
                tmem_ld32(sS + c * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++)
                    if (c * 32 + i >= nvalid) v[i] = -INFINITY;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    t4[(i >> 2) & 1] = fmax3(t4[(i >> 2) & 1], v[i], v[i + 1]);
                    t4[2 + ((i >> 2) & 1)] = fmax3(t4[2 + ((i >> 2) & 1)], v[i + 2], v[i + 3]);
                    float pp[4];
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {
                        const float2 a = fma2(make_float2(v[i + e], v[i + e + 1]), sv2, nm2);
                        if ((i >> 2) < ATT_POLY_GROUPS) {  // this share of the exponentials on the FMA pipe
                            const float2 q = ex2_poly2(a);
                            pp[e] = q.x;
                            pp[e + 1] = q.y;
                        } else {
                            pp[e] = ex2(a.x);
                            pp[e + 1] = ex2(a.y);
                        }
                        l2[e >> 1] = add2(l2[e >> 1], make_float2(pp[e], pp[e + 1]));
                    }
                    w[c * 8 + (i >> 2)] = e4m3x2(pp[0], pp[1]) | (e4m3x2(pp[2], pp[3]) << 16);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) w[c * 8 + i] = 0;
            }
        }
    }
    *tm_out = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
    *l_out = (l2[0].x + l2[0].y) + (l2[1].x + l2[1].y);
}

// fp32 -> fp16 (round to nearest) -> E4M3, as the reference's output staging (kern_common.cuh:527-541)
__device__ __forceinline__ uint32_t e4m3x2_via_f16(float a, float b)
{
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    return e4m3x2(f.x, f.y);
}

template <class SQ>
__global__ void __launch_bounds__(ATT_THREADS, 2)
    k_attention(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, uint8_t *__restrict__ out, float sinv, float vo, uint32_t *err)
{
    constexpr int NSUB = SQ::NSUB, NK = SQ::NK, RS = SQ::RS, L = SQ::L;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    uint8_t *sQ = smem;                                  // [ATT_G]
    uint8_t *sK = sQ + ATT_G * ATT_Q_BYTES;              // [ATT_KS]
    uint8_t *sV = sK + ATT_KS * ATT_K_BYTES;             // [ATT_KS]
    uint64_t *bar = (uint64_t *)(sV + ATT_KS * ATT_V_BYTES);
    uint64_t *q_full = bar;
    uint64_t *kv_full = q_full + 1;                      // [ATT_KS]
    uint64_t *kv_empty = kv_full + ATT_KS;               // [ATT_KS]
    uint64_t *s_full = kv_empty + ATT_KS;                // [ATT_G] S_g,u in TMEM (and every earlier MMA done)
    uint64_t *p_full = s_full + ATT_G;                   // [ATT_G] softmax g has read S_g,u and written P_g,u
    uint64_t *pv_done = p_full + ATT_G;                  // [ATT_G] PV_g,u done
    uint32_t *tslot = (uint32_t *)(pv_done + ATT_G);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt0 = blockIdx.x * ATT_G, h = blockIdx.y, b = blockIdx.z;
    const int ng = min(ATT_G, SQ::NQT - qt0);            // query tiles this CTA holds (CTA-uniform)
    const int bh = b * NH + h;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ATT_KS; s++) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int g = 0; g < ATT_G; g++) {
            mbar_init(&s_full[g], 1);
            mbar_init(&p_full[g], 4);
            mbar_init(&pv_done[g], 1);
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
    griddep_wait();  // the previous kernel of the stream has completed: activations may be touched

    if (warp == 0) {
        if (elect_one()) {
            mbar_arrive_expect_tx(q_full, ng * ATT_Q_BYTES);
            for (int g = 0; g < ng; g++) tma_load_2d(sQ + g * ATT_Q_BYTES, &tq, q_full, 0, bh * RS + SQ::qstart(qt0 + g));
            uint32_t ph = 0;
            int st = 0;
            for (int j = 0; j < NK; j++) {
                if (!mbar_wait(&kv_empty[st], ph ^ 1, err, XTB_ERR_WAIT_ATTN)) break;
                mbar_arrive_expect_tx(&kv_full[st], ATT_K_BYTES + ATT_V_BYTES);
                tma_load_2d(sK + st * ATT_K_BYTES, &tk, &kv_full[st], 0, bh * RS + j * 128);
                tma_load_2d(sV + st * ATT_V_BYTES, &tv, &kv_full[st], 0, bh * RS + j * 128);
                if (++st == ATT_KS) {
                    st = 0;
                    ph ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            // S: N = 64 keys. PV: A = P from TMEM (16 columns of the group's S buffer), B = V, MN-major (bit 16)
            constexpr uint32_t ID_S = idesc_m128(64), ID_PV = idesc_m128(64) | (1u << 16);
            bool ok = mbar_wait(q_full, 0, err, XTB_ERR_WAIT_ATTN);
            for (int u = 0; u <= NSUB && ok; u++) {
                const int j = u >> 1, st = j % ATT_KS;
                if (u < NSUB && !(u & 1) && !(ok = mbar_wait(&kv_full[st], (j / ATT_KS) & 1, err, XTB_ERR_WAIT_ATTN)))
                    break;
                const int w = u - 1, wst = (w >> 1) % ATT_KS;
                for (int g = 0; g < ng && ok; g++) {
                    const uint32_t tS = tbase + g * 64;
                    if (u > 0) {  // O_g += P_g,w V_w; P lives in S_g's first 16 columns until S_g,u overwrites them
                        if (!(ok = mbar_wait(&p_full[g], w & 1, err, XTB_ERR_WAIT_ATTN))) break;
                        tc_fence_after();
                        const uint32_t v0 = smem_u32(sV + wst * ATT_V_BYTES) + (w & 1) * 4096;
#pragma unroll
                        for (int kk = 0; kk < 2; kk++)
                            umma_tmem_a(tbase + 128 + g * 64, tS + kk * 8, sdesc_mn(v0 + kk * 2048, 512, SWZ_64B), ID_PV,
                                        (w > 0 || kk > 0));
                        umma_commit(&pv_done[g]);
                    }
                    if (u < NSUB) {  // S_g,u = Q_g K_u^T, issued after PV_g,w (the tensor core keeps the order)
                        const uint32_t q0 = smem_u32(sQ + g * ATT_Q_BYTES);
                        const uint32_t k0 = smem_u32(sK + st * ATT_K_BYTES) + (u & 1) * 4096;
#pragma unroll
                        for (int kk = 0; kk < 2; kk++)
                            umma<false>(tS, sdesc(q0 + kk * 32, 512, SWZ_64B), sdesc(k0 + kk * 32, 512, SWZ_64B), ID_S, kk);
                        umma_commit(&s_full[g]);
                    }
                }
                if (!ok) break;
                if (u > 0 && ((w & 1) || w == NSUB - 1)) umma_commit(&kv_empty[wst]);  // the K / V tile is used up
            }
        }
    } else if ((warp - 2) / 4 < ng) {
        const int g = (warp - 2) / 4;                    // query tile (group) of this warp
        const int quad = warp & 3;
        const int r = quad * 32 + lane;                  // query row within the tile = TMEM lane
        const uint32_t lrow = (uint32_t)(quad * 32) << 16;
        const uint32_t sS = tbase + g * 64 + lrow, sO = tbase + 128 + g * 64 + lrow;
        const float thr = ATT_RESCALE / sinv, dthr = ATT_PSKIP / sinv;
        const uint32_t half = lane < 16 ? 0x0000FFFFu : 0xFFFF0000u;  // this row's 16-row slice
        const float2 sv2 = make_float2(sinv, sinv);
        float m = -1e30f, l = 0.f;
        bool ok = true;
        for (int u = 0; u < NSUB && ok; u++) {
            const int nvalid = min(ATT_SUB, L - u * ATT_SUB);
            // S_g,u has landed, and with it every earlier MMA of the CTA (PV_g,u-1 included)
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[g], u & 1, err, XTB_ERR_WAIT_ATTN)))) break;
            tc_fence_after();
            uint32_t pw[16];
            // one pass with the running max: tile max, p = exp2(s sinv - m sinv), l_tile, P
            float tm = -INFINITY, lt = 0.f;
            const bool full = !SQ::RAGGED || u < NSUB - 1;  // EVA02-L: the last step holds one key
            if (u == 0) tm = tile_max(sS);
            else if (full) exp_pass<true>(sS, pw, nvalid, sv2, m, &tm, &lt);
            else exp_pass<false>(sS, pw, nvalid, sv2, m, &tm, &lt);
            const float mn = fmaxf(m, tm);
            const bool resc = (__ballot_sync(0xffffffffu, mn > m + thr) & half) != 0;
            if (__any_sync(0xffffffffu, resc)) {
                float sc = 1.0f;
                if (resc) {  // every row of a rescaling slice takes its max
                    sc = ex2((m - mn) * sinv);
                    l *= sc;
                    m = mn;
                }
                if (u > 0) {  // O holds P V of the earlier steps (complete): rescale it in TMEM, factor 1 for the
                              // slice that keeps its max (TMEM access is warp-collective)
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
                if (full) exp_pass<true>(sS, pw, nvalid, sv2, m, &tm2, &lt);
                else exp_pass<false>(sS, pw, nvalid, sv2, m, &tm2, &lt);
            }
            if ((__ballot_sync(0xffffffffu, tm < m - dthr) & half) == half) {  // dead slice: P zero, l unchanged
#pragma unroll
                for (int i = 0; i < 16; i++) pw[i] = 0;
                lt = 0.f;
            }
            l += lt;
            // P_g,u (the row's 64 E4M3 values) into the first 16 columns of S_g: the A operand of PV_g,u
            tmem_st16u(sS, pw);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[g]);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[g], (NSUB - 1) & 1, err, XTB_ERR_WAIT_ATTN));
        if (ok) {
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
            const int t = SQ::qstart(qt0 + g) + r;
            if (t >= (qt0 + g) * 128) {  // rows shared with the previous tile are written by that tile
                uint4 *o = (uint4 *)(out + ((size_t)b * L + t) * D + h * HD);
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

// Query row 1024 of every (head, image): one CTA of 256 threads each, in parallel over keys instead of a sequential
// walk over the 17 key tiles. The walk only matters through the running max, and for a single row it is a scan over
// the 17 tile maxima: m_u, the max in force while tile u is accumulated (m_u = tm_u when tm_u > m_{u-1} + RESCALE /
// sinv, else m_{u-1}; m_0 = tm_0), and the factor w_u = prod of exp2((m_{v-1} - m_v) sinv) over the later rescales
// v > u that the reference applies to l and O after tile u. Then p_k = exp2(s_k sinv - m_u sinv) (one fma, ex2.approx),
// l = sum_u w_u sum_{k in u} p_k and O = sum_u w_u sum_{k in u} E4M3(p_k) V_k: the reference's values, summed in
// another order.
constexpr int ATT_LAST_THREADS = 256;

__device__ __forceinline__ void e4m3x4_to_f32(uint32_t w, float *f)
{
    const float2 a = __half22float2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xffff), __NV_E4M3));
    const float2 b = __half22float2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

__global__ void __launch_bounds__(ATT_LAST_THREADS)
    k_attention_last(const uint8_t *__restrict__ q8, const uint8_t *__restrict__ k8, const uint8_t *__restrict__ v8,
                     uint8_t *__restrict__ out, float sinv, float vo)
{
    __shared__ float sq[64];
    __shared__ float ss[ATT_NSUB * 64];          // scores, then E4M3-rounded p (keys >= 1025: 0)
    __shared__ float stm[ATT_NSUB], sm_u[ATT_NSUB], sw[ATT_NSUB], sl[ATT_NSUB];
    __shared__ float2 sop[8][32];                // O partial sums: [key quarter x tile parity][dim pair]
    const int bh = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t = T - 1;
    const size_t base = (size_t)bh * TP;
    if (tid < 16) {
        float f[4];
        e4m3x4_to_f32(__ldg((const uint32_t *)(q8 + (base + t) * 64) + tid), f);
#pragma unroll
        for (int x = 0; x < 4; x++) sq[4 * tid + x] = f[x];
    }
    __syncthreads();
    // scores: keys tid, tid + 256, ...; four partial sums per dot product. Every key row of the thread is loaded
    // before any is used, so the loads' latencies overlap instead of adding up.
    constexpr int KPT_LAST = (ATT_NSUB * 64 + ATT_LAST_THREADS - 1) / ATT_LAST_THREADS;
    uint4 krow[KPT_LAST][4];
#pragma unroll
    for (int j = 0; j < KPT_LAST; j++) {
        const int key = tid + j * ATT_LAST_THREADS;
#pragma unroll
        for (int c = 0; c < 4; c++)
            krow[j][c] = key < T ? __ldg((const uint4 *)(k8 + (base + key) * 64) + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < KPT_LAST; j++) {
        const int key = tid + j * ATT_LAST_THREADS;
        if (key >= ATT_NSUB * 64) break;
        float sc = -INFINITY;
        if (key < T) {
            float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const uint4 w = krow[j][c];
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float kf[4];
                    e4m3x4_to_f32(ws[e], kf);
#pragma unroll
                    for (int x = 0; x < 4; x++) a4[x] = fmaf(sq[16 * c + 4 * e + x], kf[x], a4[x]);
                }
            }
            sc = (a4[0] + a4[1]) + (a4[2] + a4[3]);
        }
        ss[key] = sc;
    }
    __syncthreads();
    // tile maxima: warp w takes tiles w, w + 8, ...
    for (int u = warp; u < ATT_NSUB; u += ATT_LAST_THREADS / 32) {
        float tm = fmaxf(ss[u * 64 + lane], ss[u * 64 + 32 + lane]);
#pragma unroll
        for (int sh = 16; sh; sh >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, sh));
        if (lane == 0) stm[u] = tm;
    }
    __syncthreads();
    if (tid == 0) {  // the running max of the reference's walk, and the rescale factors applied after each tile
        const float thr = ATT_RESCALE / sinv;
        float m = -1e30f;
        for (int u = 0; u < ATT_NSUB; u++) {
            const float tm = stm[u];
            float sc = 1.0f;
            if (tm > m + thr) {
                sc = ex2((m - tm) * sinv);
                m = tm;
            }
            sm_u[u] = m;
            sw[u] = sc;  // factor applied to l and O when tile u starts
        }
        float w = 1.0f;  // suffix products: w_u = product of the factors of the tiles after u
        for (int u = ATT_NSUB - 1; u >= 0; u--) {
            const float sc = sw[u];
            sw[u] = w;
            w *= sc;
        }
    }
    __syncthreads();
    // p, per-tile sums of p (warp w: tiles w, w + 8, ...), E4M3-rounded p back into ss
    for (int u = warp; u < ATT_NSUB; u += ATT_LAST_THREADS / 32) {
        const float nm = -sm_u[u] * sinv;
        float lp = 0.f;
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int key = u * 64 + hh * 32 + lane;
            const float p = ex2(fmaf(ss[key], sinv, nm));  // masked keys: exp2(-inf) = 0
            lp += p;
            ss[key] = __low2float(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)e4m3x2(p, 0.f), __NV_E4M3));
        }
#pragma unroll
        for (int sh = 16; sh; sh >>= 1) lp += __shfl_xor_sync(0xffffffffu, lp, sh);
        if (lane == 0) sl[u] = lp;
    }
    __syncthreads();
    // O: thread = (dim pair, key quarter); tile weights applied per tile
    {
        const int dp = tid & 31, qk = tid >> 5;   // dims 2 dp, 2 dp + 1; keys of quarter qk % 4 in tiles (qk / 4) ...
        float o0 = 0.f, o1 = 0.f;
        for (int u = qk >> 2; u < ATT_NSUB; u += 2) {
            const int k0 = u * 64 + (qk & 3) * 16;
            // the run's 16 value pairs first (keys past the sequence read as zero and are skipped below), then the
            // products in key order
            uint32_t vv[16];
#pragma unroll
            for (int i = 0; i < 16; i++)
                vv[i] = k0 + i < T ? __ldg((const unsigned short *)(v8 + (base + k0 + i) * 64) + dp) : 0u;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                if (k0 + i >= T) break;
                const float pq = ss[k0 + i];
                const float2 vf = __half22float2(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)vv[i], __NV_E4M3));
                a0 = fmaf(pq, vf.x, a0);
                a1 = fmaf(pq, vf.y, a1);
            }
            o0 = fmaf(sw[u], a0, o0);
            o1 = fmaf(sw[u], a1, o1);
        }
        // 8 partial sums per dim pair (qk = 0..7) -> shared memory, then thread qk = 0 adds them
        sop[qk][dp] = make_float2(o0, o1);
        __syncthreads();
        if (qk == 0) {
            float2 acc = sop[0][dp];
#pragma unroll
            for (int i = 1; i < 8; i++) acc = make_float2(acc.x + sop[i][dp].x, acc.y + sop[i][dp].y);
            float l = 0.f;
            for (int u = 0; u < ATT_NSUB; u++) l = fmaf(sw[u], sl[u], l);
            const float f = vo / l;
            const int img = bh / NH, h = bh % NH;
            *(unsigned short *)(out + ((size_t)img * T + t) * D + h * HD + 2 * dp) =
                (unsigned short)e4m3x2_via_f16(acc.x * f, acc.y * f);
        }
    }
}

}  // namespace xtb

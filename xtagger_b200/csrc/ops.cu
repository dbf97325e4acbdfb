// Kernel launchers: pick the template instance, build the launch shape, enqueue. No allocation, no sync.
#include <mutex>
#include <utility>
#include <set>

#include "attention.cuh"
#include "epilogues.cuh"
#include "gemm.cuh"
#include "gemm2_mx.cuh"
#include "gemm_mx.cuh"
#include "gemm_sp.cuh"
#include "host.h"
#include "ops.h"
#include "pixai.cuh"
#include "rowops.cuh"

namespace xtb {

int current_device()
{
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int make_operand(Operand *op, const void *ptr, int rows, int row_bytes, int box_rows)
{
    op->ptr = ptr;
    op->rows = rows;
    op->row_bytes = row_bytes;
    op->box_rows = box_rows;
    return make_tmap_2d(&op->map, ptr, (uint64_t)row_bytes, (uint64_t)rows, (uint64_t)row_bytes, 128, (uint32_t)box_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
}

// Opt a kernel into its dynamic shared memory once per (kernel, device).
static int set_smem(const void *kern, size_t bytes)
{
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    const int dev = current_device();
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({kern, dev})) return 0;
    XTB_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    done.insert({kern, dev});
    return 0;
}

// Launches of the forward's kernels with programmatic stream serialisation (programmatic dependent launch): the
// kernel may be scheduled while the previous kernel on the stream finishes, so that its launch and on-chip set-up
// overlap that kernel's tail; every kernel launched this way executes griddep_wait() before it touches activations.
// Under stream capture the dependency becomes a programmatic edge of the graph. XTB_PDL=0 at build time launches
// them plainly.
// XTB_BALANCED_GRID=1 at build time: the single-CTA GEMM spreads its tiles evenly (fewer CTAs, the same number of
// tiles on the busiest one) instead of one CTA per SM.
#ifndef XTB_BALANCED_GRID
#define XTB_BALANCED_GRID 0
#endif
#ifndef XTB_PDL
#define XTB_PDL 1
#endif
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = XTB_PDL ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// One launch of the tcgen05 GEMM: A = a (M rows), B = b (N rows), K slices of 128 bytes.
template <class Epi, int BN, bool F16, bool PROMOTE, bool WS_ON_M, int EW = 8>
static int run_gemm(const Operand &a, const Operand &b, int M, int N, const float *ws, int ws_ld, int ws_rows, float ascale,
                    const typename Epi::Params &ep, cudaStream_t st, const CUtensorMap *tmc = nullptr,
                    uint32_t *err = nullptr, float wsu = 1.0f, bool b_weight = false)
{
    using Cfg = GemmCfg<BN, EW>;
    auto kern = k_gemm<Epi, BN, F16, PROMOTE, WS_ON_M, EW>;
    if (set_smem((const void *)kern, Cfg::SMEM)) return -1;
    if (a.row_bytes != b.row_bytes || M <= 0 || N <= 0 || a.box_rows != A_BOX_ROWS || b.box_rows != BN) {
        fprintf(stderr, "eva: gemm operands (K bytes %d vs %d, boxes %d / %d rows, M %d, N %d)\n", a.row_bytes,
                b.row_bytes, a.box_rows, b.box_rows, M, N);
        return -1;
    }
    const int dev = current_device();
    GemmArgs g{};
    g.M = M;
    g.N = N;
    g.kiters = (a.row_bytes + 127) / 128;
    g.m_tiles = (M + 127) / 128;
    g.n_tiles = (N + BN - 1) / BN;
    g.ws = ws;
    g.ws_ld = ws_ld;
    g.ws_rows = ws_rows;
    g.ascale = ascale;
    g.wsu = wsu;
    g.err = err ? err : error_word(dev);
    g.b_weight = b_weight ? 1 : 0;
    const int total = g.m_tiles * g.n_tiles;
    int grid = num_sms(dev);
    if (grid > total) grid = total;
#if XTB_BALANCED_GRID
    const int per = (total + grid - 1) / grid;  // tiles of the busiest CTA: spread them evenly over fewer CTAs
    grid = (total + per - 1) / per;
#endif
    XTB_CK(launch_pdl(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM, st, a.map, b.map, tmc ? *tmc : a.map, g, ep));
    return 0;
}

// One launch of the CTA-pair GEMM (block-scaled E4M3): 256 x 128 tiles, one cluster of two CTAs per tile at a
// time, as many clusters as can be resident (a persistent grid).
template <class Epi, int BN = 256, bool GROUPS = false, bool PROMOTE = true>
static int run_gemm2(const Operand &a, const Operand &b, int M, int N, const float *ws, int ws_ld, int ws_rows, float ascale,
                     const typename Epi::Params &ep, cudaStream_t st, const CUtensorMap *tmc = nullptr,
                     uint32_t *err = nullptr, float wsu = 1.0f)
{
    using Cfg = Gemm2CfgT<BN, GROUPS, StagingOf<Epi>::v>;
    auto kern = k_gemm2<Epi, PROMOTE, BN, GROUPS>;
    if (set_smem((const void *)kern, Cfg::SMEM)) return -1;
    if (a.row_bytes != b.row_bytes || M <= 0 || N <= 0 || a.box_rows != A_BOX_ROWS || b.box_rows != Cfg::BN / 2) {
        fprintf(stderr, "eva: pair gemm operands (K bytes %d vs %d, boxes %d / %d rows, M %d, N %d)\n", a.row_bytes,
                b.row_bytes, a.box_rows, b.box_rows, M, N);
        return -1;
    }
    const int dev = current_device();
    GemmArgs g{};
    g.M = M;
    g.N = N;
    g.kiters = (a.row_bytes + 127) / 128;
    g.m_tiles = (M + 255) / 256;
    g.n_tiles = (N + Cfg::BN - 1) / Cfg::BN;
    g.ws = ws;
    g.ws_ld = ws_ld;
    g.ws_rows = ws_rows;
    g.ascale = ascale;
    g.wsu = wsu;
    g.err = err ? err : error_word(dev);
    const int total = g.m_tiles * g.n_tiles;
    int pairs = max_pairs((const void *)kern, Cfg::THREADS, Cfg::SMEM);
    if (pairs <= 0) return -1;
    if (pairs > total) pairs = total;
    XTB_CK(launch_pdl(kern, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM, st, a.map, b.map, tmc ? *tmc : a.map, g,
                      ep));
    return 0;
}

static int kb(int k) { return (k + 127) / 128; }

size_t sf_image_bytes(int n, int k) { return (size_t)kb(k) * ((kb(n) + 1) & ~1) * 512; }

int sf_image(const float *ws, int n, int k, uint8_t *img)
{
    const int nbn = kb(n), nbk = kb(k), nbp = (nbn + 1) & ~1;
    for (int i = 0; i < nbn * nbk; i++) {
        uint32_t u;
        memcpy(&u, ws + i, 4);
        const uint32_t e = (u >> 23) & 0xFF;
        if ((u & 0x807FFFFFu) || e == 0 || e == 0xFF) return -1;  // positive normal powers of two only
    }
    for (int q = 0; q < nbk; q++)
        for (int b = 0; b < nbp; b++) {
            uint8_t e = 127;  // padding N block: 2^0
            if (b < nbn) {
                uint32_t u;
                memcpy(&u, ws + (size_t)b * nbk + q, 4);
                e = (uint8_t)((u >> 23) & 0xFF);
            }
            memset(img + ((size_t)q * nbp + b) * 512, e, 512);
        }
    return 0;
}

int sf_map(CUtensorMap *m, const uint8_t *sf, int n, int k)
{
    const uint64_t rows = (uint64_t)kb(k) * ((kb(n) + 1) & ~1) * 2;
    return make_tmap_2d(m, sf, 256, rows, 256, 256, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// One launch of the CTA-pair block-scaled GEMM (power-of-two block scales, w.sf, w.sfmap): 256 x 128 tiles, or
// 256 x 256 (NB2 = 2: two weight blocks per tile).
template <class Epi, int NB2>
static int run_gemm2_mx(const Operand &a, const Weight8 &w, int M, float ascale, const typename Epi::Params &ep,
                        cudaStream_t st, const CUtensorMap *tmc = nullptr, uint32_t *err = nullptr)
{
    using Cfg = Gemm2MxCfg<StagingOf<Epi>::v, NB2>;
    auto kern = k_gemm2_mx<Epi, NB2>;
    if (set_smem((const void *)kern, Cfg::SMEM)) return -1;
    if (!w.sf || a.row_bytes != w.op.row_bytes || M <= 0 || a.box_rows != A_BOX_ROWS || w.op.box_rows != 64) {
        fprintf(stderr, "eva: pair mx gemm operands (scale image %p, K bytes %d vs %d, boxes %d / %d rows, M %d)\n",
                (const void *)w.sf, a.row_bytes, w.op.row_bytes, a.box_rows, w.op.box_rows, M);
        return -1;
    }
    const int dev = current_device();
    GemmArgs g{};
    g.M = M;
    g.N = w.n;
    g.kiters = (a.row_bytes + 127) / 128;
    g.m_tiles = (M + 255) / 256;
    g.n_tiles = (w.n + Cfg::BN - 1) / Cfg::BN;
    g.ascale = ascale;
    g.wsu = 1.0f;
    g.err = err ? err : error_word(dev);
    GemmMxArgs mx{w.sf, w.sf_nbp};
    const int total = g.m_tiles * g.n_tiles;
    int pairs = max_pairs((const void *)kern, Cfg::THREADS, Cfg::SMEM);
    if (pairs <= 0) return -1;
    if (pairs > total) pairs = total;
    XTB_CK(launch_pdl(kern, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM, st, a.map, w.op.map, w.sfmap,
                      tmc ? *tmc : a.map, g, mx, ep));
    return 0;
}

// One launch of the block-scaled GEMM on the tensor core's own scaling (power-of-two block scales, w.sf).
template <class Epi>
static int run_gemm_mx(const Operand &a, const Weight8 &w, int M, float ascale, const typename Epi::Params &ep,
                       cudaStream_t st, const CUtensorMap *tmc = nullptr, uint32_t *err = nullptr)
{
    using Cfg = GemmMxCfg<StagingOf<Epi>::v>;
    auto kern = k_gemm_mx<Epi>;
    if (set_smem((const void *)kern, Cfg::SMEM)) return -1;
    if (!w.sf || a.row_bytes != w.op.row_bytes || M <= 0 || a.box_rows != A_BOX_ROWS || w.op.box_rows != Cfg::BN) {
        fprintf(stderr, "eva: mx gemm operands (scale image %p, K bytes %d vs %d, boxes %d / %d rows, M %d)\n",
                (const void *)w.sf, a.row_bytes, w.op.row_bytes, a.box_rows, w.op.box_rows, M);
        return -1;
    }
    const int dev = current_device();
    GemmArgs g{};
    g.M = M;
    g.N = w.n;
    g.kiters = (a.row_bytes + 127) / 128;
    g.m_tiles = (M + 127) / 128;
    g.n_tiles = (w.n + Cfg::BN - 1) / Cfg::BN;
    g.ascale = ascale;
    g.wsu = 1.0f;
    g.err = err ? err : error_word(dev);
    GemmMxArgs mx{w.sf, w.sf_nbp};
    const int total = g.m_tiles * g.n_tiles;
    int grid = num_sms(dev);
    if (grid > total) grid = total;
    XTB_CK(launch_pdl(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM, st, a.map, w.op.map, tmc ? *tmc : a.map, g,
                      mx, ep));
    return 0;
}

// Kernel of each projection (true: CTA pair), from timing both inside the batch-64 forward: the pair wins where the
// operand feed bounds the main loop (fc2: K = 2736, A streamed from DRAM, 5.6 against 6.4 ms per forward) and for
// QKV (7.45 against 7.7 ms); the single CTA for fc1 (10.3 against 10.8 ms) and O (2.14 against 2.19 ms).
#ifndef XTB_PAIR_MASK
#define XTB_PAIR_MASK 0x9  // bit u set: WeightUse u on the CTA-pair GEMM (QKV, fc2)
#endif
// bit u set: WeightUse u on the CTA-pair GEMM with N = 128 and two epilogue groups (takes precedence)
#ifndef XTB_PAIRG_MASK
#define XTB_PAIRG_MASK 0x0
#endif
static constexpr bool kPairG[5] = {(XTB_PAIRG_MASK & 1) != 0, (XTB_PAIRG_MASK & 2) != 0, (XTB_PAIRG_MASK & 4) != 0,
                                   (XTB_PAIRG_MASK & 8) != 0, (XTB_PAIRG_MASK & 16) != 0};
static constexpr bool kPair[5] = {(XTB_PAIR_MASK & 1) != 0 && !kPairG[0], (XTB_PAIR_MASK & 2) != 0 && !kPairG[1],
                                  (XTB_PAIR_MASK & 4) != 0 && !kPairG[2], (XTB_PAIR_MASK & 8) != 0 && !kPairG[3],
                                  (XTB_PAIR_MASK & 16) != 0 && !kPairG[4]};

// Tile width of the single-CTA GEMM per weight use: 256 for the forward's projections; the stand-alone fp32-output
// GEMM (W_F32) takes XTB_F32_BN.
// 192 runs on 12 epilogue warps (three per TMEM lane quadrant, 64 columns each, so that no thread's columns straddle
// a 128-column block of weight scales): 135 tiles of 128 x 192 for config 1's 1025 x 2730 instead of 99 of 128 x 256.
#ifndef XTB_F32_BN
#define XTB_F32_BN 192
#endif
static constexpr int kF32EW = XTB_F32_BN == 192 ? 12 : 8;
static constexpr int kSingleBN[5] = {256, 256, 256, 256, XTB_F32_BN};
static constexpr int kSingleEW[5] = {8, 8, 8, 8, kF32EW};
using EpiF32Out = EpiF32<XTB_F32_BN / (kF32EW / 4)>;

int weight_box_rows(WeightUse u) { return kPairG[u] ? Gemm2GCfg::BN / 2 : kPair[u] ? Gemm2Cfg::BN / 2 : kSingleBN[u]; }

template <class Epi, WeightUse U>
static int run_proj(const Operand &a, const Weight8 &w, int M, float ascale, const typename Epi::Params &ep, cudaStream_t st,
                    const CUtensorMap *tmc = nullptr, uint32_t *err = nullptr)
{
    if (w.sf)  // power-of-two block scales
        return !w.sf_pair ? run_gemm_mx<Epi>(a, w, M, ascale, ep, st, tmc, err)
               : w.sf_wide ? run_gemm2_mx<Epi, 2>(a, w, M, ascale, ep, st, tmc, err)
                           : run_gemm2_mx<Epi, 1>(a, w, M, ascale, ep, st, tmc, err);
    if (!kPairG[U] && w.uniform > 0.0f) {  // one scale for the whole weight: accumulate over K in TMEM, scale once
        if constexpr (kPair[U])
            return run_gemm2<Epi, 256, false, false>(a, w.op, M, w.n, nullptr, 0, 1, ascale, ep, st, tmc, err, w.uniform);
        else
            return run_gemm<Epi, kSingleBN[U], false, false, false, kSingleEW[U]>(a, w.op, M, w.n, nullptr, 0, 1, ascale,
                                                                                  ep, st, tmc, err, w.uniform, true);
    }
    if constexpr (kPairG[U])
        return run_gemm2<Epi, 128, true>(a, w.op, M, w.n, w.ws, kb(w.k), kb(w.n), ascale, ep, st, tmc, err);
    else if constexpr (kPair[U])
        return run_gemm2<Epi>(a, w.op, M, w.n, w.ws, kb(w.k), kb(w.n), ascale, ep, st, tmc, err);
    else
        return run_gemm<Epi, kSingleBN[U], false, true, false, kSingleEW[U]>(a, w.op, M, w.n, w.ws, kb(w.k), kb(w.n),
                                                                             ascale, ep, st, tmc, err, 1.0f, true);
}

// Opt the projection kernel of (Epi, U) into its shared memory and check that its clusters fit (pair kernels).
template <class Epi, WeightUse U>
static int prepare_proj()
{
    if constexpr (kPairG[U]) {
        using Cfg = Gemm2CfgT<128, true, StagingOf<Epi>::v>;
        const void *k = (const void *)k_gemm2<Epi, true, 128, true>;
        return set_smem(k, Cfg::SMEM) || max_pairs(k, Cfg::THREADS, Cfg::SMEM) <= 0 ? -1 : 0;
    } else if constexpr (kPair[U]) {
        using Cfg = Gemm2CfgT<256, false, StagingOf<Epi>::v>;
        const void *k = (const void *)k_gemm2<Epi, true>, *ku = (const void *)k_gemm2<Epi, false>;
        return set_smem(k, Cfg::SMEM) || max_pairs(k, Cfg::THREADS, Cfg::SMEM) <= 0 || set_smem(ku, Cfg::SMEM) ||
                       max_pairs(ku, Cfg::THREADS, Cfg::SMEM) <= 0
                   ? -1
                   : 0;
    } else {
        return set_smem((const void *)k_gemm<Epi, kSingleBN[U], false, true, false, kSingleEW[U]>,
                        GemmCfg<kSingleBN[U], kSingleEW[U]>::SMEM) ||
                       set_smem((const void *)k_gemm<Epi, kSingleBN[U], false, false, false, kSingleEW[U]>,
                                GemmCfg<kSingleBN[U], kSingleEW[U]>::SMEM)
                   ? -1
                   : 0;
    }
}

int launch_gemm_f32(const Operand &a, const Weight8 &w, float ascale, float *out, int ldo, cudaStream_t st)
{
    if (w.sf) {  // power-of-two block scales: the block-scaled kernels, 128 accumulator columns per epilogue thread
        EpiF32<128>::Params p{out, ldo, a.rows, w.n};
        return !w.sf_pair ? run_gemm_mx<EpiF32<128>>(a, w, a.rows, ascale, p, st)
               : w.sf_wide ? run_gemm2_mx<EpiF32<128>, 2>(a, w, a.rows, ascale, p, st)
                           : run_gemm2_mx<EpiF32<128>, 1>(a, w, a.rows, ascale, p, st);
    }
    // fp32 block scales (or one per tensor): the single-CTA kernel on XTB_F32_BN-wide tiles
    EpiF32Out::Params p{out, ldo, a.rows, w.n};
    if (w.uniform > 0.0f)
        return run_gemm<EpiF32Out, XTB_F32_BN, false, false, false, kF32EW>(a, w.op, a.rows, w.n, nullptr, 0, 1, ascale,
                                                                          p, st, nullptr, nullptr, w.uniform, true);
    return run_gemm<EpiF32Out, XTB_F32_BN, false, true, false, kF32EW>(a, w.op, a.rows, w.n, w.ws, kb(w.k), kb(w.n),
                                                                     ascale, p, st, nullptr, nullptr, 1.0f, true);
}

int launch_patch_embed(const Operand &in, const Operand &pe, int nimg, const float *pos, __half *x, cudaStream_t st)
{
    EpiPatch::Params p{x, pos, nimg * NP};
    return run_gemm<EpiPatch, 256, true, false, false>(in, pe, nimg * NP, D, nullptr, 0, 1, 1.0f, p, st, nullptr,
                                                       nullptr, 1.0f, true);
}

int launch_ln_e4m3(const __half *x, const float *g, const float *b, uint8_t *y, int rows, float qs, cudaStream_t st)
{
    if (set_smem((const void *)k_ln_e4m3, LN_SMEM)) return -1;
    if (((uintptr_t)x & 15) || rows <= 0) {
        fprintf(stderr, "eva: layernorm input %p not 16-byte aligned or %d rows\n", (const void *)x, rows);
        return -1;
    }
    const int dev = current_device();
    int grid = LN_BLOCKS_PER_SM * num_sms(dev);
    const int need = (rows + LN_WARPS - 1) / LN_WARPS;
    if (grid > need) grid = need;
    XTB_CK(launch_pdl(k_ln_e4m3, dim3(grid), dim3(LN_WARPS * 32), LN_SMEM, st, x, g, b, y, rows, qs, error_word(dev)));
    return 0;
}

int launch_qkv(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *q8, uint8_t *k8, uint8_t *v8,
               const float *cs, float cq, float ck, float cv, cudaStream_t st)
{
    EpiQKV::Params p{q8, k8, v8, (const float2 *)cs, cq, ck, cv, rows};
    return run_proj<EpiQKV, W_QKV>(h, w, rows, ascale, p, st);
}

int make_attn(Attn *a, const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg)
{
    const uint64_t rows = (uint64_t)nimg * NH * TP;
    a->q8 = q8;
    a->k8 = k8;
    a->v8 = v8;
    if (make_tmap_2d(&a->tq, q8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tk, k8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tv, v8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    return 0;
}

int launch_attention(const Attn &a, int nimg, uint8_t *out, float sinv, float vo, cudaStream_t st, cudaStream_t st_last)
{
    if (set_smem((const void *)k_attention<AttEva>, ATT_SMEM)) return -1;
    dim3 grid(AttEva::PAIRS, NH, nimg);
    XTB_CK(launch_pdl(k_attention<AttEva>, grid, dim3(ATT_THREADS), ATT_SMEM, st, a.tq, a.tk, a.tv, out, sinv, vo,
                      error_word(current_device())));
    XTB_CK(cudaGetLastError());
    k_attention_last<<<nimg * NH, ATT_LAST_THREADS, 0, st_last ? st_last : st>>>(a.q8, a.k8, a.v8, out, sinv, vo);
    XTB_CK(cudaGetLastError());
    return 0;
}

// The fp16 residual x [rows][1024] as the target of TMA reduce-adds: boxes of 64 halves x 32 rows, 128B swizzle.
int resid_map(CUtensorMap *m, __half *x, int rows)
{
    return make_tmap_2d_typed(m, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, (uint64_t)rows, D * 2, 64, 32,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_oproj(const Operand &a, const Weight8 &w, float ascale, int rows, __half *x, cudaStream_t st)
{
    CUtensorMap xm;
    if (resid_map(&xm, x, rows)) return -1;
    EpiResid::Params p{rows};
    return run_proj<EpiResid, W_O>(a, w, rows, ascale, p, st, &xm);
}

int launch_fc1(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *h8, float2 *stat, const float *rs,
               cudaStream_t st)
{
    CUtensorMap hm;  // h8 [rows][2736] E4M3, stored in boxes of 64 units x 32 rows (64B swizzle)
    if (make_tmap_2d(&hm, h8, HIDP, (uint64_t)rows, HIDP, 64, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    EpiFC1::Params p{stat, rs, rows};
    return run_proj<EpiFC1, W_FC1>(h, w, rows, ascale, p, st, &hm);
}

int launch_fc2(const Operand &h8, const Weight8 &w, float ascale, int rows, __half *x, float2 *stat, const float *c,
               const float *d, cudaStream_t st)
{
    CUtensorMap xm;
    if (resid_map(&xm, x, rows)) return -1;
    // the epilogue sums each row's partials itself (no row-statistics launch; the partials are only read)
    return launch_fc2_gemm(h8, w, ascale, rows, xm, nullptr, stat, c, d, nullptr, st);
}

int launch_fc2_gemm(const Operand &h8, const Weight8 &w, float ascale, int rows, const CUtensorMap &xm, const float2 *ms,
                    const float2 *part, const float *c, const float *d, uint32_t *err, cudaStream_t st)
{
    EpiFC2::Params p{ms, part, c, d, rows};
    return run_proj<EpiFC2, W_FC2>(h8, w, rows, ascale, p, st, &xm, err);
}

// ---- 2:4-sparse projections ----
static_assert(SP_BT == SP_BOX_ROWS, "activation box height of the sparse kernels");

int make_sparse_weight(SparseW *w, const uint8_t *vals, const uint8_t *meta, int n, int k, const float *ws)
{
    if (n <= 0 || k <= 0 || (k & 3) || !vals || !meta || !ws) {
        fprintf(stderr, "eva: sparse weight [%d][%d]: bad shape or null pointer\n", n, k);
        return -1;
    }
    w->n = n;
    w->k = k;
    w->np = (n + 127) & ~127;
    w->kp = (k + 127) & ~127;
    w->ws = ws;
    if (make_tmap_2d(&w->va, vals, (uint64_t)w->kp / 2, (uint64_t)w->np, (uint64_t)w->kp / 2, 64, 128,
                     CU_TENSOR_MAP_SWIZZLE_64B))
        return -1;
    return make_tmap_2d(&w->me, meta, (uint64_t)w->kp / 8, (uint64_t)w->np, (uint64_t)w->kp / 8, 16, 128,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
}

// One launch of the sparse GEMM: persistent grid of one CTA per SM over (weight tile, token tile) pairs.
template <class Epi, bool PROMOTE>
static int run_gemm_sp_k(const SparseW &w, const Operand &x, int M, float ascale, const typename Epi::Params &ep,
                         cudaStream_t st, const CUtensorMap *tmc)
{
    auto kern = k_gemm_sp<Epi, PROMOTE>;
    if (set_smem((const void *)kern, SpCfg::SMEM)) return -1;
    if (x.row_bytes != w.k || x.box_rows != SP_BOX_ROWS || M <= 0 || M > x.rows) {
        fprintf(stderr, "eva: sparse gemm operands (K bytes %d vs %d, box %d rows, M %d of %d)\n", x.row_bytes, w.k,
                x.box_rows, M, x.rows);
        return -1;
    }
    const int dev = current_device();
    SpArgs g;
    g.M = M;
    g.kiters = w.kp / 128;
    g.n_tiles = w.np / 128;
    g.t_tiles = (M + SP_BT - 1) / SP_BT;
    g.ws = w.ws;
    g.ws_ld = kb(w.k);
    g.ws_rows = kb(w.n);
    g.ascale = ascale;
    g.wsu = w.uniform;
    g.err = error_word(dev);
    const int total = g.n_tiles * g.t_tiles;
    int grid = num_sms(dev);
    if (grid > total) grid = total;
    XTB_CK(launch_pdl(kern, dim3(grid), dim3(SpCfg::THREADS), SpCfg::SMEM, st, w.va, w.me, x.map, tmc ? *tmc : x.map, g,
                      ep));
    XTB_CK(cudaGetLastError());
    return 0;
}

template <class Epi>
static int run_gemm_sp(const SparseW &w, const Operand &x, int M, float ascale, const typename Epi::Params &ep,
                       cudaStream_t st, const CUtensorMap *tmc = nullptr)
{
    if (w.uniform > 0.0f) return run_gemm_sp_k<Epi, false>(w, x, M, ascale, ep, st, tmc);
    return run_gemm_sp_k<Epi, true>(w, x, M, ascale, ep, st, tmc);
}

int launch_gemm_sp_f32(const Operand &x, const SparseW &w, float ascale, float *out, int ldo, cudaStream_t st)
{
    SpF32::Params p{out, ldo, x.rows, w.n};
    return run_gemm_sp<SpF32>(w, x, x.rows, ascale, p, st);
}

int launch_qkv_sp(const Operand &h, const SparseW &w, float ascale, int rows, uint8_t *q8, uint8_t *k8, uint8_t *v8,
                  const float *cs, float cq, float ck, float cv, cudaStream_t st)
{
    SpQKV::Params p{q8, k8, v8, (const float2 *)cs, cq, ck, cv, rows};
    return run_gemm_sp<SpQKV>(w, h, rows, ascale, p, st);
}

// The fp16 residual as the target of the sparse kernels' reduce-adds: boxes of 32 halves x 112 rows, unswizzled.
static int sp_resid_map(CUtensorMap *m, __half *x, int rows)
{
    return make_tmap_2d_typed(m, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, (uint64_t)rows, D * 2, 32, SP_COLS,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
}

int launch_oproj_sp(const Operand &a, const SparseW &w, float ascale, int rows, __half *x, cudaStream_t st)
{
    CUtensorMap xm;
    if (sp_resid_map(&xm, x, rows)) return -1;
    SpResid<false>::Params p{nullptr, nullptr, nullptr, rows};
    return run_gemm_sp<SpResid<false>>(w, a, rows, ascale, p, st, &xm);
}

int launch_fc1_sp(const Operand &h, const SparseW &w, float ascale, int rows, uint8_t *h8, float2 *stat, const float *rs,
                  cudaStream_t st)
{
    CUtensorMap hm;  // h8 [rows][2736] E4M3, stored in boxes of 16 units x 112 rows
    if (make_tmap_2d(&hm, h8, HIDP, (uint64_t)rows, HIDP, 16, SP_COLS, CU_TENSOR_MAP_SWIZZLE_NONE)) return -1;
    SpFC1::Params p{stat, rs, rows};
    return run_gemm_sp<SpFC1>(w, h, rows, ascale, p, st, &hm);
}

int launch_fc2_sp(const Operand &h8, const SparseW &w, float ascale, int rows, __half *x, float2 *stat, const float *c,
                  const float *d, cudaStream_t st)
{
    CUtensorMap xm;
    if (sp_resid_map(&xm, x, rows)) return -1;
    XTB_CK(launch_pdl(k_rowstat, dim3(rowstat_blocks(rows)), dim3(ROWSTAT_THREADS), 0, st, (float2 *)stat, rows));
    XTB_CK(cudaGetLastError());
    SpResid<true>::Params p{stat, c, d, rows};
    return run_gemm_sp<SpResid<true>>(w, h8, rows, ascale, p, st, &xm);
}

// The E4M3 encoders every epilogue uses, over a whole array: pairs through e4m3x2 (or, with via_f16, through the
// attention output's fp16 staging, e4m3x2_via_f16), one pair per thread, a last odd element paired with 0.
__global__ void k_e4m3_encode(const float *__restrict__ x, uint8_t *__restrict__ y, size_t n, int via_f16)
{
    const size_t i = 2 * ((size_t)blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    const float a = x[i], b = i + 1 < n ? x[i + 1] : 0.f;
    const uint32_t w = via_f16 ? e4m3x2_via_f16(a, b) : e4m3x2(a, b);
    y[i] = (uint8_t)w;
    if (i + 1 < n) y[i + 1] = (uint8_t)(w >> 8);
}

int launch_e4m3_encode(const float *x, uint8_t *y, size_t n, int via_f16, cudaStream_t st)
{
    if (!n) return 0;
    const size_t pairs = (n + 1) / 2;
    k_e4m3_encode<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(x, y, n, via_f16);
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_amax_f16(const __half *x, int K, int rows, float *amax, cudaStream_t st)
{
    if (K <= 0 || (K & 7) || rows <= 0 || ((uintptr_t)x & 15)) {
        fprintf(stderr, "eva: amax: bad shape %d x %d (K a multiple of 8, 16-byte aligned rows)\n", rows, K);
        return -1;
    }
    k_amax<<<dim3((K / 8 + 127) / 128, std::min(rows, 64)), 128, 0, st>>>(x, K, rows, (unsigned *)amax);
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_selftest_wait(uint32_t timeout_us, int arrive, cudaStream_t st)
{
    k_selftest_wait<<<1, 32, 0, st>>>((uint64_t)timeout_us * 1000, arrive, error_word(current_device()));
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_pool_ln(const __half *x, int nimg, const float *g, const float *b, float *pool, __half *pn, uint8_t *pn8,
                   float qs_head, cudaStream_t st)
{
    XTB_CK(launch_pdl(k_pool, dim3(nimg, D / 64), dim3(256), 0, st, x, pool));
    XTB_CK(cudaGetLastError());
    XTB_CK(launch_pdl(k_ln_head, dim3((nimg + 7) / 8), dim3(256), 0, st, pool, g, b, pn, pn8, nimg, qs_head));
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_head_f16(const Operand &hw, const Operand &pn, int nimg, int nt, const float *hb, float *out, cudaStream_t st)
{
    EpiHead<32>::Params p{out, hb, nt, nimg};
    return run_gemm<EpiHead<32>, 64, true, false, false>(hw, pn, nt, nimg, nullptr, 0, 1, 1.0f, p, st);
}

int launch_head_e4m3(const Weight8 &hw, const Operand &pn8, float ascale, int nimg, int nt, const float *hb, float *out,
                     cudaStream_t st)
{
    EpiHead<32>::Params p{out, hb, nt, nimg};
    return run_gemm<EpiHead<32>, 64, false, true, true>(hw.op, pn8, nt, nimg, hw.ws, kb(hw.k), kb(hw.n), ascale, p, st);
}

// Opt every kernel of the forward into its dynamic shared memory on the current device. Must run before a stream
// capture: cudaFuncSetAttribute is not a stream operation and invalidates a capture in progress.
int prepare_kernels()
{
    const int dev = current_device();
    if (!error_word(dev) || num_sms(dev) <= 0) {  // address looked up once per device: never inside a capture
        fprintf(stderr, "eva: cannot look up the error word on device %d\n", dev);
        return -1;
    }
    const void *single[] = {(const void *)k_gemm<EpiPatch, 256, true, false, false>};
    for (const void *k : single)
        if (set_smem(k, GemmCfg<256>::SMEM)) return -1;
    if (prepare_proj<EpiQKV, W_QKV>() || prepare_proj<EpiResid, W_O>() || prepare_proj<EpiFC1, W_FC1>() ||
        prepare_proj<EpiFC2, W_FC2>() || prepare_proj<EpiF32Out, W_F32>())
        return -1;
    const void *g64[] = {(const void *)k_gemm<EpiHead<32>, 64, true, false, false>,
                         (const void *)k_gemm<EpiHead<32>, 64, false, true, true>};
    for (const void *k : g64)
        if (set_smem(k, GemmCfg<64>::SMEM)) return -1;
    const void *sp[] = {(const void *)k_gemm_sp<SpF32, true>,          (const void *)k_gemm_sp<SpQKV, true>,
                        (const void *)k_gemm_sp<SpResid<false>, true>, (const void *)k_gemm_sp<SpResid<true>, true>,
                        (const void *)k_gemm_sp<SpFC1, true>,          (const void *)k_gemm_sp<SpF32, false>,
                        (const void *)k_gemm_sp<SpQKV, false>,         (const void *)k_gemm_sp<SpResid<false>, false>,
                        (const void *)k_gemm_sp<SpResid<true>, false>, (const void *)k_gemm_sp<SpFC1, false>};
    for (const void *k : sp)
        if (set_smem(k, SpCfg::SMEM)) return -1;
    if (set_smem((const void *)k_ln_e4m3, LN_SMEM)) return -1;
    if (set_smem((const void *)k_attention<AttEva>, ATT_SMEM)) return -1;
    if (set_smem((const void *)k_gemm_mx<EpiFC1>, GemmMxCfg<StagingOf<EpiFC1>::v>::SMEM) ||
        set_smem((const void *)k_gemm_mx<EpiQKV>, GemmMxCfg<StagingOf<EpiQKV>::v>::SMEM) ||
        set_smem((const void *)k_gemm_mx<EpiResid>, GemmMxCfg<StagingOf<EpiResid>::v>::SMEM) ||
        set_smem((const void *)k_gemm_mx<EpiFC2>, GemmMxCfg<StagingOf<EpiFC2>::v>::SMEM))
        return -1;
    {
        const void *k2[] = {(const void *)k_gemm2_mx<EpiQKV>, (const void *)k_gemm2_mx<EpiFC1>,
                            (const void *)k_gemm2_mx<EpiFC2>, (const void *)k_gemm2_mx<EpiResid>};
        const size_t sm2[] = {Gemm2MxCfg<StagingOf<EpiQKV>::v>::SMEM, Gemm2MxCfg<StagingOf<EpiFC1>::v>::SMEM,
                              Gemm2MxCfg<StagingOf<EpiFC2>::v>::SMEM, Gemm2MxCfg<StagingOf<EpiResid>::v>::SMEM};
        for (int i = 0; i < 4; i++)
            if (set_smem(k2[i], sm2[i]) || max_pairs(k2[i], 320, sm2[i]) <= 0) return -1;
        const void *k2w[] = {(const void *)k_gemm2_mx<EpiQKV, 2>, (const void *)k_gemm2_mx<EpiFC2, 2>,
                             (const void *)k_gemm2_mx<EpiResid, 2>, (const void *)k_gemm2_mx<EpiFC1, 2>};
        const size_t sm2w[] = {Gemm2MxCfg<StagingOf<EpiQKV>::v, 2>::SMEM, Gemm2MxCfg<StagingOf<EpiFC2>::v, 2>::SMEM,
                               Gemm2MxCfg<StagingOf<EpiResid>::v, 2>::SMEM, Gemm2MxCfg<StagingOf<EpiFC1>::v, 2>::SMEM};
        for (int i = 0; i < 4; i++)
            if (set_smem(k2w[i], sm2w[i]) || max_pairs(k2w[i], 320, sm2w[i]) <= 0) return -1;
    }
    return 0;
}

// ---- PixAI ----
using AttPxW = AttSeq<PX_LW, PX_LW, (PX_LW + 127) / 128>;
using AttPxG = AttSeq<PX_T, PX_T, (PX_T + 127) / 128>;

int launch_px_patch(const Operand &in, const Operand &pe, int rows, __half *x, cudaStream_t st)
{
    EpiPxPatch::Params p{x, rows};
    return run_gemm<EpiPxPatch, 256, true, false, false>(in, pe, rows, D, nullptr, 0, 1, 1.0f, p, st, nullptr,
                                                         nullptr, 1.0f, true);
}

int launch_px_embed(__half *x, const float *pos, const float *w, const float *b, int rows, cudaStream_t st)
{
    XTB_CK(launch_pdl(k_px_embed, dim3((rows + 7) / 8), dim3(256), 0, st, x, pos, w, b, rows));
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_px_qkv(const Operand &h, const Weight8 &w, float ascale, int rows, int L, uint8_t *q8, uint8_t *k8,
                  uint8_t *v8, const float *cs, const float *bias, float cq, float ck, float cv, cudaStream_t st)
{
    if (w.uniform <= 0.0f || (L != PX_LW && L != PX_T) || rows % L) {
        fprintf(stderr, "eva: px qkv: per-tensor weights and whole sequences of 576 or 5184 rows expected\n");
        return -1;
    }
    EpiPxQKV::Params p{q8, k8, v8, (const float2 *)cs, bias, cq, ck, cv, rows, L};
    return run_proj<EpiPxQKV, W_QKV>(h, w, rows, ascale, p, st);
}

int make_attn_rows(Attn *a, const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int rows)
{
    const uint64_t r = (uint64_t)rows * NH;
    a->q8 = q8;
    a->k8 = k8;
    a->v8 = v8;
    if (make_tmap_2d(&a->tq, q8, HD, r, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tk, k8, HD, r, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tv, v8, HD, r, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    return 0;
}

template <class SQ>
static int run_attention_seq(const Attn &a, int nseq, uint8_t *out, float sinv, float vo, cudaStream_t st)
{
    auto kern = k_attention<SQ>;
    if (set_smem((const void *)kern, ATT_SMEM)) return -1;
    dim3 grid(SQ::PAIRS, NH, nseq);
    XTB_CK(launch_pdl(kern, grid, dim3(ATT_THREADS), ATT_SMEM, st, a.tq, a.tk, a.tv, out, sinv, vo,
                      error_word(current_device())));
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_px_attention(const Attn &a, int nseq, int L, uint8_t *out, float sinv, float vo, cudaStream_t st)
{
    if (L == PX_LW) return run_attention_seq<AttPxW>(a, nseq, out, sinv, vo, st);
    if (L == PX_T) return run_attention_seq<AttPxG>(a, nseq, out, sinv, vo, st);
    fprintf(stderr, "eva: px attention: sequence length %d (576 or 5184)\n", L);
    return -1;
}

int launch_px_resid(const Operand &a, const Weight8 &w, float ascale, int rows, const CUtensorMap &xm,
                    const float *bias, WeightUse use, cudaStream_t st)
{
    if (w.uniform <= 0.0f) return -1;
    EpiPxResid::Params p{bias, rows};
    if (use == W_O) return run_proj<EpiPxResid, W_O>(a, w, rows, ascale, p, st, &xm);
    if (use == W_FC2) return run_proj<EpiPxResid, W_FC2>(a, w, rows, ascale, p, st, &xm);
    return -1;
}

int px_u8_map(CUtensorMap *m, uint8_t *u8, int rows)
{
    return make_tmap_2d(m, u8, PX_HID, (uint64_t)rows, PX_HID, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_px_fc1(const Operand &h, const Weight8 &w, float ascale, int rows, const CUtensorMap &um, const float *b1,
                  const float *rs, cudaStream_t st)
{
    if (w.uniform <= 0.0f) return -1;
    EpiPxFC1::Params p{b1, rs, rows};
    return run_proj<EpiPxFC1, W_FC1>(h, w, rows, ascale, p, st, &um);
}

int launch_px_head(const __half *x, int nimg, const float *w, const float *b, const __half *hpos, const float *U,
                   const __half *wv, __half *y, float *s, __half *P, float *part, __half *o, cudaStream_t st)
{
    if (set_smem((const void *)k_px_head_ln_score, PX_HEAD_SMEM)) return -1;
    const int rows = nimg * PX_T;
    int grid = 3 * num_sms(current_device());
    if (grid > (rows + 7) / 8) grid = (rows + 7) / 8;
    XTB_CK(launch_pdl(k_px_head_ln_score, dim3(grid), dim3(256), PX_HEAD_SMEM, st, x, w, b, hpos, U, y, s, rows));
    XTB_CK(cudaGetLastError());
    XTB_CK(launch_pdl(k_px_head_softmax, dim3(nimg * NH), dim3(256), 0, st, s, P));
    XTB_CK(cudaGetLastError());
    XTB_CK(launch_pdl(k_px_head_pool, dim3(nimg, PX_NCH), dim3(512), 0, st, P, y, part));
    XTB_CK(cudaGetLastError());
    XTB_CK(launch_pdl(k_px_head_v, dim3(nimg * NH), dim3(256), 0, st, part, wv, o));
    XTB_CK(cudaGetLastError());
    return 0;
}

// Shared-memory opt-in of the PixAI kernels (before a stream capture).
int prepare_px_kernels()
{
    if (prepare_kernels()) return -1;
    if (set_smem((const void *)k_gemm<EpiPxPatch, 256, true, false, false>, GemmCfg<256>::SMEM)) return -1;
    if (prepare_proj<EpiPxQKV, W_QKV>() || prepare_proj<EpiPxResid, W_O>() || prepare_proj<EpiPxFC1, W_FC1>() ||
        prepare_proj<EpiPxResid, W_FC2>())
        return -1;
    if (set_smem((const void *)k_attention<AttPxW>, ATT_SMEM) || set_smem((const void *)k_attention<AttPxG>, ATT_SMEM))
        return -1;
    return set_smem((const void *)k_px_head_ln_score, PX_HEAD_SMEM);
}

}  // namespace xtb

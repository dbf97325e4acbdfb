// Kernel launchers: pick the template instance, build the launch shape, enqueue. No allocation, no sync.
#include <mutex>
#include <set>

#include "attention.cuh"
#include "epilogues.cuh"
#include "gemm.cuh"
#include "host.h"
#include "ops.h"
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

// One launch of the tcgen05 GEMM: A = a (M rows), B = b (N rows), K slices of 128 bytes.
template <class Epi, int BN, bool F16, bool PROMOTE, bool WS_ON_M>
static int run_gemm(const Operand &a, const Operand &b, int M, int N, const float *ws, int ws_ld, int ws_rows, float ascale,
                    const typename Epi::Params &ep, cudaStream_t st, const CUtensorMap *tmc = nullptr)
{
    using Cfg = GemmCfg<BN>;
    auto kern = k_gemm<Epi, BN, F16, PROMOTE, WS_ON_M>;
    if (set_smem((const void *)kern, Cfg::SMEM)) return -1;
    if (a.row_bytes != b.row_bytes || M <= 0 || N <= 0) {
        fprintf(stderr, "eva: gemm shape mismatch (K bytes %d vs %d, M %d, N %d)\n", a.row_bytes, b.row_bytes, M, N);
        return -1;
    }
    const int dev = current_device();
    GemmArgs g;
    g.M = M;
    g.N = N;
    g.kiters = (a.row_bytes + 127) / 128;
    g.m_tiles = (M + 127) / 128;
    g.n_tiles = (N + BN - 1) / BN;
    g.ws = ws;
    g.ws_ld = ws_ld;
    g.ws_rows = ws_rows;
    g.ascale = ascale;
    g.err = error_word(dev);
    const int total = g.m_tiles * g.n_tiles;
    int grid = num_sms(dev);
    if (grid > total) grid = total;
    kern<<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(a.map, b.map, tmc ? *tmc : a.map, g, ep);
    XTB_CK(cudaGetLastError());
    return 0;
}

static int kb(int k) { return (k + 127) / 128; }

int launch_gemm_f32(const Operand &a, const Weight8 &w, float ascale, float *out, int ldo, cudaStream_t st)
{
    EpiF32<128>::Params p{out, ldo, a.rows, w.n};
    return run_gemm<EpiF32<128>, 256, false, true, false>(a, w.op, a.rows, w.n, w.ws, kb(w.k), kb(w.n), ascale, p, st);
}

int launch_patch_embed(const Operand &in, const Operand &pe, int nimg, const float *pos, __half *x, cudaStream_t st)
{
    EpiPatch::Params p{x, pos, nimg * NP};
    return run_gemm<EpiPatch, 256, true, false, false>(in, pe, nimg * NP, D, nullptr, 0, 1, 1.0f, p, st);
}

int launch_ln_e4m3(const __half *x, const float *g, const float *b, uint8_t *y, int rows, float qs, cudaStream_t st)
{
    k_ln_e4m3<<<(rows + 7) / 8, 256, 0, st>>>(x, g, b, y, rows, qs);
    XTB_CK(cudaGetLastError());
    return 0;
}

int launch_qkv(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *q8, uint8_t *k8, uint8_t *v8,
               const float *cs, float cq, float ck, float cv, cudaStream_t st)
{
    EpiQKV::Params p{q8, k8, v8, (const float2 *)cs, cq, ck, cv, rows};
    return run_gemm<EpiQKV, 256, false, true, false>(h, w.op, rows, 3 * D, w.ws, kb(w.k), kb(w.n), ascale, p, st);
}

int make_attn(Attn *a, const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg)
{
    const uint64_t rows = (uint64_t)nimg * NH * TP;
    if (make_tmap_2d(&a->tq, q8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tk, k8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    if (make_tmap_2d(&a->tv, v8, HD, rows, HD, HD, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    return 0;
}

int launch_attention(const Attn &a, int nimg, uint8_t *out, float sinv, float vo, cudaStream_t st)
{
    if (set_smem((const void *)k_attention, ATT_SMEM)) return -1;
    dim3 grid(QT, NH, nimg);
    k_attention<<<grid, ATT_THREADS, ATT_SMEM, st>>>(a.tq, a.tk, a.tv, out, sinv, vo, error_word(current_device()));
    XTB_CK(cudaGetLastError());
    return 0;
}

// The fp16 residual x [rows][1024] as the target of TMA reduce-adds: boxes of 64 halves x 32 rows, 128B swizzle.
static int resid_map(CUtensorMap *m, __half *x, int rows)
{
    return make_tmap_2d_typed(m, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, D, (uint64_t)rows, D * 2, 64, 32,
                              CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_oproj(const Operand &a, const Weight8 &w, float ascale, int rows, __half *x, cudaStream_t st)
{
    CUtensorMap xm;
    if (resid_map(&xm, x, rows)) return -1;
    EpiResid::Params p{rows};
    return run_gemm<EpiResid, 256, false, true, false>(a, w.op, rows, D, w.ws, kb(w.k), kb(w.n), ascale, p, st, &xm);
}

int launch_fc1(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *h8, float2 *stat, const float *rs,
               cudaStream_t st)
{
    CUtensorMap hm;  // h8 [rows][2736] E4M3, stored in boxes of 64 units x 32 rows (64B swizzle)
    if (make_tmap_2d(&hm, h8, HIDP, (uint64_t)rows, HIDP, 64, 32, CU_TENSOR_MAP_SWIZZLE_64B)) return -1;
    EpiFC1::Params p{stat, rs, rows};
    return run_gemm<EpiFC1, 256, false, true, false>(h, w.op, rows, N12, w.ws, kb(w.k), kb(w.n), ascale, p, st, &hm);
}

int launch_fc2(const Operand &h8, const Weight8 &w, float ascale, int rows, __half *x, float2 *stat, const float *c,
               const float *d, cudaStream_t st)
{
    CUtensorMap xm;
    if (resid_map(&xm, x, rows)) return -1;
    k_rowstat<<<(rows + 255) / 256, 256, 0, st>>>(stat, rows);
    XTB_CK(cudaGetLastError());
    EpiFC2::Params p{stat, c, d, rows};
    return run_gemm<EpiFC2, 256, false, true, false>(h8, w.op, rows, D, w.ws, kb(w.k), kb(w.n), ascale, p, st, &xm);
}

int launch_pool_ln(const __half *x, int nimg, const float *g, const float *b, float *pool, __half *pn, uint8_t *pn8,
                   float qs_head, cudaStream_t st)
{
    k_pool<<<dim3(nimg, D / 64), 256, 0, st>>>(x, pool);
    XTB_CK(cudaGetLastError());
    k_ln_head<<<(nimg + 7) / 8, 256, 0, st>>>(pool, g, b, pn, pn8, nimg, qs_head);
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
    if (!error_word(dev) || num_sms(dev) <= 0) {  // lazily created per device: never inside a capture
        fprintf(stderr, "eva: cannot set up the error word on device %d\n", dev);
        return -1;
    }
    const void *g256[] = {
        (const void *)k_gemm<EpiF32<128>, 256, false, true, false>, (const void *)k_gemm<EpiPatch, 256, true, false, false>,
        (const void *)k_gemm<EpiQKV, 256, false, true, false>,      (const void *)k_gemm<EpiResid, 256, false, true, false>,
        (const void *)k_gemm<EpiFC1, 256, false, true, false>,      (const void *)k_gemm<EpiFC2, 256, false, true, false>};
    for (const void *k : g256)
        if (set_smem(k, GemmCfg<256>::SMEM)) return -1;
    const void *g64[] = {(const void *)k_gemm<EpiHead<32>, 64, true, false, false>,
                         (const void *)k_gemm<EpiHead<32>, 64, false, true, true>};
    for (const void *k : g64)
        if (set_smem(k, GemmCfg<64>::SMEM)) return -1;
    return set_smem((const void *)k_attention, ATT_SMEM);
}

}  // namespace xtb

// Internal C++ interface between the engine and the kernel launchers (ops.cu). Every launcher returns 0 or -1
// (with an "eva: ..." line on stderr) and only enqueues work on the given stream: no allocation, no sync.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xtb {

// Model shapes (EVA02-Large tagger, 448^2 input, patch 14).
constexpr int D = 1024, T = 1025, NP = 1024, HID = 2730, HIDP = 2736, K0P = 592, NH = 16, HD = 64;
constexpr int N12 = 2 * HIDP;                     // fc1 output rows (g / x interleaved in 16-unit chunks)
constexpr int NSTAT = (N12 + 127) / 128;          // fc1 row-statistics partials per row (one per 128 fc1 columns)
constexpr int TP = 1152;                          // attention keys per (image, head), padded to 9 x 128
constexpr int QT = (T + 127) / 128;               // 128-query tiles per (image, head)

// Prepared operand: a row-major byte matrix plus its TMA descriptor (box = 128 bytes x box_rows, 128B swizzle).
struct Operand {
    CUtensorMap map;
    const void *ptr;
    int rows, row_bytes, box_rows;
};
// Box height of every A (activation) operand.
constexpr int A_BOX_ROWS = 128;
int make_operand(Operand *op, const void *ptr, int rows, int row_bytes, int box_rows);

// The block-scaled projections. Each runs on the GEMM kernel measured fastest for its shape (the single-CTA
// 128 x 256 tile of gemm.cuh, or the 256 x 256 CTA-pair tile of gemm2.cuh), which fixes the box height its weight
// operand is read in: weight_box_rows(use).
enum WeightUse { W_QKV = 0, W_O = 1, W_FC1 = 2, W_FC2 = 3, W_F32 = 4 };
int weight_box_rows(WeightUse u);

// Block-scaled weight: E4M3 [n][k] plus fp32 scales [ceil(n / 128)][ceil(k / 128)]. uniform > 0: every block scale
// equals it (the reference's per-tensor v3 weights): the GEMM accumulates the whole K range in TMEM and scales
// once, as the reference's kernels do (alpha = w_dq a_dq after the fp32 sum), instead of promoting every K block.
struct Weight8 {
    Operand op;
    const float *ws;
    int n, k;
    float uniform = 0.0f;
    // every block scale a power of two: its scale-factor image ([k/128][sf_nbp][512] bytes, each record one UE8M0
    // exponent repeated) for the tensor core's own block scaling (gemm_mx.cuh); null otherwise
    const uint8_t *sf = nullptr;
    int sf_nbp = 0;
    // run on the CTA-pair block-scaled kernel (gemm2_mx.cuh: the operand op in 64-row boxes, sfmap over sf)
    bool sf_pair = false;
    // on the pair kernel, 256-column tiles (two weight blocks per tile, one accumulator): half the A traffic per FLOP
    bool sf_wide = false;
    CUtensorMap sfmap;
};
// The scale-factor image as the pair kernel's tensor map (512-byte records as 2 rows of 256 bytes).
int sf_map(CUtensorMap *m, const uint8_t *sf, int n, int k);
// Scale-factor image of block scales ws [ceil(n/128)][ceil(k/128)] (host memory) into img (sf_image_bytes(n, k)
// bytes): 0 if every scale is a power of two (a normal float with a zero mantissa), else -1 and img untouched.
size_t sf_image_bytes(int n, int k);
int sf_image(const float *ws, int n, int k, uint8_t *img);

struct Attn {
    CUtensorMap tq, tk, tv;
    const uint8_t *q8, *k8, *v8;
};

// ---- launchers (device pointers; stream-ordered) ----
int launch_gemm_f32(const Operand &a, const Weight8 &w, float ascale, float *out, int ldo, cudaStream_t st);
int launch_patch_embed(const Operand &in, const Operand &pe, int nimg, const float *pos, __half *x, cudaStream_t st);
int launch_ln_e4m3(const __half *x, const float *g, const float *b, uint8_t *y, int rows, float qs, cudaStream_t st);
int launch_qkv(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *q8, uint8_t *k8, uint8_t *v8,
               const float *cs, float cq, float ck, float cv, cudaStream_t st);
int make_attn(Attn *a, const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg);
// st_last: the stream of the last query row's kernel (independent of the main kernel: both read q8 / k8 / v8 and
// write disjoint rows of out); st when null
int launch_attention(const Attn &a, int nimg, uint8_t *out, float sinv, float vo, cudaStream_t st,
                     cudaStream_t st_last = nullptr);
int launch_oproj(const Operand &a, const Weight8 &w, float ascale, int rows, __half *x, cudaStream_t st);
int launch_fc1(const Operand &h, const Weight8 &w, float ascale, int rows, uint8_t *h8, float2 *stat, const float *rs,
               cudaStream_t st);
// stat: fc1's [NSTAT][rows] partials, only read: the GEMM's epilogue sums each row's partials (EpiFC2::begin).
int launch_fc2(const Operand &h8, const Weight8 &w, float ascale, int rows, __half *x, float2 *stat, const float *c,
               const float *d, cudaStream_t st);
// The fc2 GEMM alone, with (mean, rstd) per row already in ms (part null), or summed by the epilogue from fc1's
// partials (part), bounded-wait failures reported in *err (the library's error word when null). Allocates nothing.
int launch_fc2_gemm(const Operand &h8, const Weight8 &w, float ascale, int rows, const CUtensorMap &xm, const float2 *ms,
                    const float2 *part, const float *c, const float *d, uint32_t *err, cudaStream_t st);
// The fp16 residual x [rows][1024] as the target of TMA reduce-adds.
int resid_map(CUtensorMap *m, __half *x, int rows);
int launch_pool_ln(const __half *x, int nimg, const float *g, const float *b, float *pool, __half *pn, uint8_t *pn8,
                   float qs_head, cudaStream_t st);
int launch_head_f16(const Operand &hw, const Operand &pn, int nimg, int nt, const float *hb, float *out,
                    cudaStream_t st);
int launch_head_e4m3(const Weight8 &hw, const Operand &pn8, float ascale, int nimg, int nt, const float *hb, float *out,
                     cudaStream_t st);

// ---- 2:4-sparse projections (gemm_sp.cuh, tcgen05.mma.sp) ----
// Weight compressed by sparse24_compress: values [np][kp / 2] (64-byte x 128-row boxes, 64B swizzle) and metadata
// [np][kp / 8] (16-byte x 128-row boxes), np / kp = n / k rounded up to 128, plus the dense block scales.
struct SparseW {
    CUtensorMap va, me;
    const float *ws;
    int n, k, np, kp;
    float uniform = 0.0f;  // > 0: every block scale equals it (no per-K-block promotion, see Weight8)
};
// Box height of the activation operand of the sparse kernels (tokens per tile).
constexpr int SP_BOX_ROWS = 112;
// 1 if every group of four consecutive k of every row holds at most two nonzero E4M3 codes (k a multiple of 4).
int sparse24_check(const uint8_t *w, int n, int k);
// Bytes of the compressed form (values, then metadata at *meta_off).
size_t sparse24_bytes(int n, int k, size_t *meta_off);
// Host memory in and out; -1 (with a stderr line) if w is not 2:4.
int sparse24_compress(const uint8_t *w, int n, int k, uint8_t *vals, uint8_t *meta);
int make_sparse_weight(SparseW *w, const uint8_t *vals, const uint8_t *meta, int n, int k, const float *ws);
int launch_gemm_sp_f32(const Operand &x, const SparseW &w, float ascale, float *out, int ldo, cudaStream_t st);
int launch_qkv_sp(const Operand &h, const SparseW &w, float ascale, int rows, uint8_t *q8, uint8_t *k8, uint8_t *v8,
                  const float *cs, float cq, float ck, float cv, cudaStream_t st);
int launch_oproj_sp(const Operand &a, const SparseW &w, float ascale, int rows, __half *x, cudaStream_t st);
int launch_fc1_sp(const Operand &h, const SparseW &w, float ascale, int rows, uint8_t *h8, float2 *stat, const float *rs,
                  cudaStream_t st);
int launch_fc2_sp(const Operand &h8, const SparseW &w, float ascale, int rows, __half *x, float2 *stat, const float *c,
                  const float *d, cudaStream_t st);

// ---- PixAI tagger (pixai.cuh; ViTDet-L at 1008^2, window-major tokens) ----
constexpr int PXT = 5184, PXLW = 576, PXHID = 4736;
int launch_px_patch(const Operand &in, const Operand &pe, int rows, __half *x, cudaStream_t st);
int launch_px_embed(__half *x, const float *pos, const float *w, const float *b, int rows, cudaStream_t st);
int launch_px_qkv(const Operand &h, const Weight8 &w, float ascale, int rows, int L, uint8_t *q8, uint8_t *k8,
                  uint8_t *v8, const float *cs, const float *bias, float cq, float ck, float cv, cudaStream_t st);
// q8 / k8 / v8 [rows / L][16][L][64] for both sequence lengths: one set of tensor maps over rows * 16 rows of 64
int make_attn_rows(Attn *a, const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int rows);
// L = 576 (windows) or 5184 (global): nseq sequences of L tokens -> out [nseq L][1024] E4M3
int launch_px_attention(const Attn &a, int nseq, int L, uint8_t *out, float sinv, float vo, cudaStream_t st);
// x (fp16 [rows][1024], as the TMA target xm) += alpha a W^T + bias
int launch_px_resid(const Operand &a, const Weight8 &w, float ascale, int rows, const CUtensorMap &xm,
                    const float *bias, WeightUse use, cudaStream_t st);
// u8 [rows][4736] = E4M3(rs * gelu(alpha h W1^T + b1)); um: its tensor map (128-byte x 32-row boxes)
int launch_px_fc1(const Operand &h, const Weight8 &w, float ascale, int rows, const CUtensorMap &um, const float *b1,
                  const float *rs, cudaStream_t st);
int px_u8_map(CUtensorMap *m, uint8_t *u8, int rows);
// attention-pool head: y, s, P, part scratch; o [nimg][1024] fp16
int prepare_px_kernels();
int launch_px_head(const __half *x, int nimg, const float *w, const float *b, const __half *hpos, const float *U,
                   const __half *wv, __half *y, float *s, __half *P, float *part, __half *o, cudaStream_t st);

// Per-column max |x| of an fp16 [rows][K] tensor folded into amax (fp32, K a multiple of 8).
int launch_amax_f16(const __half *x, int K, int rows, float *amax, cudaStream_t st);
int launch_e4m3_encode(const float *x, uint8_t *y, size_t n, int via_f16, cudaStream_t st);

// Failure-path self-test: a wait of at most timeout_us on a barrier that is (arrive) or is not arrived on.
int launch_selftest_wait(uint32_t timeout_us, int arrive, cudaStream_t st);

int current_device();
// Shared-memory opt-in of every kernel on the current device (call before any stream capture).
int prepare_kernels();

}  // namespace xtb

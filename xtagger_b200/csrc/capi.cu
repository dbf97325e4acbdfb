// Kernel-level C ABI: one entry point per hot-path kernel, device pointers in, stream-ordered, no allocation.
// These are what the parity tests drive; the engine (engine.cpp) strings the same launchers into a CUDA graph.
#include "../../include/xtagger_b200.h"
#include "host.h"
#include "ops.h"

using namespace xtb;

static cudaStream_t S(void *s)
{
    prepare_kernels();  // once per device; cheap afterwards
    return (cudaStream_t)s;
}

extern "C" {

int xtb_gemm_e4m3_f32(const uint8_t *a, int m, int k, const uint8_t *w, int n, const float *wscale, float ascale,
                      float *out, void *stream)
{
    Operand A;
    Weight8 W;
    if (m <= 0 || n <= 0 || k <= 0 || (k & 15)) {
        fprintf(stderr, "eva: xtb_gemm_e4m3_f32: bad shape m %d n %d k %d (k must be a multiple of 16)\n", m, n, k);
        return -1;
    }
    if (make_operand(&A, a, m, k, A_BOX_ROWS) || make_operand(&W.op, w, n, k, weight_box_rows(W_F32))) return -1;
    W.ws = wscale;
    W.n = n;
    W.k = k;
    return launch_gemm_f32(A, W, ascale, out, n, S(stream));
}

static int rows_ok(int rows, const char *what)
{
    if (rows <= 0) {
        fprintf(stderr, "eva: %s: bad row count %d\n", what, rows);
        return 0;
    }
    return 1;
}

static int weight(Weight8 *w, const uint8_t *p, int n, int k, const float *ws, WeightUse use)
{
    w->ws = ws;
    w->n = n;
    w->k = k;
    return make_operand(&w->op, p, n, k, weight_box_rows(use));
}

int xtb_ln_e4m3(const uint16_t *x, const float *g, const float *b, uint8_t *y, int rows, float qs, void *stream)
{
    if (!rows_ok(rows, "xtb_ln_e4m3")) return -1;
    return launch_ln_e4m3((const __half *)x, g, b, y, rows, qs, S(stream));
}

int xtb_qkv(const uint8_t *h, int rows, const uint8_t *w, const float *ws, float ascale, uint8_t *q8, uint8_t *k8,
            uint8_t *v8, const float *cs, float cq, float ck, float cv, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(rows, "xtb_qkv") || make_operand(&A, h, rows, D, 128) || weight(&W, w, 3 * D, D, ws, W_QKV)) return -1;
    return launch_qkv(A, W, ascale, rows, q8, k8, v8, cs, cq, ck, cv, S(stream));
}

int xtb_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg, uint8_t *out, float sinv, float vo,
                  void *stream)
{
    Attn a;
    if (nimg <= 0 || make_attn(&a, q8, k8, v8, nimg)) return -1;
    return launch_attention(a, nimg, out, sinv, vo, S(stream));
}

int xtb_px_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nseq, int L, uint8_t *out,
                     float sinv, float vo, void *stream)
{
    Attn a;
    if (nseq <= 0 || (L != PXLW && L != PXT) || make_attn_rows(&a, q8, k8, v8, nseq * L)) return -1;
    return launch_px_attention(a, nseq, L, out, sinv, vo, S(stream));
}

int xtb_px_fc1(const uint8_t *h, int rows, const uint8_t *w1, float wscale, float ascale, const float *b1,
               const float *rs, uint8_t *u8, void *stream)
{
    Operand A;
    Weight8 W;
    CUtensorMap um;
    if (!rows_ok(rows, "xtb_px_fc1") || !(wscale > 0.0f) || make_operand(&A, h, rows, D, 128) ||
        make_operand(&W.op, w1, PXHID, D, weight_box_rows(W_FC1)) || px_u8_map(&um, u8, rows))
        return -1;
    W.ws = nullptr;
    W.n = PXHID;
    W.k = D;
    W.uniform = wscale;
    return launch_px_fc1(A, W, ascale, rows, um, b1, rs, S(stream));
}

int xtb_oproj(const uint8_t *a, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(rows, "xtb_oproj") || make_operand(&A, a, rows, D, 128) || weight(&W, w, D, D, ws, W_O)) return -1;
    return launch_oproj(A, W, ascale, rows, (__half *)x, S(stream));
}

int xtb_fc1(const uint8_t *h, int rows, const uint8_t *w, const float *ws, float ascale, uint8_t *h8, float *stat,
            const float *rs, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(rows, "xtb_fc1") || make_operand(&A, h, rows, D, 128) || weight(&W, w, N12, D, ws, W_FC1)) return -1;
    return launch_fc1(A, W, ascale, rows, h8, (float2 *)stat, rs, S(stream));
}

size_t xtb_sf_image_bytes(int n, int k) { return n > 0 && k > 0 ? sf_image_bytes(n, k) : 0; }

int xtb_sf_image(const float *ws, int n, int k, uint8_t *img)
{
    if (!ws || !img || n <= 0 || k <= 0) return -1;
    return sf_image(ws, n, k, img);
}

int xtb_gemm_mx_f32(const uint8_t *a, int m, int k, const uint8_t *w, int n, const uint8_t *sf, int pair, float ascale,
                    float *out, int ldo, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(m, "xtb_gemm_mx_f32") || !sf || n <= 0 || k <= 0 || (k & 15) || ldo < n ||
        pair < 0 || pair > 2 || make_operand(&A, a, m, k, 128) || make_operand(&W.op, w, n, k, pair ? 64 : 256))
        return -1;
    W.ws = nullptr;
    W.n = n;
    W.k = k;
    W.sf = sf;
    W.sf_nbp = (((n + 127) / 128) + 1) & ~1;
    W.sf_pair = pair != 0;
    W.sf_wide = pair == 2;
    if (W.sf_pair && sf_map(&W.sfmap, sf, n, k)) return -1;
    return launch_gemm_f32(A, W, ascale, out, ldo, S(stream));
}

int xtb_fc1_mx(const uint8_t *h, int rows, const uint8_t *w, const uint8_t *sf, float ascale, uint8_t *h8, float *stat,
               const float *rs, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(rows, "xtb_fc1_mx") || !sf || make_operand(&A, h, rows, D, 128) ||
        make_operand(&W.op, w, N12, D, 256))
        return -1;
    W.ws = nullptr;
    W.n = N12;
    W.k = D;
    W.sf = sf;
    W.sf_nbp = (((N12 + 127) / 128) + 1) & ~1;
    return launch_fc1(A, W, ascale, rows, h8, (float2 *)stat, rs, S(stream));
}

int xtb_fc2(const uint8_t *h8, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x, float *stat,
            const float *c, const float *d, void *stream)
{
    Operand A;
    Weight8 W;
    if (!rows_ok(rows, "xtb_fc2") || make_operand(&A, h8, rows, HIDP, 128) || weight(&W, w, D, HIDP, ws, W_FC2)) return -1;
    return launch_fc2(A, W, ascale, rows, (__half *)x, (float2 *)stat, c, d, S(stream));
}

int xtb_patch_embed(const uint16_t *in, int nimg, const uint16_t *pe, const float *pos, uint16_t *x, void *stream)
{
    Operand A, B;
    if (nimg <= 0 || make_operand(&A, in, nimg * NP, K0P * 2, 128) || make_operand(&B, pe, D, K0P * 2, 256)) return -1;
    return launch_patch_embed(A, B, nimg, pos, (__half *)x, S(stream));
}

int xtb_pool_ln(const uint16_t *x, int nimg, const float *g, const float *b, float *pool, uint16_t *pn, uint8_t *pn8,
                float qs, void *stream)
{
    if (nimg <= 0) return -1;
    return launch_pool_ln((const __half *)x, nimg, g, b, pool, (__half *)pn, pn8, qs, S(stream));
}

int xtb_head_f16(const uint16_t *hw, int nt, const uint16_t *pn, int nimg, const float *hb, float *out, void *stream)
{
    Operand A, B;
    if (nt <= 0 || nimg <= 0 || make_operand(&A, hw, nt, D * 2, 128) || make_operand(&B, pn, nimg, D * 2, 64)) return -1;
    return launch_head_f16(A, B, nimg, nt, hb, out, S(stream));
}

int xtb_head_e4m3(const uint8_t *hw8, int nt, const float *hws, const uint8_t *pn8, int nimg, float ascale,
                  const float *hb, float *out, void *stream)
{
    Weight8 W;
    Operand B;
    if (nt <= 0 || nimg <= 0) return -1;
    W.ws = hws;
    W.n = nt;
    W.k = D;
    if (make_operand(&W.op, hw8, nt, D, 128) || make_operand(&B, pn8, nimg, D, 64)) return -1;
    return launch_head_e4m3(W, B, ascale, nimg, nt, hb, out, S(stream));
}

int xtb_amax_f16(const uint16_t *x, int k, int rows, float *amax, void *stream)
{
    return launch_amax_f16((const __half *)x, k, rows, amax, S(stream));
}

int xtb_e4m3_encode(const float *x, uint8_t *y, size_t n, int via_f16, void *stream)
{
    if (n && (!x || !y)) return -1;
    if (n > ((size_t)1 << 40)) {
        fprintf(stderr, "eva: xtb_e4m3_encode: %zu elements is too many\n", n);
        return -1;
    }
    return launch_e4m3_encode(x, y, n, via_f16, S(stream));
}

// ---- 2:4-sparse weights ----
int xtb_sparse24_check(const uint8_t *w, int n, int k) { return sparse24_check(w, n, k); }

int xtb_sparse24_compress(const uint8_t *w, int n, int k, uint8_t *vals, uint8_t *meta)
{
    if (!vals || !meta) return -1;
    return sparse24_compress(w, n, k, vals, meta);
}

static int sp_weight(SparseW *w, const uint8_t *vals, const uint8_t *meta, int n, int k, const float *ws)
{
    return make_sparse_weight(w, vals, meta, n, k, ws);
}

int xtb_gemm_sp_e4m3_f32(const uint8_t *x, int m, int k, const uint8_t *vals, const uint8_t *meta, int n,
                         const float *wscale, float ascale, float *out, void *stream)
{
    Operand X;
    SparseW W;
    if (m <= 0 || n <= 0 || k <= 0 || (k & 15)) {
        fprintf(stderr, "eva: xtb_gemm_sp_e4m3_f32: bad shape m %d n %d k %d (k must be a multiple of 16)\n", m, n, k);
        return -1;
    }
    if (make_operand(&X, x, m, k, SP_BOX_ROWS) || sp_weight(&W, vals, meta, n, k, wscale)) return -1;
    return launch_gemm_sp_f32(X, W, ascale, out, n, S(stream));
}

int xtb_qkv_sp(const uint8_t *h, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint8_t *q8, uint8_t *k8, uint8_t *v8, const float *cs, float cq, float ck, float cv, void *stream)
{
    Operand A;
    SparseW W;
    if (!rows_ok(rows, "xtb_qkv_sp") || make_operand(&A, h, rows, D, SP_BOX_ROWS) || sp_weight(&W, vals, meta, 3 * D, D, ws))
        return -1;
    return launch_qkv_sp(A, W, ascale, rows, q8, k8, v8, cs, cq, ck, cv, S(stream));
}

int xtb_oproj_sp(const uint8_t *a, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
                 uint16_t *x, void *stream)
{
    Operand A;
    SparseW W;
    if (!rows_ok(rows, "xtb_oproj_sp") || make_operand(&A, a, rows, D, SP_BOX_ROWS) || sp_weight(&W, vals, meta, D, D, ws))
        return -1;
    return launch_oproj_sp(A, W, ascale, rows, (__half *)x, S(stream));
}

int xtb_fc1_sp(const uint8_t *h, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint8_t *h8, float *stat, const float *rs, void *stream)
{
    Operand A;
    SparseW W;
    if (!rows_ok(rows, "xtb_fc1_sp") || make_operand(&A, h, rows, D, SP_BOX_ROWS) || sp_weight(&W, vals, meta, N12, D, ws))
        return -1;
    return launch_fc1_sp(A, W, ascale, rows, h8, (float2 *)stat, rs, S(stream));
}

int xtb_fc2_sp(const uint8_t *h8, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint16_t *x, float *stat, const float *c, const float *d, void *stream)
{
    Operand A;
    SparseW W;
    if (!rows_ok(rows, "xtb_fc2_sp") || make_operand(&A, h8, rows, HIDP, SP_BOX_ROWS) ||
        sp_weight(&W, vals, meta, D, HIDP, ws))
        return -1;
    return launch_fc2_sp(A, W, ascale, rows, (__half *)x, (float2 *)stat, c, d, S(stream));
}

int xtb_selftest_wait(uint32_t timeout_us, int arrive, void *stream)
{
    if (timeout_us > 10000000u) return -1;  // at most 10 s
    return launch_selftest_wait(timeout_us, arrive, S(stream));
}

int xtb_copy_async(void *dst, const void *src, size_t bytes, void *stream)
{
    if (!dst || !src) return -1;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, S(stream)) == cudaSuccess ? 0 : -1;
}

uint32_t xtb_error_word(int device)
{
    uint32_t *p = error_word(device), v = 0;
    if (p && cudaMemcpy(&v, p, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 0xFFFFFFFFu;
    return v;
}

void xtb_error_clear(int device)
{
    uint32_t *p = error_word(device);
    if (p) cudaMemset(p, 0, 4);
}

}  // extern "C"

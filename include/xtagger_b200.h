/* xtagger_b200: B200-native (sm_100a) EVA02-Large tagger forward behind xTagger's engine C ABI.
 *
 * Two layers of entry points, all plain C (pointers and sizes, no torch types):
 *
 *  1. The engine (eva_*): a drop-in for the wd engine of HoloArchivists/xTagger, src/engine/eva.h. Same names,
 *     same argument meaning, same 0 / -1 / NULL error convention with an "eva: ..." line on stderr, same
 *     ownership rules. xtag.c, the router (procimg.h) and tag stealing (steal.h) call exactly these.
 *  2. Kernel-level entry points (xtb_*): one per hot-path kernel, device pointers in, enqueued on a caller
 *     stream, no allocation. The parity tests drive these; they have no counterpart in the reference, which
 *     launches its kernels only from inside eva.h.
 *
 * Input contract per model input (eva.h:15-16): fp16 [1024 patches][592], column c*196 + ky*14 + kx, BGR,
 * (x/127.5 - 1), columns 588..591 zero.
 */
#ifndef XTAGGER_B200_H
#define XTAGGER_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Constants the callers use (values kept from eva.h:38-69). */
#ifndef EVA_NB
#define EVA_NB 8                              /* model inputs per submit (eva.h:38-40) */
#endif
#define EVA_NBUF 8                            /* host output slots (eva.h:41) */
#define EVA_S 448
#define EVA_D 1024
#define EVA_T 1025
#define EVA_NP 1024
#define EVA_HIDP 2736
#define EVA_K0P 592
#define EVA_NL 24
#define EVA_NH 16
#define EVA_IN ((size_t)EVA_NP * EVA_K0P)     /* halves per model input (eva.h:57) */
#define EVA_HB_OFF 0xC1800000u                /* -16.0f: bias of an extra head row nothing has written (eva.h:69) */
#define EVA_MAXDEV 8

/* Engine handle. Caller-allocated like the reference's `eva` (eva.h:117-151); the fields below are the ones the
 * reference's callers read (nt: procimg.h:1689, hpn[buf]: procimg.h:1983) plus the batch size. Everything else
 * lives behind impl. */
typedef struct eva {
    uint32_t nt, ntp, nt0;                    /* tags: nt = nt0 of the file + extra rows (tag stealing) */
    uint32_t nb;                              /* model inputs per submit (EVA_NB, or eva_open_ex's nb) */
    float *hout[EVA_NBUF];                    /* per slot: scores [nb][nt] fp32, engine-owned */
    uint16_t *hpn[EVA_NBUF];                  /* per slot, with extra rows: head inputs [nb][1024] fp16 */
    void *impl;
} eva;

/* Replaces eva_open (eva.h:573-604). Validates the header of `weights` (eva02.bin v3 per-tensor E4M3, or the
 * block-scaled v4 this library adds) and returns at once; the CUDA bring-up (weights, buffers, CUDA graph) runs on
 * its own thread. `pool` (poolb bytes) is the caller's input pool, page-locked in place by the bring-up and still
 * caller-owned. `extra` head rows past the file's tags (written later with eva_head_put) also enable the per-batch
 * copy of the head inputs into hpn. 0, or -1 with a stderr line. */
int eva_open(eva *e, const char *weights, int device, void *pool, size_t poolb, uint32_t extra);

/* Multi-GPU variant (no counterpart in the reference, which drives one GPU): one engine replica per listed
 * device, each submit's inputs split into contiguous shards, one per device, scores gathered into one hout[buf].
 * nb = model inputs per submit over all devices (0 = EVA_NB). ndev = -1 with devices NULL: all visible devices. */
int eva_open_ex(eva *e, const char *weights, const int *devices, int ndev, uint32_t nb, void *pool, size_t poolb,
                uint32_t extra);

/* Replaces eva_ready (eva.h:607-617): join the bring-up once. 0 or -1. */
int eva_ready(eva *e);
/* Replaces eva_poll (eva.h:620-623): 1 once the bring-up has finished. */
int eva_poll(eva *e);
/* Replaces eva_submit (eva.h:627-641): n <= nb inputs (pointers, EVA_IN halves each; adjacent ones go in one
 * copy) into slot buf < EVA_NBUF. Async: H2D, forward graph, D2H into hout[buf] (+ hpn[buf]). Do not resubmit buf
 * before eva_wait(buf). */
int eva_submit(eva *e, uint32_t buf, uint16_t *const *in, uint32_t n);
/* Replaces eva_query (eva.h:662-665): 1 if slot buf is done (or failed). */
int eva_query(eva *e, uint32_t buf);
/* Replaces eva_wait (eva.h:667-680): blocking (sleeping) wait; engine-owned [n][nt] scores or NULL on error. */
const float *eva_wait(eva *e, uint32_t buf);
/* Replaces eva_head_put (eva.h:645-650): stream-ordered write of head row j (fp16 [1024] + bias); later submits
 * see it, w may be reused at once. With an FP8 head the row is quantised with its row block's scales. */
int eva_head_put(eva *e, uint32_t j, const uint16_t *w, float bias);
/* Replaces eva_head_get (eva.h:653-659): blocking read of the file's nt0 head rows (fp16) and biases. */
int eva_head_get(eva *e, uint16_t *w, float *bias);
/* Replaces eva_close (eva.h:704-745): join, sync, unregister the pool, free everything. Safe after a failed open. */
void eva_close(eva *e);

/* ---- engine extensions (no counterpart in the reference) ---- */
/* Run the forward graph on inputs already resident on the devices (uploaded by eva_upload), no host copies.
 * Used to time the device-resident throughput. */
int eva_forward_resident(eva *e);
/* Copy n inputs to the devices' input buffers (same sharding as eva_submit), synchronously. */
int eva_upload(eva *e, uint16_t *const *in, uint32_t n);
/* Scores of the last resident forward into out [n][nt] (synchronous). */
int eva_download(eva *e, float *out, uint32_t n);
/* The CUDA stream (cudaStream_t) the engine uses on its i-th device; NULL if out of range. */
void *eva_stream(eva *e, int i);
/* Device addresses of the i-th device's resident batch: the inputs [nb_i][EVA_IN] halves that eva_forward_resident
 * reads (a producer on that device, such as xtb_prep_crop ordered on eva_stream(e, i), may write them in place of
 * eva_upload) and the scores [nb_i][nt] floats it writes. nb_i is that device's share of nb. NULL if out of range. */
void *eva_input(eva *e, int i);
void *eva_output(eva *e, int i);
/* Number of kernel launches in one forward on one device. */
int eva_launches_per_forward(eva *e);
/* Projection kinds running on the 2:4-sparse tensor-core kernels (bit 0 QKV, 1 O, 2 W12, 3 W2): with XTB_SPARSE=1 in
 * the environment at open, the kinds whose weights are 2:4 along k in every layer (as prune24.py writes them);
 * otherwise 0 (the dense kernels are faster on the same weights). */
int eva_sparse_kinds(eva *e);
/* Projection kinds (bit 0 QKV, 1 O, 2 W12, 3 W2) running on the tensor core's own block scaling: block-scaled (v4)
 * weights whose block scales are all powers of two, in every layer: all four by default (XTB_MX=0 in the
 * environment at open keeps the promoting kernels; XTB_MX_KINDS, a hex mask, chooses the kinds). */
int eva_block_scale_kinds(eva *e);
/* One direct (non-graph) forward on device 0 with an event after every kernel; per-kernel-kind milliseconds into
 * ms[kinds] (names from eva_prof_name), returns the number of kinds or -1. Mirrors the reference's EVA_PROF
 * probe (eva.h:312-339). */
int eva_profile(eva *e, float *ms, int kinds);
const char *eva_prof_name(int kind);

/* ---- kernel-level entry points (device pointers, enqueued on `stream`) ----
 * None of them allocates device memory; the first call on a device looks up the library's static error word and
 * sets the kernels' shared-memory attributes, so it should come before any stream capture. */
/* D[m][n] fp32 = ascale * sum_kb wscale[n/128][kb] * sum_{k in kb} e4m3(A[m][k]) * e4m3(W[n][k]).
 * A: E4M3 [m][k], W: E4M3 [n][k], wscale: fp32 [ceil(n/128)][ceil(k/128)], k a multiple of 16. */
int xtb_gemm_e4m3_f32(const uint8_t *a, int m, int k, const uint8_t *w, int n, const float *wscale, float ascale,
                      float *out, void *stream);

/* LayerNorm over 1024 (eps 1e-6) * g + b, * qs, E4M3: x fp16 [rows][1024] -> y [rows][1024]. Replaces k_ln
 * (kern_common.cuh:147-186). */
int xtb_ln_e4m3(const uint16_t *x, const float *g, const float *b, uint8_t *y, int rows, float qs, void *stream);
/* QKV projection with its attention-layout epilogue; rows = images * 1025. q8 / k8 / v8 [img][16][1152][64]
 * (rows t >= 1025 must be zero). Replaces k_qkv (eva_kernels.cu:41-114). */
int xtb_qkv(const uint8_t *h, int rows, const uint8_t *w, const float *ws, float ascale, uint8_t *q8, uint8_t *k8,
            uint8_t *v8, const float *cs, float cq, float ck, float cv, void *stream);
/* FP8 attention: out E4M3 [img * 1025][1024] (head h at column 64 h). Replaces k_flash / flash8
 * (eva_kernels.cu:116-122, kern_common.cuh:403-543). */
int xtb_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg, uint8_t *out, float sinv, float vo,
                  void *stream);
/* x fp16 [rows][1024] += ascale * a . Wo^T (block-scaled). Replaces k_oproj (eva_kernels.cu:134-162). */
int xtb_oproj(const uint8_t *a, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x, void *stream);
/* fc1 + SwiGLU: h8 E4M3 [rows][2736], stat fp32 [43][rows][2] row-statistics partials. Replaces k_fc1
 * (eva_kernels.cu:211-279). */
int xtb_fc1(const uint8_t *h, int rows, const uint8_t *w, const float *ws, float ascale, uint8_t *h8, float *stat,
            const float *rs, void *stream);
/* fc2 with the MLP LayerNorm folded in: x += rstd (acc - mean c) + d. Replaces k_fc2 (eva_kernels.cu:286-334).
 * stat: fc1's partials [43][rows][2], only read: the GEMM's epilogue sums each row's partials itself. */
int xtb_fc2(const uint8_t *h8, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x, float *stat,
            const float *c, const float *d, void *stream);
/* Patch embedding (fp16 tcgen05 GEMM) + position rows: in [img][1024][592] fp16 -> x [img][1025][1024] fp16.
 * Replaces k_pe + k_embed (eva_kernels.cu:21-33, 126-130). */
int xtb_patch_embed(const uint16_t *in, int nimg, const uint16_t *pe, const float *pos, uint16_t *x, void *stream);
/* Mean pool over patch tokens + fc_norm -> pn fp16 [img][1024] (pn8 = E4M3(pn * qs) if not NULL). Replaces
 * k_pool + k_lnh (eva_kernels.cu:404-431, kern_common.cuh:188-192). */
int xtb_pool_ln(const uint16_t *x, int nimg, const float *g, const float *b, float *pool, uint16_t *pn, uint8_t *pn8,
                float qs, void *stream);
/* Tag head + sigmoid: out [img][nt]. fp16 head replaces k_headmv (kern_common.cuh:695-727); the E4M3
 * block-scaled head (hws [ceil(nt/128)][8]) has no counterpart in the reference. */
int xtb_head_f16(const uint16_t *hw, int nt, const uint16_t *pn, int nimg, const float *hb, float *out, void *stream);
int xtb_head_e4m3(const uint8_t *hw8, int nt, const float *hws, const uint8_t *pn8, int nimg, float ascale,
                  const float *hb, float *out, void *stream);

/* fc2 as xtb_fc2, allocating nothing: its scratch (per-row mean / rstd) lives in a static device array of the
 * library, sized for XTB_NOALLOC_MAX_ROWS rows. No counterpart in the reference. For callers that cannot let the
 * library allocate device memory (their own fixed memory arena, no cudaMalloc synchronisation on a latency-critical
 * path, no out-of-memory failure after start-up). `stat` (fc1's partials) is only read. Rows beyond the maximum are
 * rejected (-1). A bounded wait that runs out sets a bit of the device's error word (xtb_error_word). The first call
 * on a device sets up the array's address and should come before any stream capture. All calls on a device share
 * the array: calls that overlap on the GPU race and must be serialised by the caller. */
#define XTB_NOALLOC_MAX_ROWS (16 * 1025)
int xtb_fc2_noalloc(const uint8_t *h8, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x,
                    const float *stat, const float *c, const float *d, void *stream);

/* Calibration statistic (the reference's k_amax, kern_common.cuh:194-217): amax[c] = max(amax[c], max over rows of
 * |x[row][c]|) for an fp16 [rows][k] tensor (k a multiple of 8, 16-byte aligned); amax holds non-negative fp32 values
 * (start from zeros). Used by the calibration forward (xtagger_b200/calib.py). */
int xtb_amax_f16(const uint16_t *x, int k, int rows, float *amax, void *stream);

/* The E4M3 encoder of every epilogue, over an array: y[i] = E4M3(x[i]) (round to nearest even, finite values beyond
 * 448 saturate, NaN stays NaN), pairs packed as __nv_cvt_float2_to_fp8x2(..., __NV_SATFINITE, __NV_E4M3), the
 * reference's q2 (kern_common.cuh:96-100); with via_f16 the attention output's staging: y[i] = E4M3(fp16(x[i]))
 * (kern_common.cuh:527-541). x fp32, y bytes, device pointers. For the encoder's exhaustive parity tests. */
int xtb_e4m3_encode(const float *x, uint8_t *y, size_t n, int via_f16, void *stream);

/* ---- 2:4-sparse weights on the sparse tensor cores (tcgen05.mma.sp) ----
 * The reference prunes weights 2:4 offline (prune24.py:44-56: in every group of four consecutive k the two least
 * important bytes are zeroed) and runs them through its dense kernels. These entry points run such weights on the
 * sparse MMA instead, with the same results as the dense xtb_qkv / xtb_oproj / xtb_fc1 / xtb_fc2 on the same
 * weights (same epilogue arithmetic; only the order of the fp32 sums inside a 128-k block may differ).
 * Compressed form (host memory, from xtb_sparse24_compress): values [np][kp / 2] (the two kept bytes of every group
 * of four, in k order) and metadata [np][kp / 8] (per group the in-group indices i0 < i1 of the kept bytes as
 * i0 | i1 << 2, two groups per byte, low nibble first), np / kp = n / k rounded up to a multiple of 128. */
/* 1 if every group of four consecutive k of every row of w [n][k] holds at most two nonzero E4M3 codes. */
int xtb_sparse24_check(const uint8_t *w, int n, int k);
/* Compress a 2:4 weight (host pointers; vals np * kp / 2 bytes, meta np * kp / 8 bytes). 0, or -1 if not 2:4. */
int xtb_sparse24_compress(const uint8_t *w, int n, int k, uint8_t *vals, uint8_t *meta);
/* out[m][n] (fp32) = ascale * sum_k x[m][k] W[n][k] * wscale[n / 128][k / 128], W compressed (device pointers). */
int xtb_gemm_sp_e4m3_f32(const uint8_t *x, int m, int k, const uint8_t *vals, const uint8_t *meta, int n,
                         const float *wscale, float ascale, float *out, void *stream);
/* Block scales that are all powers of two run on the tensor core's own block scaling (tcgen05.mma
 * kind::mxf8f6f4.block_scale) instead of promoting every 128-deep K block through the epilogue. xtb_sf_image (host
 * memory in and out) turns block scales ws [ceil(n/128)][ceil(k/128)] into the scale-factor image that kernel reads
 * (xtb_sf_image_bytes(n, k) bytes); it returns -1 if some scale is not a power of two. xtb_fc1_mx is xtb_fc1 with
 * the weight's scale-factor image sf (device memory) in place of ws: the same results up to the fp32 summation
 * order. */
size_t xtb_sf_image_bytes(int n, int k);
int xtb_sf_image(const float *ws, int n, int k, uint8_t *img);
int xtb_fc1_mx(const uint8_t *h, int rows, const uint8_t *w, const uint8_t *sf, float ascale, uint8_t *h8, float *stat,
               const float *rs, void *stream);
/* out[m][n] (fp32, row stride ldo) = ascale * A W^T on the block-scaled MMA: A E4M3 [m][k], W E4M3 [n][k] with its
 * scale-factor image sf (xtb_sf_image); pair = 1 runs the CTA-pair kernel (256 x 128 tiles), pair = 2 the CTA pair
 * on 256 x 256 tiles (two weight blocks per tile), pair = 0 the single-CTA one (128 x 256). k a multiple of 16. */
int xtb_gemm_mx_f32(const uint8_t *a, int m, int k, const uint8_t *w, int n, const uint8_t *sf, int pair, float ascale,
                    float *out, int ldo, void *stream);
/* As xtb_qkv / xtb_oproj / xtb_fc1 / xtb_fc2 with the weight compressed (vals, meta) and its block scales ws. */
int xtb_qkv_sp(const uint8_t *h, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint8_t *q8, uint8_t *k8, uint8_t *v8, const float *cs, float cq, float ck, float cv, void *stream);
int xtb_oproj_sp(const uint8_t *a, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
                 uint16_t *x, void *stream);
int xtb_fc1_sp(const uint8_t *h, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint8_t *h8, float *stat, const float *rs, void *stream);
int xtb_fc2_sp(const uint8_t *h8, int rows, const uint8_t *vals, const uint8_t *meta, const float *ws, float ascale,
               uint16_t *x, float *stat, const float *c, const float *d, void *stream);

/* ---- GPU preprocessing (procimg.h's wd path: pi_ingest / pi_prep, done there on the host) ----
 * A decoded image on the device: h rows of w RGBA (or RGBX) pixels, `stride` bytes apart (a multiple of 4, at least
 * 4 w; 4-byte aligned). xtb_prep_ingest applies alpha over white in place when `alpha` (X = 255 either way) and
 * builds the 2x2 box pyramid into `scratch`; xtb_prep_crop then writes the model input (EVA_IN halves, device
 * pointer `out`) of the rect (x0, y0, cw, ch) of that image: resampled into a 448^2 white square with the
 * antialiased bicubic (or only normalised when its long side is 448), [-1, 1] fp16, BGR planes, the patch operand
 * layout. Outputs are bit-identical to the reference's arithmetic. scratch: xtb_prep_scratch_bytes(w, h) device
 * bytes, owned by the caller, for one image at a time. Stream-ordered, no allocation. */
size_t xtb_prep_scratch_bytes(int w, int h);
int xtb_prep_ingest(uint8_t *rgba, int w, int h, int stride, int alpha, void *scratch, void *stream);
int xtb_prep_crop(const uint8_t *rgba, int w, int h, int stride, int x0, int y0, int cw, int ch, void *scratch,
                  uint16_t *out, void *stream);
/* Kernels one call launches: xtb_prep_crop of that rect, or xtb_prep_ingest of a w x h image when cw <= 0; -1 on a
 * bad rect. */
int xtb_prep_kernels(int w, int h, int x0, int y0, int cw, int ch);

/* One stream-ordered copy of `bytes` between any two of host (pinned for asynchrony) and device memory, for hosts
 * with no CUDA binding of their own (e.g. scores of eva_output back to the host after a device-side batch). */
int xtb_copy_async(void *dst, const void *src, size_t bytes, void *stream);

/* Library error word of a device: bits set by kernels whose bounded waits ran out (0 = healthy). A static device
 * array of the library (no allocation). The engine copies it back with every batch; eva_wait returns NULL (with an
 * "eva:" line) for a batch after which it is set. Reading and clearing synchronise with the device. */
uint32_t xtb_error_word(int device);
void xtb_error_clear(int device);
/* Failure-path self-test on the current device: a kernel waits at most timeout_us (<= 10 s) on a barrier that is
 * (arrive != 0) or is not arrived on; a wait that runs out sets bit 16 of the error word and the kernel returns
 * normally. Nothing faults or hangs. */
int xtb_selftest_wait(uint32_t timeout_us, int arrive, void *stream);

/* ---- PixAI engine (px_*): a drop-in for src/engine/px.h (ViTDet-L tagger at 1008^2, 30877 tags) ----
 * Input per model input (px.h:9-10): fp16 [5184 window-major patches][592], RGB c * 196 + ky * 14 + kx, [-1, 1],
 * columns 588..591 zero. Weights: pixai.bin v3 (export_pixai.py with a calibration file: E4M3 with one scale per
 * tensor); header words 4 / 5 (zero in the reference's files) may give the number of blocks and the mask of global
 * blocks. Errors: 0 / -1 / NULL with a "px: ..." line on stderr, as the reference. */
#ifndef PX_NB
#define PX_NB 4                               /* model inputs per submit (px.h:19-21) */
#endif
#define PX_NBUF 4                             /* host output slots (px.h:27) */
#define PX_NL 32
#define PX_IN ((size_t)5184 * EVA_K0P)        /* halves per model input (px.h:33) */

/* Engine handle, caller-allocated like the reference's `px` (px.h:59-89); impl holds the rest. */
typedef struct px {
    uint32_t nt, ntp;                         /* tags (and rounded up to 8) */
    uint32_t nb;                              /* model inputs per submit */
    float *hout[PX_NBUF];                     /* per slot: scores [nb][nt] fp32, engine-owned */
    void *impl;
} px;

/* Replaces px_open (px.h:355-384): validate the header, start the bring-up on its own thread, return at once.
 * `pool` (poolb bytes): the caller's input pool, page-locked in place by the bring-up. */
int px_open(px *p, const char *weights, int device, void *pool, size_t poolb);
/* Same with nb inputs per submit (no counterpart in the reference, which fixes PX_NB). */
int px_open_ex(px *p, const char *weights, int device, uint32_t nb, void *pool, size_t poolb);
/* Same on ndev devices (no counterpart in the reference, which drives one GPU): one complete engine replica per
 * device (weights copied to each), nb inputs per submit split into contiguous shards (sizes differ by at most one,
 * at most 64 per device), each shard's forward on its own device and stream, the scores gathered into hout[buf] by
 * px_wait. px_stream / px_input / px_profile / px_launches_per_forward report the first device's replica. */
int px_open_multi(px *p, const char *weights, const int *devices, int ndev, uint32_t nb, void *pool, size_t poolb);
int px_ready(px *p);                          /* px.h:386-397: join the bring-up; 0 or -1 */
int px_poll(px *p);                           /* px.h:399-402: 1 once the bring-up has finished */
/* Replaces px_submit (px.h:405-418): n <= nb inputs (PX_IN halves each; adjacent ones in one copy) into slot
 * buf < PX_NBUF; async H2D, forward graph, D2H into hout[buf]. */
int px_submit(px *p, uint32_t buf, uint16_t *const *in, uint32_t n);
int px_query(px *p, uint32_t buf);            /* px.h:420-423 */
const float *px_wait(px *p, uint32_t buf);    /* px.h:425-428: scores [n][nt] or NULL */
void px_close(px *p);                         /* px.h:455-492 */
/* PixAI attention kernel alone: q8 / k8 / v8 [nseq][16][L][64] E4M3 (L = 576 or 5184) -> out [nseq L][1024] E4M3,
 * the flash8<L> arithmetic of kern_common.cuh:403-543 (px_kernels.cu:140-154). */
int xtb_px_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nseq, int L, uint8_t *out,
                     float sinv, float vo, void *stream);
/* PixAI fc1 GEMM alone: u8 [rows][4736] = E4M3(rs * gelu(ascale wscale h W1^T + b1)), h E4M3 [rows][1024], W1 E4M3
 * [4736][1024] with one scale per tensor (k_pfc1, px_kernels.cu:203-239). */
int xtb_px_fc1(const uint8_t *h, int rows, const uint8_t *w1, float wscale, float ascale, const float *b1,
               const float *rs, uint8_t *u8, void *stream);
/* extensions: resident forward (inputs uploaded with px_upload or written at px_input), scores / head vectors of
 * the last forward, the engine's stream, launches per forward, per-kind kernel times of one direct forward */
int px_forward_resident(px *p);
int px_upload(px *p, uint16_t *const *in, uint32_t n);
int px_download(px *p, float *out, uint32_t n);
int px_head_input(px *p, uint16_t *o, uint32_t n);
void *px_stream(px *p);
void *px_input(px *p);
int px_launches_per_forward(px *p);
int px_profile(px *p, float *ms, int kinds);
const char *px_prof_name(int k);

#ifdef __cplusplus
}
#endif
#endif

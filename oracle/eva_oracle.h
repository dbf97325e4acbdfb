/* CPU oracle of the EVA02-L tagger forward — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C (C11 + OpenMP) restatement of the reference's algorithm for the hot path (HoloArchivists/xTagger,
 * src/engine/eva.h + eva_kernels.cu + kern_common.cuh), used as the checker by tests/, by
 * __graft_entry__.smoke() and as bench.py's CPU baseline. Nothing in the shipped library links or calls it.
 * Each function cites the reference lines it restates. Parity pins: see tests/test_oracle_pins.py.
 */
#ifndef EVA_ORACLE_H
#define EVA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#define OR_D 1024
#define OR_T 1025
#define OR_NP 1024
#define OR_HID 2730
#define OR_HIDP 2736
#define OR_K0P 592
#define OR_NH 16
#define OR_HD 64
#define OR_TP 1152
#define OR_N12 (2 * OR_HIDP)

/* numeric formats */
uint8_t or_e4m3(float x);                     /* OCP E4M3: round to nearest even, saturate to +-448, NaN -> 0x7F */
float or_e4m3_dec(uint8_t b);
void or_e4m3_n(const float *x, uint8_t *y, size_t n);
void or_e4m3_dec_n(const uint8_t *x, float *y, size_t n);
uint16_t or_f2h(float x);                     /* IEEE binary16, round to nearest even */
float or_h2f(uint16_t h);
void or_f2h_n(const float *x, uint16_t *y, size_t n);
void or_h2f_n(const uint16_t *x, float *y, size_t n);

/* out[m][n] = ascale * sum_kb ws[n/128][kb] * sum_{k in kb} e4m3(a[m][k]) e4m3(w[n][k]) */
void or_gemm_e4m3(const uint8_t *a, int m, int k, const uint8_t *w, int n, const float *ws, float ascale, float *out);
/* out[m][n] = sum_k h(a[m][k]) h(w[n][k]) (fp16 operands, fp32 result) */
void or_gemm_f16(const uint16_t *a, int m, int k, const uint16_t *w, int n, float *out);

/* forward pieces */
void or_ln_e4m3(const uint16_t *x, const float *g, const float *b, int rows, float qs, uint8_t *y);
void or_qkv_epilogue(const float *acc, int rows, const float *cs, float cq, float ck, float cv, uint8_t *q8,
                     uint8_t *k8, uint8_t *v8);
/* key_tile keys per tile and decisions per slice of slice_rows query rows: 64 and 16 are the reference's */
void or_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg, float sinv, float vo,
                  int key_tile, int slice_rows, uint8_t *out);
void or_resid_add(uint16_t *x, const float *acc, int rows);
void or_fc1_epilogue(const float *acc, int rows, const float *rs, uint8_t *h8, double *rowsum, double *rowsq);
void or_fc2_epilogue(uint16_t *x, const float *acc, int rows, const double *rowsum, const double *rowsq,
                     const float *c, const float *d);
void or_patch_embed(const uint16_t *in, int nimg, const uint16_t *pe, const float *pos, uint16_t *x);
void or_pool_ln(const uint16_t *x, int nimg, const float *g, const float *b, float *pool, uint16_t *pn, uint8_t *pn8,
                float qs);
void or_head_f16(const uint16_t *pn, int nimg, const uint16_t *hw, const float *hb, int nt, float *out);
void or_head_e4m3(const uint8_t *pn8, int nimg, const uint8_t *hw8, const float *hws, float ascale, const float *hb,
                  int nt, float *out);

/* whole forward from a model file (eva02.bin v3 or the block-scaled v4); in: nimg x [1024][592] fp16.
 * scores [nimg][nt]; pn (optional) [nimg][1024] fp16. key_tile / slice_rows: the attention's key tiling and
 * decision slices (64 / 16: the reference's). Returns 0, or -1 with a message on stderr. */
int or_forward(const char *model, const uint16_t *in, int nimg, int key_tile, int slice_rows, float *scores,
               uint16_t *pn);
/* number of tags of a model file (-1 on error) */
int or_model_nt(const char *model);

/* 2:4 selection of prune24.py (magnitude or Wanda score): zero the 2 least important of every 4 consecutive k */
void or_prune24(uint8_t *w, int n, int k, int wanda);

int or_threads(void);
int or_set_threads(int n);                    /* threads of later parallel regions (OMP_NUM_THREADS overridden) */

/* PixAI tagger (px_oracle.c; src/engine/px.h + px_kernels.cu): window-major tokens, sequences of L tokens */
void or_px_embed(const uint16_t *in, int rows, const uint16_t *pe, const float *pos, const float *w, const float *b,
                 uint16_t *x);
void or_px_qkv_epilogue(const float *acc, int rows, int L, const float *bias, const float *cs, float cq, float ck,
                        float cv, uint8_t *q8, uint8_t *k8, uint8_t *v8);
void or_px_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nseq, int L, float sinv, float vo,
                     int key_tile, int slice_rows, uint8_t *out);
void or_px_resid_bias(uint16_t *x, const float *acc, const float *bias, int rows);
void or_px_fc1_epilogue(const float *acc, int rows, const float *b1, const float *rs, uint8_t *u8);
void or_px_head(const uint16_t *x, int nimg, const float *w, const float *b, const float *U, const uint16_t *hpos,
                const uint16_t *wv, const uint16_t *hw, const float *hb, int nt, float *scores, uint16_t *o_out);
/* whole forward from a pixai.bin v3; in: nimg x [5184][592] fp16; scores [nimg][nt]; o_out (optional) the head's
 * pooled-and-projected vectors [nimg][1024] fp16 */
int or_px_forward(const char *model, const uint16_t *in, int nimg, int key_tile, int slice_rows, float *scores,
                  uint16_t *o_out);
int or_px_model_nt(const char *model);

/* GPU preprocessing restated (prep_oracle.c; src/core/procimg.h's wd path) */
uint32_t or_div255(uint32_t x);
void or_over_white(uint8_t *img, int w, int h, int stride, int alpha);
void or_half(const uint8_t *s, int sw, int sh, int sstride, uint8_t *d, int dstride);
void or_prep(uint8_t *img, int w, int h, int stride, int alpha, int x0, int y0, int cw, int ch, uint16_t *out);
int or_prep_level(int w, int h, int side);
#endif

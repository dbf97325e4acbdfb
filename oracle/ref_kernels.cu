// Launch harness for the reference's own GPU kernels (eva_kernels.cu, which includes kern_common.cuh), compiled from
// the reference's sources where they lie with the reference's own flags (oracle/Makefile, target `ref`, output
// oracle/_ref/libref_kernels.so, git-ignored).
// TEST AND BASELINE INFRASTRUCTURE ONLY: tests/ load it to pin the oracle (and this library's kernels) to the
// reference's code on the same inputs, and oracle/ref_time.py times the reference's forward on the same GPU. Nothing in
// the product loads it.
//
//   ref_attention: the reference's flash8<1025> (k_flash) on q / k / v given in this library's layouts. The
//     reference's k_qkv permutes the 64 dims of q and k identically, which leaves every dot product unchanged, so the
//     harness keeps them in order; v becomes the reference's per-64-key-tile transpose vt8 (eva_kernels.cu:111).
//   ref_forward / ref_forward_time: the reference's whole FP8 forward (eva_forward, eva.h:252-307, the non-calibration
//     branch) for an eva02.bin v3 file, with the per-layer multipliers of eva_layout (eva.h:380-430) and the buffer
//     shapes of eva_up (rows padded to 16, keys padded to 1088, vt8, the fc1 statistics partials). The forward is
//     captured into a CUDA graph as the reference does; its fp16 head serves at most 8 images per launch
//     (k_headmv's shared staging), so larger batches launch it per 8 images.
#include "eva_kernels.cu"

#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <string>
#include <vector>

#define CK(x)                                                                                    \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "ref_kernels: %s: %s\n", #x, cudaGetErrorString(e_));                \
            return -1;                                                                           \
        }                                                                                        \
    } while (0)

namespace {

constexpr int NL = 24, NS = 12, NG = 4, NP = 1024;

struct Layer {
    const float *ln1w, *ln1b, *ln2w, *ln2b, *rs, *cn, *dn;
    const unsigned char *wqkv, *wo, *w12, *w2;
    float qs[NG], cq, ck, cv, sinv, vo, a0, a1, a12, a3;
};

struct Model {
    unsigned char *blob = nullptr;  // device copy of the weight blob
    unsigned nt = 0, ntp = 0;
    const __half *pe = nullptr, *hw = nullptr;
    const float *pos = nullptr, *cs = nullptr, *fnw = nullptr, *fnb = nullptr, *hb = nullptr;
    Layer L[NL];
};

size_t take(size_t *off, size_t bytes)
{
    const size_t o = (*off + 255) & ~(size_t)255;
    *off = o + bytes;
    return o;
}

// eva_open's header checks (eva.h:576-592) and eva_layout's walk (eva.h:380-430) for a v3 file.
int load(const char *path, Model *m)
{
    FILE *f = fopen(path, "rb");
    uint32_t hdr[4];
    if (!f || fread(hdr, 4, 4, f) != 4 || memcmp(hdr, "EVA2", 4) || hdr[1] != 3) {
        fprintf(stderr, "ref_kernels: %s is not an eva02.bin v3\n", path);
        if (f) fclose(f);
        return -1;
    }
    m->nt = hdr[2];
    m->ntp = (hdr[2] + 7) & ~7u;
    const size_t wbytes = hdr[3];
    std::vector<unsigned char> host(wbytes);
    if (fseek(f, 256, SEEK_SET) || fread(host.data(), 1, wbytes, f) != wbytes) {
        fprintf(stderr, "ref_kernels: short read of %s\n", path);
        fclose(f);
        return -1;
    }
    fclose(f);
    CK(cudaMalloc(&m->blob, wbytes));
    CK(cudaMemcpy(m->blob, host.data(), wbytes, cudaMemcpyHostToDevice));
    size_t off = 0;
    const float *scl = (const float *)(host.data() + take(&off, (size_t)NL * NS * 4));
    unsigned char *b = m->blob;
    m->pe = (const __half *)(b + take(&off, (size_t)D * K0P * 2));
    m->pos = (const float *)(b + take(&off, (size_t)T * D * 4));
    m->cs = (const float *)(b + take(&off, (size_t)NP * 32 * 2 * 4));
    for (int i = 0; i < NL; i++) {
        Layer &L = m->L[i];
        L.ln1w = (const float *)(b + take(&off, D * 4));
        L.ln1b = (const float *)(b + take(&off, D * 4));
        L.wqkv = b + take(&off, (size_t)3 * D * D);
        L.wo = b + take(&off, (size_t)D * D);
        L.ln2w = (const float *)(b + take(&off, D * 4));
        L.ln2b = (const float *)(b + take(&off, D * 4));
        L.w12 = b + take(&off, (size_t)2 * HIDP * D);
        L.rs = (const float *)(b + take(&off, HIDP * 4));
        L.w2 = b + take(&off, (size_t)D * HIDP);
        L.cn = (const float *)(b + take(&off, D * 4));
        L.dn = (const float *)(b + take(&off, D * 4));
        const float *s = scl + i * NS;
        for (int g = 0; g < NG; g++) L.qs[g] = 1.0f / s[NG + g];
        L.cq = 1.0f / s[8];
        L.ck = 1.0f / s[9];
        L.cv = 1.0f / s[10];
        L.sinv = s[8] * s[9];
        L.vo = L.qs[1] * s[10];
        L.a0 = s[0] * s[NG];
        L.a1 = s[1] * s[NG + 1];
        L.a12 = s[2] * s[NG + 2];
        L.a3 = s[3] * s[NG + 3];
    }
    m->fnw = (const float *)(b + take(&off, D * 4));
    m->fnb = (const float *)(b + take(&off, D * 4));
    m->hw = (const __half *)(b + take(&off, (size_t)m->ntp * D * 2));
    m->hb = (const float *)(b + take(&off, (size_t)m->ntp * 4));
    if (off != wbytes) {
        fprintf(stderr, "ref_kernels: weight layout mismatch (%zu vs %zu bytes)\n", off, wbytes);
        return -1;
    }
    return 0;
}

struct Bufs {
    int nb = 0;
    unsigned M = 0, rows = 0;
    __half *in = nullptr, *x = nullptr, *pn = nullptr;
    unsigned char *h = nullptr, *q8 = nullptr, *k8 = nullptr, *v8 = nullptr, *m8 = nullptr;
    float *stat = nullptr, *pool = nullptr, *out = nullptr;
};

int alloc(Bufs *B, const Model &m, int nb)
{
    B->nb = nb;
    B->rows = (unsigned)nb * T;
    B->M = (B->rows + 15) & ~15u;
    const size_t qk = (size_t)nb * 16 * TP * 64, vt = (size_t)nb * 16 * NKT * 4096;
    CK(cudaMalloc(&B->in, (size_t)nb * NP * K0P * 2));
    CK(cudaMalloc(&B->x, (size_t)B->M * D * 2));
    CK(cudaMalloc(&B->h, (size_t)B->M * D));
    CK(cudaMalloc(&B->q8, qk));
    CK(cudaMalloc(&B->k8, qk));
    CK(cudaMalloc(&B->v8, vt));
    CK(cudaMalloc(&B->m8, (size_t)B->M * HIDP));
    CK(cudaMalloc(&B->stat, (size_t)NCT * B->M * 2 * 4));
    CK(cudaMalloc(&B->pool, (size_t)nb * D * 4));
    CK(cudaMalloc(&B->pn, (size_t)nb * D * 2));
    CK(cudaMalloc(&B->out, (size_t)nb * m.nt * 4));
    CK(cudaMemset(B->x, 0, (size_t)B->M * D * 2));
    CK(cudaMemset(B->h, 0, (size_t)B->M * D));
    CK(cudaMemset(B->q8, 0, qk));  // padded key rows stay zero, as eva_up arranges
    CK(cudaMemset(B->k8, 0, qk));
    CK(cudaMemset(B->v8, 0, vt));
    CK(cudaMemset(B->m8, 0, (size_t)B->M * HIDP));
    return 0;
}

void release(Bufs *B, Model *m)
{
    void *p[] = {B->in, B->x, B->h, B->q8, B->k8, B->v8, B->m8, B->stat, B->pool, B->pn, B->out, m->blob};
    for (void *q : p)
        if (q) cudaFree(q);
}

// eva_forward (eva.h:252-307), FP8 branch, on stream st.
int forward(const Model &m, Bufs &B, cudaStream_t st)
{
    const unsigned prows = (unsigned)B.nb * NP, lnb = B.M >> 3;
    k_pe<<<dim3(D / 128, prows / 128), 128, 0, st>>>(B.in, m.pe, B.x, prows);
    k_embed<<<B.nb * T, 256, 0, st>>>(B.x, m.pos);
    for (int i = 0; i < NL; i++) {
        const Layer &L = m.L[i];
        k_ln<<<lnb, 256, 0, st>>>(B.x, L.ln1w, L.ln1b, B.h, B.M, L.qs[0]);
        k_qkv<<<dim3(3 * D / 128, (B.rows + 127) / 128), 128, 0, st>>>(B.h, L.wqkv, B.q8, B.k8, B.v8, m.cs, L.a0, L.cq,
                                                                        L.ck, L.cv, B.rows);
        k_flash<<<dim3(NKT, 16, B.nb), 128, 0, st>>>(B.q8, B.k8, B.v8, B.h, L.sinv, L.vo);
        k_oproj<<<dim3(D / 128, (B.rows + 127) / 128), 128, 0, st>>>(B.h, L.wo, B.x, L.a1, B.rows);
        k_ln<<<lnb, 256, 0, st>>>(B.x, L.ln2w, L.ln2b, B.h, B.M, L.qs[2]);
        k_fc1<<<dim3((B.M + 127) / 128, NCT), 128, 0, st>>>(B.h, L.w12, B.m8, B.stat, L.rs, L.a12, B.M);
        k_fc2<<<dim3(D / 128, (B.M + 127) / 128), 128, 0, st>>>(B.m8, L.w2, B.x, B.stat, L.cn, L.dn, L.a3, B.M);
    }
    k_pool<<<dim3(B.nb, 16), 256, 0, st>>>(B.x, B.pool);
    k_lnh<<<(B.nb + 7) >> 3, 256, 0, st>>>(B.pool, m.fnw, m.fnb, B.pn, (unsigned)B.nb);
    for (int c = 0; c < B.nb; c += 8) {
        const unsigned n = B.nb - c < 8 ? (unsigned)(B.nb - c) : 8u;
        k_headmv<<<(m.nt + 63) / 64, 256, 0, st>>>(B.pn + (size_t)c * D, m.hw, m.hb, B.out + (size_t)c * m.nt, m.nt, n);
    }
    CK(cudaGetLastError());
    return 0;
}

int forward_graph(const Model &m, Bufs &B, cudaStream_t st, cudaGraphExec_t *ge)
{
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    if (forward(m, B, st)) {
        cudaStreamEndCapture(st, &g);
        return -1;
    }
    CK(cudaStreamEndCapture(st, &g));
    CK(cudaGraphInstantiate(ge, g, 0));
    CK(cudaGraphDestroy(g));
    return 0;
}

}  // namespace

// q8 / k8 / v8: host, this library's layout [nimg][16][tp_in][64] (rows >= 1025 ignored); out: host [nimg][1025][1024].
extern "C" int ref_attention(const uint8_t *q8, const uint8_t *k8, const uint8_t *v8, int nimg, int tp_in, float sinv,
                             float vo, uint8_t *out)
{
    const size_t heads = (size_t)nimg * 16;
    std::vector<uint8_t> q(heads * TP * 64, 0), k(heads * TP * 64, 0), vt(heads * NKT * 4096, 0);
    for (size_t bh = 0; bh < heads; bh++)
        for (int t = 0; t < T; t++) {
            memcpy(&q[(bh * TP + t) * 64], q8 + (bh * tp_in + t) * 64, 64);
            memcpy(&k[(bh * TP + t) * 64], k8 + (bh * tp_in + t) * 64, 64);
            for (int d = 0; d < 64; d++) vt[(bh * NKT + (t >> 6)) * 4096 + d * 64 + (t & 63)] = v8[(bh * tp_in + t) * 64 + d];
        }
    uint8_t *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
    const size_t out_bytes = (size_t)nimg * T * D;
    CK(cudaMalloc(&dq, q.size()));
    CK(cudaMalloc(&dk, k.size()));
    CK(cudaMalloc(&dv, vt.size()));
    CK(cudaMalloc(&dout, out_bytes));
    CK(cudaMemcpy(dq, q.data(), q.size(), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dk, k.data(), k.size(), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dv, vt.data(), vt.size(), cudaMemcpyHostToDevice));
    CK(cudaMemset(dout, 0, out_bytes));
    k_flash<<<dim3(NKT, 16, nimg), 128>>>(dq, dk, dv, dout, sinv, vo);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(out, dout, out_bytes, cudaMemcpyDeviceToHost));
    CK(cudaFree(dq));
    CK(cudaFree(dk));
    CK(cudaFree(dv));
    CK(cudaFree(dout));
    return 0;
}

// Scores [nimg][nt] of the reference's forward for the v3 model at path on the patch operands in (host fp16
// [nimg][1024][592]).
extern "C" int ref_forward(const char *path, const uint16_t *in, int nimg, float *scores)
{
    Model m;
    Bufs B;
    int rc = -1;
    cudaStream_t st = nullptr;
    cudaGraphExec_t ge = nullptr;
    if (nimg > 0 && !load(path, &m) && !alloc(&B, m, nimg) && cudaStreamCreate(&st) == cudaSuccess &&
        cudaMemcpy(B.in, in, (size_t)nimg * NP * K0P * 2, cudaMemcpyHostToDevice) == cudaSuccess &&
        !forward_graph(m, B, st, &ge) && cudaGraphLaunch(ge, st) == cudaSuccess &&
        cudaStreamSynchronize(st) == cudaSuccess &&
        cudaMemcpy(scores, B.out, (size_t)nimg * m.nt * 4, cudaMemcpyDeviceToHost) == cudaSuccess)
        rc = 0;
    if (rc) fprintf(stderr, "ref_kernels: ref_forward failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    if (ge) cudaGraphExecDestroy(ge);
    if (st) cudaStreamDestroy(st);
    release(&B, &m);
    return rc;
}

// Device time of the reference's forward graph for nimg inputs already on the device (CUDA events on the
// launching stream around iters graph launches after warmup launches): *ms = milliseconds per forward.
extern "C" int ref_forward_time(const char *path, const uint16_t *in, int nimg, int warmup, int iters, float *ms)
{
    Model m;
    Bufs B;
    int rc = -1;
    cudaStream_t st = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (nimg > 0 && iters > 0 && !load(path, &m) && !alloc(&B, m, nimg) && cudaStreamCreate(&st) == cudaSuccess &&
        cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess &&
        cudaMemcpy(B.in, in, (size_t)nimg * NP * K0P * 2, cudaMemcpyHostToDevice) == cudaSuccess &&
        !forward_graph(m, B, st, &ge)) {
        bool ok = true;
        for (int i = 0; i < warmup && ok; i++) ok = cudaGraphLaunch(ge, st) == cudaSuccess;
        ok = ok && cudaEventRecord(e0, st) == cudaSuccess;
        for (int i = 0; i < iters && ok; i++) ok = cudaGraphLaunch(ge, st) == cudaSuccess;
        ok = ok && cudaEventRecord(e1, st) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess;
        float t = 0.f;
        if (ok && cudaEventElapsedTime(&t, e0, e1) == cudaSuccess) {
            *ms = t / iters;
            rc = 0;
        }
    }
    if (rc) fprintf(stderr, "ref_kernels: ref_forward_time failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (st) cudaStreamDestroy(st);
    release(&B, &m);
    return rc;
}

// ---------------------------------------------------------------------------------------------------------------
// Per-kernel entry points (host buffers in this library's layouts; per-tensor multipliers as in v3): the reference's
// k_ln, k_qkv, k_oproj and k_fc1 + k_fc2, each launched with the grid eva_forward gives it (rows padded to 16 where
// the reference pads them).
// ---------------------------------------------------------------------------------------------------------------
namespace {
template <class E>
struct Dev {
    E *p = nullptr;
    ~Dev()
    {
        if (p) cudaFree(p);
    }
};
unsigned pad16(unsigned rows) { return (rows + 15) & ~15u; }

// logical dim of the byte at position s of a q / k row written by k_qkv (eva_kernels.cu:77-79: the dim pair
// (8 a + 2 c, + 1) lands at 16 (a >> 1) + 4 c + 2 (a & 1))
int qk_dim(int s) { return 8 * (2 * (s >> 4) + ((s & 3) >> 1)) + 2 * ((s & 15) >> 2) + (s & 1); }
}  // namespace

// y = E4M3(LN(x) * qs) for rows rows of 1024 fp16 values.
extern "C" int ref_ln(const uint16_t *x, const float *g, const float *b, int rows, float qs, uint8_t *y)
{
    const unsigned M = pad16(rows);
    Dev<__half> dx;
    Dev<unsigned char> dy;
    Dev<float> dg, db;
    CK(cudaMalloc(&dx.p, (size_t)M * D * 2));
    CK(cudaMalloc(&dy.p, (size_t)M * D));
    CK(cudaMalloc(&dg.p, D * 4));
    CK(cudaMalloc(&db.p, D * 4));
    CK(cudaMemset(dx.p, 0, (size_t)M * D * 2));
    CK(cudaMemcpy(dx.p, x, (size_t)rows * D * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dg.p, g, D * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(db.p, b, D * 4, cudaMemcpyHostToDevice));
    k_ln<<<M >> 3, 256>>>(dx.p, dg.p, db.p, dy.p, M, qs);
    CK(cudaGetLastError());
    CK(cudaMemcpy(y, dy.p, (size_t)rows * D, cudaMemcpyDeviceToHost));
    return 0;
}

// q8 / k8 / v8 (this library's layout [nimg][16][tp_out][64], rows >= 1025 left as given) from h (E4M3 [rows][1024],
// rows = nimg * 1025) and w (E4M3 [3072][1024]); alpha = weight x activation dequantisation.
extern "C" int ref_qkv(const uint8_t *h, int rows, const uint8_t *w, const float *cs, float alpha, float cq, float ck,
                       float cv, uint8_t *q8, uint8_t *k8, uint8_t *v8, int tp_out)
{
    if (rows % T) return -1;
    const int nimg = rows / T;
    const size_t qk = (size_t)nimg * 16 * TP * 64, vt = (size_t)nimg * 16 * NKT * 4096;
    Dev<unsigned char> dh, dw, dq, dk, dv;
    Dev<float> dcs;
    CK(cudaMalloc(&dh.p, (size_t)rows * D));
    CK(cudaMalloc(&dw.p, (size_t)3 * D * D));
    CK(cudaMalloc(&dq.p, qk));
    CK(cudaMalloc(&dk.p, qk));
    CK(cudaMalloc(&dv.p, vt));
    CK(cudaMalloc(&dcs.p, (size_t)NP * 64 * 4));
    CK(cudaMemcpy(dh.p, h, (size_t)rows * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dw.p, w, (size_t)3 * D * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dcs.p, cs, (size_t)NP * 64 * 4, cudaMemcpyHostToDevice));
    CK(cudaMemset(dq.p, 0, qk));
    CK(cudaMemset(dk.p, 0, qk));
    CK(cudaMemset(dv.p, 0, vt));
    k_qkv<<<dim3(3 * D / 128, (rows + 127) / 128), 128>>>(dh.p, dw.p, dq.p, dk.p, dv.p, dcs.p, alpha, cq, ck, cv,
                                                          (unsigned)rows);
    CK(cudaGetLastError());
    std::vector<unsigned char> q(qk), k(qk), v(vt);
    CK(cudaMemcpy(q.data(), dq.p, qk, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(k.data(), dk.p, qk, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(v.data(), dv.p, vt, cudaMemcpyDeviceToHost));
    for (size_t bh = 0; bh < (size_t)nimg * 16; bh++)
        for (int t = 0; t < T; t++)
            for (int s = 0; s < 64; s++) {
                q8[(bh * tp_out + t) * 64 + qk_dim(s)] = q[(bh * TP + t) * 64 + s];
                k8[(bh * tp_out + t) * 64 + qk_dim(s)] = k[(bh * TP + t) * 64 + s];
                v8[(bh * tp_out + t) * 64 + s] = v[(bh * NKT + (t >> 6)) * 4096 + s * 64 + (t & 63)];
            }
    return 0;
}

// x (fp16 [rows][1024], in / out) += alpha * a w^T, a E4M3 [rows][1024], w E4M3 [1024][1024].
extern "C" int ref_oproj(const uint8_t *a, int rows, const uint8_t *w, float alpha, uint16_t *x)
{
    Dev<unsigned char> da, dw;
    Dev<__half> dx;
    CK(cudaMalloc(&da.p, (size_t)rows * D));
    CK(cudaMalloc(&dw.p, (size_t)D * D));
    CK(cudaMalloc(&dx.p, (size_t)rows * D * 2));
    CK(cudaMemcpy(da.p, a, (size_t)rows * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dw.p, w, (size_t)D * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dx.p, x, (size_t)rows * D * 2, cudaMemcpyHostToDevice));
    k_oproj<<<dim3(D / 128, (rows + 127) / 128), 128>>>(da.p, dw.p, dx.p, alpha, (unsigned)rows);
    CK(cudaGetLastError());
    CK(cudaMemcpy(x, dx.p, (size_t)rows * D * 2, cudaMemcpyDeviceToHost));
    return 0;
}

// The MLP: k_fc1 (h8 = E4M3(rs * SwiGLU(a12 * h W12^T)), per-tile row statistics) then k_fc2 (x += rstd * (a3 * h8
// W2^T - mean * cn) + dn). Outputs h8 [rows][2736], the row totals of the statistics (sum u, sum u^2, summed over the
// reference's 57 partials in double), and x (in / out).
extern "C" int ref_mlp(const uint8_t *h, int rows, const uint8_t *w12, const float *rs, float a12, const uint8_t *w2,
                       const float *cn, const float *dn, float a3, uint8_t *h8, double *rowsum, double *rowsq, uint16_t *x)
{
    const unsigned M = pad16(rows);
    Dev<unsigned char> dh, dw12, dw2, dh8;
    Dev<float> drs, dst, dcn, ddn;
    Dev<__half> dx;
    CK(cudaMalloc(&dh.p, (size_t)M * D));
    CK(cudaMalloc(&dw12.p, (size_t)2 * HIDP * D));
    CK(cudaMalloc(&dw2.p, (size_t)D * HIDP));
    CK(cudaMalloc(&dh8.p, (size_t)M * HIDP));
    CK(cudaMalloc(&drs.p, HIDP * 4));
    CK(cudaMalloc(&dst.p, (size_t)NCT * M * 2 * 4));
    CK(cudaMalloc(&dcn.p, D * 4));
    CK(cudaMalloc(&ddn.p, D * 4));
    CK(cudaMalloc(&dx.p, (size_t)M * D * 2));
    CK(cudaMemset(dh.p, 0, (size_t)M * D));
    CK(cudaMemset(dx.p, 0, (size_t)M * D * 2));
    CK(cudaMemcpy(dh.p, h, (size_t)rows * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dw12.p, w12, (size_t)2 * HIDP * D, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dw2.p, w2, (size_t)D * HIDP, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(drs.p, rs, HIDP * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dcn.p, cn, D * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ddn.p, dn, D * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dx.p, x, (size_t)rows * D * 2, cudaMemcpyHostToDevice));
    k_fc1<<<dim3((M + 127) / 128, NCT), 128>>>(dh.p, dw12.p, dh8.p, dst.p, drs.p, a12, M);
    CK(cudaGetLastError());
    k_fc2<<<dim3(D / 128, (M + 127) / 128), 128>>>(dh8.p, dw2.p, dx.p, dst.p, dcn.p, ddn.p, a3, M);
    CK(cudaGetLastError());
    std::vector<float> st((size_t)NCT * M * 2);
    CK(cudaMemcpy(h8, dh8.p, (size_t)rows * HIDP, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(st.data(), dst.p, st.size() * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(x, dx.p, (size_t)rows * D * 2, cudaMemcpyDeviceToHost));
    for (int r = 0; r < rows; r++) {
        double s = 0, q = 0;
        for (int c = 0; c < NCT; c++) {
            s += st[((size_t)c * M + r) * 2];
            q += st[((size_t)c * M + r) * 2 + 1];
        }
        rowsum[r] = s;
        rowsq[r] = q;
    }
    return 0;
}

// Launch harness for the reference's own PixAI GPU kernels (px_kernels.cu, which includes kern_common.cuh), compiled
// from the reference's sources where they lie with the reference's own flags (oracle/Makefile, target `ref`, output
// oracle/_ref/libref_px.so, git-ignored).
// TEST INFRASTRUCTURE ONLY: tests/ load it to pin the PixAI oracle (oracle/px_oracle.c) and this library's px_*
// engine to the reference's code on the same inputs. Nothing in the product loads it.
//
//   ref_px_forward: the reference's FP8 PixAI forward (px_forward, px.h:115-190, the non-calibration branch) for a
//     pixai.bin v3 file, with the per-block multipliers of px_layout (px.h:222-235) and the buffer shapes of px_up
//     (px.h:286-310). Two departures, both for reduced test models, neither touching a kernel: the number of blocks and
//     the global-block mask come from header words 4 / 5 when set (zero: 32 blocks, PX_GLOBAL's 7, 15, 23, 31), and
//     the batch is the caller's (even, so that the token rows stay a multiple of 128; the fp16 head serves 8 images
//     per launch, so larger batches launch it per 8 images).
#include "px_kernels.cu"

#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <vector>

#define CK(x)                                                                                    \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "ref_px: %s: %s\n", #x, cudaGetErrorString(e_));                     \
            return -1;                                                                           \
        }                                                                                        \
    } while (0)

namespace {

constexpr int PNS = 12, PNG = 4, PNCH = T / 144;

struct PLayer {
    const float *ln1w, *ln1b, *bqkv, *bo, *ln2w, *ln2b, *b1, *rs, *b2;
    const unsigned char *wqkv, *wo, *w1, *w2;
    float qs[PNG], cq, ck, cv, sinv, vo, a0, a1, a2, a3;
    bool glob;
};

struct PModel {
    unsigned char *blob = nullptr;
    unsigned nt = 0, ntp = 0;
    int nl = 32;
    uint32_t gmask = 0;
    const __half *pe = nullptr, *hpos = nullptr, *wv = nullptr, *hw = nullptr;
    const float *pos = nullptr, *lnpw = nullptr, *lnpb = nullptr, *csw = nullptr, *csg = nullptr;
    const float *hnw = nullptr, *hnb = nullptr, *U = nullptr, *hb = nullptr;
    std::vector<PLayer> L;
};

size_t take(size_t *off, size_t bytes)
{
    const size_t o = (*off + 255) & ~(size_t)255;
    *off = o + bytes;
    return o;
}

// px_open's header checks (px.h:359-368) and px_layout's walk (px.h:196-245) for a v3 file.
int load(const char *path, PModel *m)
{
    FILE *f = fopen(path, "rb");
    uint32_t hdr[6];
    if (!f || fread(hdr, 4, 6, f) != 6 || memcmp(hdr, "PXAI", 4) || hdr[1] != 3) {
        fprintf(stderr, "ref_px: %s is not a pixai.bin v3\n", path);
        if (f) fclose(f);
        return -1;
    }
    m->nt = hdr[2];
    m->ntp = (hdr[2] + 7) & ~7u;
    m->nl = hdr[4] ? (int)hdr[4] : 32;
    m->gmask = hdr[5];
    const size_t wbytes = hdr[3];
    std::vector<unsigned char> host(wbytes);
    if (fseek(f, 256, SEEK_SET) || fread(host.data(), 1, wbytes, f) != wbytes) {
        fprintf(stderr, "ref_px: short read of %s\n", path);
        fclose(f);
        return -1;
    }
    fclose(f);
    CK(cudaMalloc(&m->blob, wbytes));
    CK(cudaMemcpy(m->blob, host.data(), wbytes, cudaMemcpyHostToDevice));
    size_t off = 0;
    const float *tab = (const float *)(host.data() + take(&off, (size_t)m->nl * PNS * 4));
    unsigned char *b = m->blob;
    m->pe = (const __half *)(b + take(&off, (size_t)D * K0P * 2));
    m->pos = (const float *)(b + take(&off, (size_t)T * D * 4));
    m->lnpw = (const float *)(b + take(&off, D * 4));
    m->lnpb = (const float *)(b + take(&off, D * 4));
    m->csw = (const float *)(b + take(&off, (size_t)LW * 32 * 2 * 4));
    m->csg = (const float *)(b + take(&off, (size_t)T * 32 * 2 * 4));
    m->L.resize(m->nl);
    for (int i = 0; i < m->nl; i++) {
        PLayer &L = m->L[i];
        L.ln1w = (const float *)(b + take(&off, D * 4));
        L.ln1b = (const float *)(b + take(&off, D * 4));
        L.wqkv = b + take(&off, (size_t)3 * D * D);
        L.bqkv = (const float *)(b + take(&off, 3 * D * 4));
        L.wo = b + take(&off, (size_t)D * D);
        L.bo = (const float *)(b + take(&off, D * 4));
        L.ln2w = (const float *)(b + take(&off, D * 4));
        L.ln2b = (const float *)(b + take(&off, D * 4));
        L.w1 = b + take(&off, (size_t)HID * D);
        L.b1 = (const float *)(b + take(&off, HID * 4));
        L.rs = (const float *)(b + take(&off, HID * 4));
        L.w2 = b + take(&off, (size_t)D * HID);
        L.b2 = (const float *)(b + take(&off, D * 4));
        const float *t = tab + (size_t)i * PNS;
        for (int g = 0; g < PNG; g++) L.qs[g] = 1.0f / t[PNG + g];
        L.cq = 1.0f / t[8];
        L.ck = 1.0f / t[9];
        L.cv = 1.0f / t[10];
        L.sinv = t[8] * t[9];
        L.vo = L.qs[1] * t[10];
        L.a0 = t[0] * t[PNG];
        L.a1 = t[1] * t[PNG + 1];
        L.a2 = t[2] * t[PNG + 2];
        L.a3 = t[3] * t[PNG + 3];
        L.glob = m->gmask ? ((m->gmask >> i) & 1) != 0 : (i & 7) == 7;
    }
    m->hnw = (const float *)(b + take(&off, D * 4));
    m->hnb = (const float *)(b + take(&off, D * 4));
    m->U = (const float *)(b + take(&off, (size_t)16 * D * 4));
    m->hpos = (const __half *)(b + take(&off, (size_t)T * D * 2));
    m->wv = (const __half *)(b + take(&off, (size_t)D * D * 2));
    m->hw = (const __half *)(b + take(&off, (size_t)m->ntp * D * 2));
    m->hb = (const float *)(b + take(&off, (size_t)m->ntp * 4));
    if (off != wbytes) {
        fprintf(stderr, "ref_px: weight layout mismatch (%zu vs %zu bytes)\n", off, wbytes);
        return -1;
    }
    return 0;
}

struct PBufs {
    int nb = 0;
    unsigned rows = 0;
    __half *in = nullptr, *x = nullptr, *y = nullptr, *P = nullptr, *o = nullptr;
    unsigned char *h = nullptr, *q8 = nullptr, *k8 = nullptr, *v8 = nullptr, *u = nullptr;
    float *s = nullptr, *pooled = nullptr, *out = nullptr;
};

int alloc(PBufs *B, const PModel &m, int nb)
{
    B->nb = nb;
    B->rows = (unsigned)nb * T;
    const size_t M = B->rows;
    CK(cudaMalloc(&B->in, (size_t)nb * T * K0P * 2));
    CK(cudaMalloc(&B->x, M * D * 2));
    CK(cudaMalloc(&B->h, M * D * 2));
    CK(cudaMalloc(&B->y, M * D * 2));
    CK(cudaMalloc(&B->u, M * HID));
    CK(cudaMalloc(&B->q8, M * D));
    CK(cudaMalloc(&B->k8, M * D));
    CK(cudaMalloc(&B->v8, M * D));
    CK(cudaMalloc(&B->s, M * 16 * 4));
    CK(cudaMalloc(&B->P, (size_t)nb * 16 * T * 2));
    CK(cudaMalloc(&B->pooled, (size_t)nb * PNCH * 16 * D * 4));
    CK(cudaMalloc(&B->o, (size_t)nb * D * 2));
    CK(cudaMalloc(&B->out, (size_t)nb * m.nt * 4));
    return 0;
}

void release(PBufs *B, PModel *m)
{
    void *p[] = {B->in, B->x, B->h, B->y, B->u, B->q8, B->k8, B->v8, B->s, B->P, B->pooled, B->o, B->out, m->blob};
    for (void *q : p)
        if (q) cudaFree(q);
}

// px_forward (px.h:115-190), FP8 branch, on stream st.
int forward(const PModel &m, PBufs &B, cudaStream_t st)
{
    const unsigned rows = B.rows, lnb = rows >> 3, nch = PNCH;
    k_ppe<<<dim3(D / 128, rows / 128), 128, 0, st>>>(B.in, m.pe, B.x, rows);
    k_pembed<<<lnb, 256, 0, st>>>(B.x, m.pos, m.lnpw, m.lnpb, rows);
    for (int i = 0; i < m.nl; i++) {
        const PLayer &L = m.L[i];
        const float *cs = L.glob ? m.csg : m.csw;
        const unsigned L1 = L.glob ? T : LW;
        k_ln<<<lnb, 256, 0, st>>>(B.x, L.ln1w, L.ln1b, B.h, rows, L.qs[0]);
        k_pqkv<<<dim3(24, rows / 128), 128, 0, st>>>(B.h, L.wqkv, L.bqkv, B.q8, B.k8, B.v8, cs, L1, L.a0, L.cq, L.ck,
                                                      L.cv, rows);
        if (L.glob) k_pflash_g<<<dim3(T / 64, 16, B.nb), 128, 0, st>>>(B.q8, B.k8, B.v8, B.h, L.sinv, L.vo);
        else k_pflash_w<<<dim3(LW / 64, 16, B.nb * 9), 128, 0, st>>>(B.q8, B.k8, B.v8, B.h, L.sinv, L.vo);
        k_pproj<<<dim3(D / 128, rows / 128), 128, 0, st>>>(B.h, L.wo, B.x, L.bo, L.a1, rows);
        k_ln<<<lnb, 256, 0, st>>>(B.x, L.ln2w, L.ln2b, B.h, rows, L.qs[2]);
        k_pfc1<<<dim3(HID / 128, rows / 128), 128, 0, st>>>(B.h, L.w1, L.b1, L.rs, B.u, L.a2, rows);
        k_pfc2<<<dim3(D / 128, rows / 128), 128, 0, st>>>(B.u, L.w2, B.x, L.b2, L.a3, rows);
    }
    k_phln<<<lnb, 256, 0, st>>>(B.x, m.hnw, m.hnb, m.hpos, B.y, rows);
    k_phscore<<<lnb, 256, 0, st>>>(B.y, m.U, B.s, rows);
    k_phsoft<<<B.nb * 16, 256, 0, st>>>(B.s, B.P);
    k_phpool<<<dim3(B.nb, PNCH), 512, 0, st>>>(B.P, B.y, B.pooled);
    k_phv<<<B.nb * 16, 256, 0, st>>>(B.pooled, m.wv, B.o, nch);
    for (int c = 0; c < B.nb; c += 8) {
        const unsigned n = B.nb - c < 8 ? (unsigned)(B.nb - c) : 8u;
        k_headmv<<<(m.nt + 63) / 64, 256, 0, st>>>(B.o + (size_t)c * D, m.hw, m.hb, B.out + (size_t)c * m.nt, m.nt, n);
    }
    CK(cudaGetLastError());
    return 0;
}

}  // namespace

// Scores [nimg][nt] (and, when o_out is not null, the head's o [nimg][1024] fp16) of the reference's PixAI forward for
// the v3 model at path on the patch operands in (host fp16 [nimg][5184][592]); nimg even.
extern "C" int ref_px_forward(const char *path, const uint16_t *in, int nimg, float *scores, uint16_t *o_out)
{
    PModel m;
    PBufs B;
    int rc = -1;
    cudaStream_t st = nullptr;
    if (nimg > 0 && (nimg & 1) == 0 && !load(path, &m) && !alloc(&B, m, nimg) &&
        cudaStreamCreate(&st) == cudaSuccess &&
        cudaMemcpy(B.in, in, (size_t)nimg * T * K0P * 2, cudaMemcpyHostToDevice) == cudaSuccess &&
        !forward(m, B, st) && cudaStreamSynchronize(st) == cudaSuccess &&
        cudaMemcpy(scores, B.out, (size_t)nimg * m.nt * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
        (!o_out || cudaMemcpy(o_out, B.o, (size_t)nimg * D * 2, cudaMemcpyDeviceToHost) == cudaSuccess))
        rc = 0;
    if (rc) fprintf(stderr, "ref_px: ref_px_forward failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    if (st) cudaStreamDestroy(st);
    release(&B, &m);
    return rc;
}

// Device time of the reference's PixAI forward for nimg inputs already on the device: the forward captured into a
// CUDA graph as px_up does (px.h:331-336), CUDA events around iters graph launches after warmup launches; *ms =
// milliseconds per forward.
extern "C" int ref_px_forward_time(const char *path, const uint16_t *in, int nimg, int warmup, int iters, float *ms)
{
    PModel m;
    PBufs B;
    int rc = -1;
    cudaStream_t st = nullptr;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (nimg > 0 && (nimg & 1) == 0 && iters > 0 && !load(path, &m) && !alloc(&B, m, nimg) &&
        cudaStreamCreate(&st) == cudaSuccess && cudaEventCreate(&e0) == cudaSuccess &&
        cudaEventCreate(&e1) == cudaSuccess &&
        cudaMemcpy(B.in, in, (size_t)nimg * T * K0P * 2, cudaMemcpyHostToDevice) == cudaSuccess &&
        cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        const int frc = forward(m, B, st);
        if (cudaStreamEndCapture(st, &g) == cudaSuccess && !frc && cudaGraphInstantiate(&ge, g, 0) == cudaSuccess) {
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
    }
    if (rc) fprintf(stderr, "ref_px: ref_px_forward_time failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (st) cudaStreamDestroy(st);
    release(&B, &m);
    return rc;
}

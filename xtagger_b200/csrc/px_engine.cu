// The px_* engine: a drop-in for the PixAI engine of xTagger (src/engine/px.h) on one B200.
//
// Bring-up (px_open -> boot thread): read pixai.bin v3 into pinned host memory, copy it to the device, resolve the
// tensor layout (px.h:196-245), allocate the activations for nb inputs, build the TMA descriptors and capture the
// whole forward (2 + 7 per block + 5 launches) into one CUDA graph. Per batch (px_submit): H2D of the inputs
// (adjacent pool inputs in one copy), graph launch, D2H of the scores, event; px_wait sleeps on the event and fails
// the batch when a kernel's bounded wait ran out (the library error word rides back with every batch).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include <cuda_fp16.h>

#include "../../include/xtagger_b200.h"
#include "host.h"
#include "ops.h"

using namespace xtb;

namespace {

constexpr int NG = 4;  // block GEMMs: QKV, O, fc1, fc2

struct PxLayer {
    const float *ln1w, *ln1b, *bqkv, *bo, *ln2w, *ln2b, *b1, *rs, *b2;
    Weight8 w[NG];
    float adq[NG], cq, ck, cv, sinv, vo;
    bool glob;
};

enum PxProf { Q_PATCH, Q_LN1, Q_QKV, Q_ATTW, Q_ATTG, Q_OPROJ, Q_LN2, Q_FC1, Q_FC2, Q_HEAD, Q_KINDS };
const char *const px_prof_names[Q_KINDS] = {"patch+embed", "ln1",  "qkv", "attention (window)", "attention (global)",
                                            "oproj",       "ln2",  "fc1", "fc2",                "pool+head"};

struct PxImpl {
    std::thread boot;
    bool boot_running = false, up = false;
    int bstatus = -1, dev = 0, nl = PX_NL, launches = 0;
    uint32_t gmask = 0;
    std::string path;
    size_t wbytes = 0;
    std::vector<float> table;
    void *ipool = nullptr;
    size_t ipoolb = 0;
    bool pool_reg = false, out_reg = false;
    cudaStream_t st = nullptr;
    uint8_t *wts = nullptr;
    const __half *pe = nullptr, *hpos = nullptr, *wv = nullptr, *hw = nullptr;
    const float *pos = nullptr, *lnpw = nullptr, *lnpb = nullptr, *csw = nullptr, *csg = nullptr;
    const float *hnw = nullptr, *hnb = nullptr, *U = nullptr, *hb = nullptr;
    std::vector<PxLayer> L;
    __half *in = nullptr, *x = nullptr, *y = nullptr, *P = nullptr, *o = nullptr;
    uint8_t *h8 = nullptr, *q8 = nullptr, *k8 = nullptr, *v8 = nullptr, *u8 = nullptr;
    float *s = nullptr, *part = nullptr, *out = nullptr;
    Operand op_in, op_pe, op_h8, op_u8, op_hw, op_o;
    CUtensorMap xm, um;
    Attn attn;
    cudaGraphExec_t graph = nullptr;
    cudaEvent_t done[PX_NBUF] = {};
    uint32_t *errh = nullptr;  // pinned, per slot: the device error word after the slot's forward
    // several devices (px_open_multi): one complete single-device engine per device, each with its contiguous shard
    // of every submit (shard i starts at input lo[i]); the scores are gathered into this handle's hout[buf]
    std::vector<px> subs;
    std::vector<uint32_t> lo;
    uint32_t slot_n[PX_NBUF] = {};
    bool multi() const { return !subs.empty(); }
};

// Inputs [lo, lo + nb) of a submit of n go to shard i: how many of them there are.
uint32_t shard_n(const PxImpl *im, size_t i, uint32_t n)
{
    const uint32_t lo = im->lo[i];
    return n > lo ? std::min(n - lo, im->subs[i].nb) : 0;
}

PxImpl *I(px *p) { return (PxImpl *)p->impl; }

#define ECK(call)                                                                                 \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) {                                                                  \
            fprintf(stderr, "px: %s: %s\n", #call, cudaGetErrorString(e_));                       \
            return -1;                                                                            \
        }                                                                                         \
    } while (0)
#define RCK(call)              \
    do {                       \
        if ((call)) return -1; \
    } while (0)

size_t take(size_t *off, size_t bytes)
{
    const size_t o = (*off + 255) & ~(size_t)255;
    *off = o + bytes;
    return o;
}

bool is_global(const PxImpl *im, int i) { return im->gmask ? ((im->gmask >> i) & 1) != 0 : (i & 7) == 7; }

// Tensor addresses in the device blob (px.h:196-245) and the per-block multipliers (px.h:224-235).
int layout(PxImpl *im, px *p)
{
    size_t off = 0;
    uint8_t *B = im->wts;
    take(&off, (size_t)im->nl * 12 * 4);
    im->pe = (const __half *)(B + take(&off, (size_t)D * K0P * 2));
    im->pos = (const float *)(B + take(&off, (size_t)PXT * D * 4));
    im->lnpw = (const float *)(B + take(&off, D * 4));
    im->lnpb = (const float *)(B + take(&off, D * 4));
    im->csw = (const float *)(B + take(&off, (size_t)PXLW * 64 * 4));
    im->csg = (const float *)(B + take(&off, (size_t)PXT * 64 * 4));
    const int kn[NG][2] = {{3 * D, D}, {D, D}, {PXHID, D}, {D, PXHID}};
    im->L.resize(im->nl);
    for (int i = 0; i < im->nl; i++) {
        PxLayer &L = im->L[i];
        const float *t = &im->table[(size_t)i * 12];
        const uint8_t *wp[NG];
        L.ln1w = (const float *)(B + take(&off, D * 4));
        L.ln1b = (const float *)(B + take(&off, D * 4));
        wp[0] = B + take(&off, (size_t)3 * D * D);
        L.bqkv = (const float *)(B + take(&off, 3 * D * 4));
        wp[1] = B + take(&off, (size_t)D * D);
        L.bo = (const float *)(B + take(&off, D * 4));
        L.ln2w = (const float *)(B + take(&off, D * 4));
        L.ln2b = (const float *)(B + take(&off, D * 4));
        wp[2] = B + take(&off, (size_t)PXHID * D);
        L.b1 = (const float *)(B + take(&off, PXHID * 4));
        L.rs = (const float *)(B + take(&off, PXHID * 4));
        wp[3] = B + take(&off, (size_t)D * PXHID);
        L.b2 = (const float *)(B + take(&off, D * 4));
        for (int g = 0; g < NG; g++) {
            if (!(t[g] > 0.0f) || !(t[4 + g] > 0.0f)) {
                fprintf(stderr, "px: block %d: scale table entries must be positive\n", i);
                return -1;
            }
            L.w[g].ws = nullptr;
            L.w[g].uniform = t[g];
            L.w[g].n = kn[g][0];
            L.w[g].k = kn[g][1];
            RCK(make_operand(&L.w[g].op, wp[g], kn[g][0], kn[g][1], weight_box_rows((WeightUse)g)));
            L.adq[g] = t[4 + g];
        }
        L.cq = 1.0f / t[8];
        L.ck = 1.0f / t[9];
        L.cv = 1.0f / t[10];
        L.sinv = t[8] * t[9];
        L.vo = (1.0f / t[5]) * t[10];
        L.glob = is_global(im, i);
    }
    im->hnw = (const float *)(B + take(&off, D * 4));
    im->hnb = (const float *)(B + take(&off, D * 4));
    im->U = (const float *)(B + take(&off, (size_t)NH * D * 4));
    im->hpos = (const __half *)(B + take(&off, (size_t)PXT * D * 2));
    im->wv = (const __half *)(B + take(&off, (size_t)D * D * 2));
    im->hw = (const __half *)(B + take(&off, (size_t)p->ntp * D * 2));
    im->hb = (const float *)(B + take(&off, (size_t)p->ntp * 4));
    if (off != im->wbytes) {
        fprintf(stderr, "px: weight layout mismatch (%zu vs %zu bytes)\n", off, im->wbytes);
        return -1;
    }
    return 0;
}

struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
};

int record(Prof *pr, cudaStream_t st, int kind)
{
    if (!pr) return 0;
    cudaEvent_t ev;
    ECK(cudaEventCreate(&ev));
    ECK(cudaEventRecord(ev, st));
    pr->ev.push_back(ev);
    pr->kind.push_back(kind);
    return 0;
}

// The forward of nb inputs (px.h:115-190).
int forward(PxImpl *im, px *p, Prof *pr)
{
    const int nb = (int)p->nb, rows = nb * PXT;
    cudaStream_t st = im->st;
    int n = 0;
    RCK(record(pr, st, -1));
    RCK(launch_px_patch(im->op_in, im->op_pe, rows, im->x, st));
    RCK(launch_px_embed(im->x, im->pos, im->lnpw, im->lnpb, rows, st));
    n += 2;
    RCK(record(pr, st, Q_PATCH));
    for (int i = 0; i < im->nl; i++) {
        PxLayer &L = im->L[i];
        const int Ls = L.glob ? PXT : PXLW;
        RCK(launch_ln_e4m3(im->x, L.ln1w, L.ln1b, im->h8, rows, 1.0f / L.adq[0], st));
        RCK(record(pr, st, Q_LN1));
        RCK(launch_px_qkv(im->op_h8, L.w[0], L.adq[0], rows, Ls, im->q8, im->k8, im->v8, L.glob ? im->csg : im->csw,
                          L.bqkv, L.cq, L.ck, L.cv, st));
        RCK(record(pr, st, Q_QKV));
        RCK(launch_px_attention(im->attn, rows / Ls, Ls, im->h8, L.sinv, L.vo, st));
        RCK(record(pr, st, L.glob ? Q_ATTG : Q_ATTW));
        RCK(launch_px_resid(im->op_h8, L.w[1], L.adq[1], rows, im->xm, L.bo, W_O, st));
        RCK(record(pr, st, Q_OPROJ));
        RCK(launch_ln_e4m3(im->x, L.ln2w, L.ln2b, im->h8, rows, 1.0f / L.adq[2], st));
        RCK(record(pr, st, Q_LN2));
        RCK(launch_px_fc1(im->op_h8, L.w[2], L.adq[2], rows, im->um, L.b1, L.rs, st));
        RCK(record(pr, st, Q_FC1));
        RCK(launch_px_resid(im->op_u8, L.w[3], L.adq[3], rows, im->xm, L.b2, W_FC2, st));
        RCK(record(pr, st, Q_FC2));
        n += 7;
    }
    RCK(launch_px_head(im->x, nb, im->hnw, im->hnb, im->hpos, im->U, im->wv, im->y, im->s, im->P, im->part, im->o, st));
    RCK(launch_head_f16(im->op_hw, im->op_o, nb, (int)p->nt, im->hb, im->out, st));
    n += 5;
    RCK(record(pr, st, Q_HEAD));
    im->launches = n;
    return 0;
}

int engine_up(px *p)
{
    PxImpl *im = I(p);
    ECK(cudaSetDevice(im->dev));
    RCK(prepare_px_kernels());
    FILE *f = fopen(im->path.c_str(), "rb");
    if (!f) {
        fprintf(stderr, "px: cannot open %s\n", im->path.c_str());
        return -1;
    }
    uint8_t *blob = nullptr;
    ECK(cudaHostAlloc((void **)&blob, im->wbytes, cudaHostAllocPortable));
    bool ok = fseek(f, 256, SEEK_SET) == 0 && fread(blob, 1, im->wbytes, f) == im->wbytes;
    fclose(f);
    if (!ok) {
        fprintf(stderr, "px: cannot stream weights from %s\n", im->path.c_str());
        cudaFreeHost(blob);
        return -1;
    }
    im->table.assign((const float *)blob, (const float *)blob + (size_t)im->nl * 12);
    ECK(cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking));
    ECK(cudaMalloc(&im->wts, im->wbytes));
    ECK(cudaMemcpyAsync(im->wts, blob, im->wbytes, cudaMemcpyHostToDevice, im->st));
    ECK(cudaStreamSynchronize(im->st));
    cudaFreeHost(blob);
    RCK(layout(im, p));
    const int nb = (int)p->nb, rows = nb * PXT;
    ECK(cudaMalloc(&im->in, (size_t)nb * PX_IN * 2));
    ECK(cudaMalloc(&im->x, (size_t)rows * D * 2));
    ECK(cudaMalloc(&im->y, (size_t)rows * D * 2));
    ECK(cudaMalloc(&im->h8, (size_t)rows * D));
    ECK(cudaMalloc(&im->q8, (size_t)rows * D));
    ECK(cudaMalloc(&im->k8, (size_t)rows * D));
    ECK(cudaMalloc(&im->v8, (size_t)rows * D));
    ECK(cudaMalloc(&im->u8, (size_t)rows * PXHID));
    ECK(cudaMalloc(&im->s, (size_t)rows * NH * 4));
    ECK(cudaMalloc(&im->P, (size_t)nb * NH * PXT * 2));
    ECK(cudaMalloc(&im->part, (size_t)nb * (PXT / 144) * NH * D * 4));
    ECK(cudaMalloc(&im->o, (size_t)nb * D * 2));
    ECK(cudaMalloc(&im->out, (size_t)nb * p->nt * 4));
    ECK(cudaMemsetAsync(im->in, 0, (size_t)nb * PX_IN * 2, im->st));
    RCK(make_operand(&im->op_in, im->in, rows, K0P * 2, 128));
    RCK(make_operand(&im->op_pe, im->pe, D, K0P * 2, 256));
    RCK(make_operand(&im->op_h8, im->h8, rows, D, 128));
    RCK(make_operand(&im->op_u8, im->u8, rows, PXHID, 128));
    RCK(make_operand(&im->op_hw, im->hw, (int)p->nt, D * 2, 128));
    RCK(make_operand(&im->op_o, im->o, nb, D * 2, 64));
    RCK(resid_map(&im->xm, im->x, rows));
    RCK(px_u8_map(&im->um, im->u8, rows));
    RCK(make_attn_rows(&im->attn, im->q8, im->k8, im->v8, rows));
    for (int s = 0; s < PX_NBUF; s++)
        ECK(cudaEventCreateWithFlags(&im->done[s], cudaEventDisableTiming | cudaEventBlockingSync));
    ECK(cudaHostAlloc((void **)&im->errh, PX_NBUF * sizeof(uint32_t), cudaHostAllocPortable));
    memset(im->errh, 0, PX_NBUF * sizeof(uint32_t));
    ECK(cudaStreamSynchronize(im->st));
    cudaGraph_t g;
    ECK(cudaStreamBeginCapture(im->st, cudaStreamCaptureModeThreadLocal));
    if (forward(im, p, nullptr)) {
        cudaStreamEndCapture(im->st, &g);
        return -1;
    }
    ECK(cudaStreamEndCapture(im->st, &g));
    ECK(cudaGraphInstantiate(&im->graph, g, 0));
    ECK(cudaGraphDestroy(g));
    ECK(cudaGraphUpload(im->graph, im->st));
    for (int s = 0; s < PX_NBUF; s++)
        ECK(cudaHostRegister(p->hout[s], (((size_t)p->nb * p->nt * 4) + 4095) & ~(size_t)4095, cudaHostRegisterPortable));
    im->out_reg = true;
    if (im->ipool && im->ipoolb) {
        ECK(cudaHostRegister(im->ipool, im->ipoolb, cudaHostRegisterPortable));
        im->pool_reg = true;
    }
    ECK(cudaStreamSynchronize(im->st));
    return 0;
}

}  // namespace

extern "C" {

int px_open_ex(px *p, const char *weights, int device, uint32_t nb, void *pool, size_t poolb)
{
    memset(p, 0, sizeof(*p));
    FILE *f = fopen(weights, "rb");
    uint32_t hdr[6] = {0, 0, 0, 0, 0, 0};
    if (!f || fread(hdr, 4, 6, f) != 6 || memcmp(hdr, "PXAI", 4) || hdr[1] != 3) {
        fprintf(stderr, "px: %s is not a pixai.bin v3 (run export_pixai.py with the calibration file)\n", weights);
        if (f) fclose(f);
        return -1;
    }
    fclose(f);
    const int nl = hdr[4] ? (int)hdr[4] : PX_NL;
    if (nl < 1 || nl > 32 || hdr[2] == 0 || nb == 0 || nb > 64) {
        fprintf(stderr, "px: %s: %d blocks, %u tags, batch %u not supported\n", weights, nl, hdr[2], nb);
        return -1;
    }
    PxImpl *im = new PxImpl();
    im->path = weights;
    im->wbytes = hdr[3];
    im->nl = nl;
    im->gmask = hdr[5];
    im->dev = device;
    im->ipool = pool;
    im->ipoolb = poolb;
    p->impl = im;
    p->nt = hdr[2];
    p->ntp = (hdr[2] + 7) & ~7u;
    p->nb = nb;
    for (int s = 0; s < PX_NBUF; s++) {
        p->hout[s] = (float *)aligned_alloc(4096, (((size_t)nb * p->nt * 4) + 4095) & ~(size_t)4095);
        if (!p->hout[s]) return -1;
    }
    im->boot_running = true;
    im->boot = std::thread([p, im] { im->bstatus = engine_up(p); });
    return 0;
}

int px_open_multi(px *p, const char *weights, const int *devices, int ndev, uint32_t nb, void *pool, size_t poolb)
{
    if (ndev == 1 && devices) return px_open_ex(p, weights, devices[0], nb, pool, poolb);
    memset(p, 0, sizeof(*p));
    if (!devices || ndev < 1 || ndev > 8 || nb < (uint32_t)ndev || nb > 64u * (uint32_t)ndev) {
        fprintf(stderr, "px: %d devices with batch %u not supported (1..8 devices, 1..64 inputs per device)\n", ndev, nb);
        return -1;
    }
    PxImpl *im = new PxImpl();
    im->subs.resize(ndev);
    im->lo.resize(ndev);
    uint32_t lo = 0;
    for (int i = 0; i < ndev; i++) {
        const uint32_t ni = (nb + ndev - 1 - i) / ndev;  // contiguous shards, sizes differ by at most 1
        im->lo[i] = lo;
        // the caller's pool is page-locked once, by the first device's bring-up (portable: every device reads it)
        if (px_open_ex(&im->subs[i], weights, devices[i], ni, i == 0 ? pool : nullptr, i == 0 ? poolb : 0)) {
            for (int j = 0; j < i; j++) px_close(&im->subs[j]);
            delete im;
            return -1;
        }
        lo += ni;
    }
    p->impl = im;
    p->nt = im->subs[0].nt;
    p->ntp = im->subs[0].ntp;
    p->nb = nb;
    for (int s = 0; s < PX_NBUF; s++) {
        p->hout[s] = (float *)aligned_alloc(4096, (((size_t)nb * p->nt * 4) + 4095) & ~(size_t)4095);
        if (!p->hout[s]) {
            px_close(p);
            return -1;
        }
    }
    return 0;
}

int px_open(px *p, const char *weights, int device, void *pool, size_t poolb)
{
    return px_open_ex(p, weights, device, PX_NB, pool, poolb);
}

int px_ready(px *p)
{
    PxImpl *im = I(p);
    if (!im) return -1;
    if (im->up) return 0;
    if (im->multi()) {
        int rc = 0;
        for (px &q : im->subs) rc |= px_ready(&q);  // join every bring-up, even after a failure
        if (rc) return -1;
        im->up = true;
        return 0;
    }
    if (im->boot_running) {
        im->boot.join();
        im->boot_running = false;
    }
    if (im->bstatus) return -1;
    if (cudaSetDevice(im->dev) != cudaSuccess) return -1;
    im->up = true;
    return 0;
}

int px_poll(px *p)
{
    PxImpl *im = I(p);
    if (im && im->multi() && !im->up) {
        for (px &q : im->subs)
            if (!px_poll(&q)) return 0;
        return 1;
    }
    return im && (im->up || im->bstatus != -1 || !im->boot_running);
}

int px_submit(px *p, uint32_t buf, uint16_t *const *in, uint32_t n)
{
    if (px_ready(p) || buf >= PX_NBUF || n > p->nb) return -1;
    PxImpl *im = I(p);
    if (im->multi()) {
        for (size_t i = 0; i < im->subs.size(); i++) {
            const uint32_t ni = shard_n(im, i, n);
            if (ni && px_submit(&im->subs[i], buf, in + im->lo[i], ni)) return -1;
        }
        im->slot_n[buf] = n;
        return 0;
    }
    for (uint32_t i = 0, j; i < n; i = j) {
        for (j = i + 1; j < n && in[j] == in[j - 1] + PX_IN; j++)
            ;
        ECK(cudaMemcpyAsync(im->in + (size_t)i * PX_IN, in[i], (size_t)(j - i) * PX_IN * 2, cudaMemcpyHostToDevice,
                            im->st));
    }
    ECK(cudaGraphLaunch(im->graph, im->st));
    ECK(cudaMemcpyAsync(p->hout[buf], im->out, (size_t)n * p->nt * 4, cudaMemcpyDeviceToHost, im->st));
    ECK(cudaMemcpyAsync(&im->errh[buf], error_word(im->dev), 4, cudaMemcpyDeviceToHost, im->st));
    ECK(cudaEventRecord(im->done[buf], im->st));
    return 0;
}

int px_query(px *p, uint32_t buf)
{
    PxImpl *im = I(p);
    if (!im || !im->up || buf >= PX_NBUF) return 1;
    if (im->multi()) {
        for (size_t i = 0; i < im->subs.size(); i++)
            if (shard_n(im, i, im->slot_n[buf]) && !px_query(&im->subs[i], buf)) return 0;
        return 1;
    }
    return cudaEventQuery(im->done[buf]) != cudaErrorNotReady;
}

const float *px_wait(px *p, uint32_t buf)
{
    PxImpl *im = I(p);
    if (!im || !im->up || buf >= PX_NBUF) return nullptr;
    if (im->multi()) {  // every shard's scores into its rows of this handle's slot
        const float *ok = p->hout[buf];
        for (size_t i = 0; i < im->subs.size(); i++) {
            const uint32_t ni = shard_n(im, i, im->slot_n[buf]);
            if (!ni) continue;
            const float *r = px_wait(&im->subs[i], buf);
            if (!r) ok = nullptr;
            else memcpy(p->hout[buf] + (size_t)im->lo[i] * p->nt, r, (size_t)ni * p->nt * 4);
        }
        return ok;
    }
    if (cudaEventSynchronize(im->done[buf]) != cudaSuccess) return nullptr;
    if (im->errh[buf]) {
        fprintf(stderr, "px: batch %u: device error word 0x%x (a bounded wait ran out)\n", buf, im->errh[buf]);
        return nullptr;
    }
    return p->hout[buf];
}

void px_close(px *p)
{
    PxImpl *im = I(p);
    if (!im) return;
    if (im->multi()) {
        for (px &q : im->subs) px_close(&q);
        for (int s = 0; s < PX_NBUF; s++) free(p->hout[s]);
        delete im;
        memset(p, 0, sizeof(*p));
        return;
    }
    if (im->boot_running) {
        im->boot.join();
        im->boot_running = false;
    }
    cudaSetDevice(im->dev);
    if (im->st) cudaStreamSynchronize(im->st);
    if (im->graph) cudaGraphExecDestroy(im->graph);
    for (int s = 0; s < PX_NBUF; s++) {
        if (im->done[s]) cudaEventDestroy(im->done[s]);
        if (im->out_reg && p->hout[s]) cudaHostUnregister(p->hout[s]);
        free(p->hout[s]);
        p->hout[s] = nullptr;
    }
    if (im->pool_reg) cudaHostUnregister(im->ipool);
    void *bufs[] = {im->in, im->x, im->y, im->h8, im->q8, im->k8, im->v8, im->u8, im->s, im->P, im->part, im->o,
                    im->out, im->wts};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (im->errh) cudaFreeHost(im->errh);
    if (im->st) cudaStreamDestroy(im->st);
    delete im;
    p->impl = nullptr;
}

// ---- extensions (no counterpart in the reference) ----
int px_forward_resident(px *p)
{
    if (px_ready(p)) return -1;
    if (I(p)->multi()) {
        for (px &q : I(p)->subs)
            if (px_forward_resident(&q)) return -1;
        return 0;
    }
    ECK(cudaGraphLaunch(I(p)->graph, I(p)->st));
    return 0;
}

int px_upload(px *p, uint16_t *const *in, uint32_t n)
{
    if (px_ready(p) || n > p->nb) return -1;
    PxImpl *im = I(p);
    if (im->multi()) {
        for (size_t i = 0; i < im->subs.size(); i++) {
            const uint32_t ni = shard_n(im, i, n);
            if (ni && px_upload(&im->subs[i], in + im->lo[i], ni)) return -1;
        }
        return 0;
    }
    for (uint32_t i = 0; i < n; i++)
        ECK(cudaMemcpyAsync(im->in + (size_t)i * PX_IN, in[i], PX_IN * 2, cudaMemcpyHostToDevice, im->st));
    ECK(cudaStreamSynchronize(im->st));
    return 0;
}

int px_download(px *p, float *out, uint32_t n)
{
    if (px_ready(p) || n > p->nb) return -1;
    PxImpl *im = I(p);
    if (im->multi()) {
        for (size_t i = 0; i < im->subs.size(); i++) {
            const uint32_t ni = shard_n(im, i, n);
            if (ni && px_download(&im->subs[i], out + (size_t)im->lo[i] * p->nt, ni)) return -1;
        }
        return 0;
    }
    ECK(cudaStreamSynchronize(im->st));
    ECK(cudaMemcpy(out, im->out, (size_t)n * p->nt * 4, cudaMemcpyDeviceToHost));
    return 0;
}

int px_head_input(px *p, uint16_t *o, uint32_t n)
{
    if (px_ready(p) || n > p->nb) return -1;
    PxImpl *im = I(p);
    if (im->multi()) {
        for (size_t i = 0; i < im->subs.size(); i++) {
            const uint32_t ni = shard_n(im, i, n);
            if (ni && px_head_input(&im->subs[i], o + (size_t)im->lo[i] * D, ni)) return -1;
        }
        return 0;
    }
    ECK(cudaStreamSynchronize(im->st));
    ECK(cudaMemcpy(o, im->o, (size_t)n * D * 2, cudaMemcpyDeviceToHost));
    return 0;
}

// with several devices: the first device's (its shard's inputs, its stream, its launches)
void *px_stream(px *p) { return px_ready(p) ? nullptr : I(p)->multi() ? px_stream(&I(p)->subs[0]) : (void *)I(p)->st; }
void *px_input(px *p) { return px_ready(p) ? nullptr : I(p)->multi() ? px_input(&I(p)->subs[0]) : (void *)I(p)->in; }
int px_launches_per_forward(px *p)
{
    return px_ready(p) ? -1 : I(p)->multi() ? px_launches_per_forward(&I(p)->subs[0]) : I(p)->launches;
}

int px_profile(px *p, float *ms, int kinds)
{
    if (px_ready(p)) return -1;
    PxImpl *im = I(p);
    if (im->multi()) return px_profile(&im->subs[0], ms, kinds);  // the first device's shard
    for (int w = 0; w < 2; w++)
        if (forward(im, p, nullptr)) return -1;
    Prof pr;
    if (forward(im, p, &pr)) return -1;
    ECK(cudaStreamSynchronize(im->st));
    for (int k = 0; k < kinds && k < Q_KINDS; k++) ms[k] = 0.f;
    for (size_t i = 1; i < pr.ev.size(); i++) {
        float t = 0.f;
        ECK(cudaEventElapsedTime(&t, pr.ev[i - 1], pr.ev[i]));
        if (pr.kind[i] >= 0 && pr.kind[i] < kinds) ms[pr.kind[i]] += t;
    }
    for (cudaEvent_t e : pr.ev) cudaEventDestroy(e);
    return Q_KINDS;
}

const char *px_prof_name(int k) { return k >= 0 && k < Q_KINDS ? px_prof_names[k] : nullptr; }

}  // extern "C"

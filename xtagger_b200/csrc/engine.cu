// The eva_* engine: a drop-in for the wd engine of xTagger (src/engine/eva.h) on one or more B200s.
//
// Bring-up (eva_open / eva_open_ex -> boot thread): read the weight file (v3 per-tensor or v4 block-scaled) into
// pinned host memory, copy it to every device, resolve the tensor layout, allocate the activations for the
// device's batch, build the TMA descriptors, capture the whole forward (196 launches) into one CUDA graph per
// device (one per input buffer). Per batch (eva_submit): H2D of the inputs (adjacent pool inputs in one copy) on a
// copy stream into one of two input buffers, graph launch once they have landed, D2H of the
// scores (and head inputs), event; eva_wait sleeps on the events. Multi-GPU: one replica per device with its own
// stream and graph; a submit's inputs are split into contiguous shards, one per device, and the scores land in
// disjoint rows of one host slot. No collective is involved.
// 2:4-sparse weights (prune24.py's output, or a block-scaled file pruned the same way): with XTB_SPARSE=1 in the
// environment, every projection kind whose weights are 2:4 along k in all layers is compressed at bring-up and runs
// on the sparse tensor cores (tcgen05.mma.sp, gemm_sp.cuh) with the same results. Off by default: on B200 the
// transposed epilogues the sparse operand forces cost more than the sparse MMA saves, so the dense kernels are
// faster on the same pruned weights.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cmath>
#include <string>
#include <thread>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "../../include/xtagger_b200.h"
#include "host.h"
#include "ops.h"

using namespace xtb;

namespace {

constexpr int NG = 4;  // block GEMMs per layer: QKV, O, W12, W2

struct Layer {
    const float *ln1w, *ln1b, *ln2w, *ln2b, *rs, *c, *d;
    Weight8 w[NG];
    SparseW sw[NG];  // kinds in Impl::sp_mask: the compressed weight
    float adq[NG], cq, ck, cv, sinv, vo;
};

enum ProfKind { P_PATCH, P_LN1, P_QKV, P_ATTN, P_OPROJ, P_LN2, P_FC1, P_FC2, P_HEAD, P_KINDS };
const char *const prof_names[P_KINDS] = {"patch+embed", "ln1", "qkv", "attention", "oproj", "ln2", "fc1", "fc2", "pool+head"};

struct Replica {
    int dev = 0, nb = 0;
    cudaStream_t st = nullptr;
    uint8_t *wts = nullptr;
    float *sexp = nullptr;         // v3: expanded per-tensor scales
    __half *in = nullptr, *x = nullptr, *pn = nullptr;
    uint8_t *h = nullptr, *q8 = nullptr, *k8 = nullptr, *v8 = nullptr, *h8 = nullptr, *pn8 = nullptr;
    float2 *stat = nullptr;
    float *pool = nullptr, *out = nullptr;
    uint8_t *hw = nullptr;         // head weights used by the forward (a copy when there are extra rows)
    float *hb = nullptr, *hws = nullptr;
    bool head_copy = false;
    const uint8_t *hw0 = nullptr;  // head inside the blob
    const float *hb0 = nullptr, *hws0 = nullptr;
    const __half *pe = nullptr;
    const float *pos = nullptr, *cs = nullptr, *fnw = nullptr, *fnb = nullptr;
    std::vector<Layer> L;
    Operand op_in, op_pe, op_h, op_h8, op_hw, op_pn;
    Operand op_h_sp, op_h8_sp;     // the same activations in the sparse kernels' token boxes
    uint8_t *spw = nullptr;        // compressed 2:4 weights (Impl::sp_host on this device)
    uint8_t *sfimg = nullptr;      // fc1 scale-factor images (power-of-two block scales), every layer
    Weight8 whead;
    Attn attn;
    cudaGraphExec_t graph = nullptr;   // the forward reading input buffer 0 (in)
    cudaEvent_t done[EVA_NBUF] = {};
    int launches = 0;
    // submits alternate between two input buffers so that the copies of one batch (on cst) overlap the forward of
    // the previous one (on st): graph reads in, graph_b reads in_b; in_ready[k] / in_free[k] order the copy stream
    // and the compute stream for buffer k
    __half *in_b = nullptr;             // input buffer 1 (buffer 0 is in)
    cudaGraphExec_t graph_b = nullptr;  // the forward reading in_b
    cudaStream_t cst = nullptr;
    // the last query row's attention kernel runs on its own branch of the forward (fork / join events)
    cudaStream_t ast = nullptr;
    cudaEvent_t afork = nullptr, ajoin = nullptr;
    cudaEvent_t in_ready[2] = {}, in_free[2] = {};
    int ib = 0;                         // input buffer of the next submit
    uint32_t *errh = nullptr;           // pinned, per slot: the device error word after the slot's forward
};

struct Impl {
    std::thread boot;
    bool boot_running = false;
    int bstatus = -1;
    bool up = false;
    std::string path;
    size_t wbytes = 0;
    int ver = 3, nl = 24, head8 = 0;
    float head_adq = 1.0f;
    std::vector<float> table;
    std::vector<int> devices;
    std::vector<Replica> reps;
    void *ipool = nullptr;
    size_t ipoolb = 0;
    bool pool_reg = false, out_reg = false;
    uint32_t extra = 0;
    std::vector<float> hws_host;   // FP8 head block scales (host copy, for eva_head_put)
    // 2:4-sparse projections: bit g set = kind g (QKV, O, W12, W2) runs on the sparse kernels; the compressed
    // weights of every layer in one host buffer (layer i, kind g at sp_off[i * NG + g]; metadata after the values)
    int sp_mask = 0;
    bool sp_ready = false;
    std::vector<uint8_t> sp_host;
    std::vector<size_t> sp_off;
    uint32_t last_n = 0;
};

Impl *I(eva *e) { return (Impl *)e->impl; }

#define ECK(call)                                                                                 \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) {                                                                  \
            fprintf(stderr, "eva: %s: %s\n", #call, cudaGetErrorString(e_));                      \
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

int kblocks(int k) { return (k + 127) / 128; }

// Blob offsets of the head tensors (walks the layout of model.py / eva.h:378-430 without touching memory).
struct HeadOff {
    size_t hsc, hw, hws, hb, end;
};
HeadOff head_offsets(const Impl *im, uint32_t ntp)
{
    size_t off = 0;
    const bool v4 = im->ver == 4;
    take(&off, (size_t)im->nl * 12 * 4);
    take(&off, (size_t)D * K0P * 2);
    take(&off, (size_t)T * D * 4);
    take(&off, (size_t)NP * 32 * 2 * 4);
    const int kn[NG][2] = {{3 * D, D}, {D, D}, {N12, D}, {D, HIDP}};
    for (int i = 0; i < im->nl; i++) {
        take(&off, D * 4);
        take(&off, D * 4);
        for (int g = 0; g < NG; g++) {
            if (g == 2) {
                take(&off, D * 4);
                take(&off, D * 4);
            }
            if (g == 3) take(&off, HIDP * 4);
            take(&off, (size_t)kn[g][0] * kn[g][1]);
            if (v4) take(&off, (size_t)kblocks(kn[g][0]) * kblocks(kn[g][1]) * 4);
        }
        take(&off, D * 4);
        take(&off, D * 4);
    }
    take(&off, D * 4);
    take(&off, D * 4);
    HeadOff h{};
    if (im->head8) {
        h.hsc = take(&off, 16);
        h.hw = take(&off, (size_t)ntp * D);
        h.hws = take(&off, (size_t)((ntp + 127) / 128) * 8 * 4);
    } else {
        h.hw = take(&off, (size_t)ntp * D * 2);
    }
    h.hb = take(&off, (size_t)ntp * 4);
    h.end = off;
    return h;
}

// Tensor addresses of the blob on device (layout: model.py / eva.h:378-430) and the per-layer multipliers
// (eva.h:408-418). v3 per-tensor weight scales are expanded to uniform block-scale arrays.
int layout(Impl *im, Replica &r, const uint8_t *hostblob)
{
    (void)hostblob;
    size_t off = 0;
    const int v4 = im->ver == 4;
    uint8_t *B = r.wts;
    take(&off, (size_t)im->nl * 12 * 4);
    r.pe = (const __half *)(B + take(&off, (size_t)D * K0P * 2));
    r.pos = (const float *)(B + take(&off, (size_t)T * D * 4));
    r.cs = (const float *)(B + take(&off, (size_t)NP * 32 * 2 * 4));
    const int kn[NG][2] = {{3 * D, D}, {D, D}, {N12, D}, {D, HIDP}};
    size_t sexp_n = 0;
    for (int g = 0; g < NG; g++) sexp_n += (size_t)kblocks(kn[g][0]) * kblocks(kn[g][1]);
    std::vector<float> sexp_h;
    if (!v4) {
        sexp_h.resize(sexp_n * im->nl);
        ECK(cudaMalloc(&r.sexp, sexp_h.size() * 4));
    }
    r.L.resize(im->nl);
    size_t so = 0;
    for (int i = 0; i < im->nl; i++) {
        Layer &L = r.L[i];
        const float *tb = &im->table[(size_t)i * 12];
        L.ln1w = (const float *)(B + take(&off, D * 4));
        L.ln1b = (const float *)(B + take(&off, D * 4));
        const uint8_t *wp[NG];
        const float *sp[NG] = {nullptr, nullptr, nullptr, nullptr};
        wp[0] = B + take(&off, (size_t)3 * D * D);
        if (v4) sp[0] = (const float *)(B + take(&off, (size_t)kblocks(3 * D) * kblocks(D) * 4));
        wp[1] = B + take(&off, (size_t)D * D);
        if (v4) sp[1] = (const float *)(B + take(&off, (size_t)kblocks(D) * kblocks(D) * 4));
        L.ln2w = (const float *)(B + take(&off, D * 4));
        L.ln2b = (const float *)(B + take(&off, D * 4));
        wp[2] = B + take(&off, (size_t)N12 * D);
        if (v4) sp[2] = (const float *)(B + take(&off, (size_t)kblocks(N12) * kblocks(D) * 4));
        L.rs = (const float *)(B + take(&off, HIDP * 4));
        wp[3] = B + take(&off, (size_t)D * HIDP);
        if (v4) sp[3] = (const float *)(B + take(&off, (size_t)kblocks(D) * kblocks(HIDP) * 4));
        L.c = (const float *)(B + take(&off, D * 4));
        L.d = (const float *)(B + take(&off, D * 4));
        for (int g = 0; g < NG; g++) {
            const int n = kn[g][0], k = kn[g][1];
            if (!v4) {
                const size_t cnt = (size_t)kblocks(n) * kblocks(k);
                for (size_t j = 0; j < cnt; j++) sexp_h[so + j] = tb[g];
                sp[g] = r.sexp + so;
                so += cnt;
            }
            L.w[g].ws = sp[g];
            L.w[g].uniform = v4 ? 0.0f : tb[g];  // v3: one scale per tensor, applied once after the K sum
            L.w[g].n = n;
            L.w[g].k = k;
            RCK(make_operand(&L.w[g].op, wp[g], n, k, weight_box_rows((WeightUse)g)));  // g: W_QKV, W_O, W_FC1, W_FC2
            L.adq[g] = tb[4 + g];
        }
        L.cq = 1.0f / tb[8];
        L.ck = 1.0f / tb[9];
        L.cv = 1.0f / tb[10];
        L.sinv = tb[8] * tb[9];
        L.vo = (1.0f / tb[5]) * tb[10];
    }
    if (!v4) ECK(cudaMemcpy(r.sexp, sexp_h.data(), sexp_h.size() * 4, cudaMemcpyHostToDevice));
    r.fnw = (const float *)(B + take(&off, D * 4));
    r.fnb = (const float *)(B + take(&off, D * 4));
    return (int)off;  // caller continues with the head
}

int head_layout(Impl *im, Replica &r, eva *e, size_t off)
{
    uint8_t *B = r.wts;
    const uint32_t ntp0 = e->ntp;
    if (im->head8) {
        take(&off, 16);
        r.hw0 = B + take(&off, (size_t)ntp0 * D);
        r.hws0 = (const float *)(B + take(&off, (size_t)((ntp0 + 127) / 128) * 8 * 4));
    } else {
        r.hw0 = B + take(&off, (size_t)ntp0 * D * 2);
    }
    r.hb0 = (const float *)(B + take(&off, (size_t)ntp0 * 4));
    if (off != im->wbytes) {
        fprintf(stderr, "eva: weight layout mismatch (%zu vs %zu bytes)\n", off, im->wbytes);
        return -1;
    }
    return 0;
}

// The forward of nb images on replica r's stream. prof: events after each launch (direct, non-graph runs).
struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
};

int record(Prof *p, cudaStream_t st, int kind)
{
    if (!p) return 0;
    cudaEvent_t ev;
    ECK(cudaEventCreate(&ev));
    ECK(cudaEventRecord(ev, st));
    p->ev.push_back(ev);
    p->kind.push_back(kind);
    return 0;
}

int forward(Impl *im, Replica &r, eva *e, Prof *p)
{
    const int nb = r.nb, rows = nb * T;
    cudaStream_t st = r.st;
    int n = 0;
    RCK(record(p, st, -1));
    RCK(launch_patch_embed(r.op_in, r.op_pe, nb, r.pos, r.x, st));
    n++;
    RCK(record(p, st, P_PATCH));
    for (int i = 0; i < im->nl; i++) {
        Layer &L = r.L[i];
        RCK(launch_ln_e4m3(r.x, L.ln1w, L.ln1b, r.h, rows, 1.0f / L.adq[0], st));
        RCK(record(p, st, P_LN1));
        const int sm = im->sp_mask;
        if (sm & 1) RCK(launch_qkv_sp(r.op_h_sp, L.sw[0], L.adq[0], rows, r.q8, r.k8, r.v8, r.cs, L.cq, L.ck, L.cv, st));
        else RCK(launch_qkv(r.op_h, L.w[0], L.adq[0], rows, r.q8, r.k8, r.v8, r.cs, L.cq, L.ck, L.cv, st));
        RCK(record(p, st, P_QKV));
        // the last query row (k_attention_last) on a parallel branch: it overlaps the main attention kernel
        ECK(cudaEventRecord(r.afork, st));
        ECK(cudaStreamWaitEvent(r.ast, r.afork, 0));
        RCK(launch_attention(r.attn, nb, r.h, L.sinv, L.vo, st, r.ast));
        ECK(cudaEventRecord(r.ajoin, r.ast));
        ECK(cudaStreamWaitEvent(st, r.ajoin, 0));
        RCK(record(p, st, P_ATTN));
        if (sm & 2) RCK(launch_oproj_sp(r.op_h_sp, L.sw[1], L.adq[1], rows, r.x, st));
        else RCK(launch_oproj(r.op_h, L.w[1], L.adq[1], rows, r.x, st));
        RCK(record(p, st, P_OPROJ));
        RCK(launch_ln_e4m3(r.x, L.ln2w, L.ln2b, r.h, rows, 1.0f / L.adq[2], st));
        RCK(record(p, st, P_LN2));
        if (sm & 4) RCK(launch_fc1_sp(r.op_h_sp, L.sw[2], L.adq[2], rows, r.h8, r.stat, L.rs, st));
        else RCK(launch_fc1(r.op_h, L.w[2], L.adq[2], rows, r.h8, r.stat, L.rs, st));
        RCK(record(p, st, P_FC1));
        if (sm & 8) RCK(launch_fc2_sp(r.op_h8_sp, L.sw[3], L.adq[3], rows, r.x, r.stat, L.c, L.d, st));
        else RCK(launch_fc2(r.op_h8, L.w[3], L.adq[3], rows, r.x, r.stat, L.c, L.d, st));
        RCK(record(p, st, P_FC2));
        n += (sm & 8) ? 9 : 8;  // ln1, qkv, attention (2), oproj, ln2, fc1, fc2 (+ row statistics when sparse)
    }
    RCK(launch_pool_ln(r.x, nb, r.fnw, r.fnb, r.pool, r.pn, im->head8 ? r.pn8 : nullptr, 1.0f / im->head_adq, st));
    n += 2;
    if (im->head8) RCK(launch_head_e4m3(r.whead, r.op_pn, im->head_adq, nb, (int)e->nt, r.hb, r.out, st));
    else RCK(launch_head_f16(r.op_hw, r.op_pn, nb, (int)e->nt, r.hb, r.out, st));
    n++;
    RCK(record(p, st, P_HEAD));
    r.launches = n;
    return 0;
}

// Which projection kinds are 2:4 in every layer, and their compressed form (once per engine, from the host blob;
// r is the first replica, whose layout gives the weight offsets). Layers are compressed on parallel threads.
int sparse_prepare(Impl *im, Replica &r, const uint8_t *hostblob)
{
    im->sp_ready = true;
    const char *env = getenv("XTB_SPARSE");
    if (!env || env[0] != '1') return 0;
    auto host_w = [&](int i, int g) { return hostblob + ((const uint8_t *)r.L[i].w[g].op.ptr - r.wts); };
    for (int g = 0; g < NG; g++) {
        bool all = true;
        for (int i = 0; i < im->nl && all; i++) all = sparse24_check(host_w(i, g), r.L[i].w[g].n, r.L[i].w[g].k) != 0;
        if (all) im->sp_mask |= 1 << g;
    }
    if (!im->sp_mask) return 0;
    im->sp_off.assign((size_t)im->nl * NG, 0);
    size_t total = 0;
    for (int i = 0; i < im->nl; i++)
        for (int g = 0; g < NG; g++)
            if (im->sp_mask & (1 << g)) {
                im->sp_off[(size_t)i * NG + g] = total;
                total += (sparse24_bytes(r.L[i].w[g].n, r.L[i].w[g].k, nullptr) + 255) & ~(size_t)255;
            }
    im->sp_host.resize(total);
    const int nthr = std::max(1, std::min(im->nl, 8));
    std::vector<std::thread> th;
    std::vector<int> rcs(nthr, 0);
    for (int t = 0; t < nthr; t++)
        th.emplace_back([&, t] {
            for (int i = t; i < im->nl; i += nthr)
                for (int g = 0; g < NG; g++)
                    if (im->sp_mask & (1 << g)) {
                        const int n = r.L[i].w[g].n, k = r.L[i].w[g].k;
                        size_t moff = 0;
                        sparse24_bytes(n, k, &moff);
                        uint8_t *v = im->sp_host.data() + im->sp_off[(size_t)i * NG + g];
                        if (sparse24_compress(host_w(i, g), n, k, v, v + moff)) rcs[t] = -1;
                    }
        });
    for (auto &x : th) x.join();
    for (int rc : rcs)
        if (rc) return -1;
    return 0;
}

int replica_up(Impl *im, Replica &r, eva *e, const uint8_t *hostblob)
{
    ECK(cudaSetDevice(r.dev));
    RCK(prepare_kernels());
    ECK(cudaStreamCreateWithFlags(&r.st, cudaStreamNonBlocking));
    ECK(cudaStreamCreateWithFlags(&r.cst, cudaStreamNonBlocking));
    ECK(cudaStreamCreateWithFlags(&r.ast, cudaStreamNonBlocking));
    ECK(cudaEventCreateWithFlags(&r.afork, cudaEventDisableTiming));
    ECK(cudaEventCreateWithFlags(&r.ajoin, cudaEventDisableTiming));
    ECK(cudaMalloc(&r.wts, im->wbytes));
    ECK(cudaMemcpyAsync(r.wts, hostblob, im->wbytes, cudaMemcpyHostToDevice, r.st));
    int off = layout(im, r, hostblob);
    if (off < 0) return -1;
    RCK(head_layout(im, r, e, (size_t)off));
    if (!im->sp_ready) RCK(sparse_prepare(im, r, hostblob));
    if (im->ver == 4 && !im->sp_mask) {
        // projection kinds whose block scales are all powers of two, in every layer, run on the tensor core's own
        // block scaling (no per-K-block promotion); XTB_MX=0 in the environment keeps the promoting kernels
        // (promoting, the batch-64 forward spends 7.0 ms in QKV and 10.9 in fc1)
        // the CTA-pair block-scaled kernel (gemm2_mx.cuh) for the kinds in kMxPair, on 256 x 256 tiles (two weight
        // blocks per tile, half the A traffic per FLOP) for those in kMxWide (N a multiple of 256), else 256 x 128.
        // Measured in the batch-64 forward (power-capped clocks, ms per forward): fc2 4.97 on the pair's wide tiles
        // against 6.2 on the promoting pair and 6.5 on 128-column block-scaled tiles; QKV 4.41 wide against 4.95 on
        // 128-column tiles and 5.3 on one CTA; fc1 7.25-7.6 wide against 8.3 on one CTA and 8.25 on 128-column pair
        // tiles; the out-projection 1.86 on 128-column tiles against 1.96 wide and 2.4 promoting.
        // XTB_MX_KINDS / XTB_MX_PAIR / XTB_MX_WIDE (hex masks) in the environment override these for measurements.
        int kMxKinds = 0xF, kMxPair = 0xF, kMxWide = 0xD;
        if (const char *m = getenv("XTB_MX_KINDS")) kMxKinds = (int)strtol(m, nullptr, 16);
        if (const char *m = getenv("XTB_MX_PAIR")) kMxPair = (int)strtol(m, nullptr, 16);
        if (const char *m = getenv("XTB_MX_WIDE")) kMxWide = (int)strtol(m, nullptr, 16);
        const char *env = getenv("XTB_MX");
        if (!(env && env[0] == '0')) {
            size_t per[NG], off[NG], total = 0;
            int mask = 0;
            std::vector<uint8_t> img;
            for (int g = 0; g < NG; g++) {
                const int n = r.L[0].w[g].n, k = r.L[0].w[g].k;
                per[g] = sf_image_bytes(n, k);
                off[g] = total;
                if (!(kMxKinds & (1 << g))) continue;
                std::vector<uint8_t> part(per[g] * im->nl);
                bool all = true;
                for (int i = 0; i < im->nl && all; i++) {
                    const float *ws_h = (const float *)(hostblob + ((const uint8_t *)r.L[i].w[g].ws - r.wts));
                    all = sf_image(ws_h, n, k, part.data() + (size_t)i * per[g]) == 0;
                }
                if (!all) continue;
                mask |= 1 << g;
                img.insert(img.end(), part.begin(), part.end());
                total += part.size();
            }
            if (mask) {
                ECK(cudaMalloc(&r.sfimg, img.size()));
                ECK(cudaMemcpyAsync(r.sfimg, img.data(), img.size(), cudaMemcpyHostToDevice, r.st));
                ECK(cudaStreamSynchronize(r.st));  // the host image is pageable
                for (int g = 0; g < NG; g++) {
                    if (!(mask & (1 << g))) continue;
                    for (int i = 0; i < im->nl; i++) {
                        Weight8 &w = r.L[i].w[g];
                        w.sf = r.sfimg + off[g] + (size_t)i * per[g];
                        w.sf_nbp = ((w.n + 127) / 128 + 1) & ~1;
                        w.sf_pair = (kMxPair >> g) & 1;
                        // wide tiles need N a multiple of 256, or an epilogue that skips a half tile past N (fc1's)
                        w.sf_wide = w.sf_pair && ((kMxWide >> g) & 1) && (w.n % 256 == 0 || g == W_FC1);
                        // the block-scaled kernels' B boxes: 256 rows (one CTA) or 64 per CTA (pair)
                        RCK(make_operand(&w.op, w.op.ptr, w.n, w.k, w.sf_pair ? 64 : 256));
                        if (w.sf_pair) RCK(sf_map(&w.sfmap, w.sf, w.n, w.k));
                    }
                }
            }
        }
    }
    if (im->sp_mask) {
        ECK(cudaMalloc(&r.spw, im->sp_host.size()));
        ECK(cudaMemcpyAsync(r.spw, im->sp_host.data(), im->sp_host.size(), cudaMemcpyHostToDevice, r.st));
        for (int i = 0; i < im->nl; i++)
            for (int g = 0; g < NG; g++)
                if (im->sp_mask & (1 << g)) {
                    Layer &L = r.L[i];
                    size_t moff = 0;
                    sparse24_bytes(L.w[g].n, L.w[g].k, &moff);
                    const uint8_t *v = r.spw + im->sp_off[(size_t)i * NG + g];
                    RCK(make_sparse_weight(&L.sw[g], v, v + moff, L.w[g].n, L.w[g].k, L.w[g].ws));
                    L.sw[g].uniform = L.w[g].uniform;  // v3: one scale per tensor
                }
        ECK(cudaStreamSynchronize(r.st));  // the host buffer is pageable
    }
    const int nb = r.nb, rows = nb * T;
    // head used by the forward: the blob's rows, or a copy with the extra rows (zero weights, bias -16)
    const uint32_t nt = e->nt, nt0 = e->nt0;
    const size_t rowb = im->head8 ? D : (size_t)D * 2;
    if (nt > nt0) {
        const size_t nsb = (nt + 127) / 128, nsb0 = (e->ntp + 127) / 128;
        r.head_copy = true;
        ECK(cudaMalloc(&r.hw, (size_t)nt * rowb));
        ECK(cudaMalloc(&r.hb, (size_t)nt * 4));
        ECK(cudaMemcpyAsync(r.hw, r.hw0, (size_t)nt0 * rowb, cudaMemcpyDeviceToDevice, r.st));
        ECK(cudaMemsetAsync(r.hw + (size_t)nt0 * rowb, 0, (size_t)(nt - nt0) * rowb, r.st));
        ECK(cudaMemcpyAsync(r.hb, r.hb0, (size_t)nt0 * 4, cudaMemcpyDeviceToDevice, r.st));
        std::vector<float> tail(nt - nt0, -16.0f);  // EVA_HB_OFF: a row nothing has written never fires
        ECK(cudaMemcpyAsync(r.hb + nt0, tail.data(), tail.size() * 4, cudaMemcpyHostToDevice, r.st));
        if (im->head8) {
            ECK(cudaMalloc(&r.hws, nsb * 8 * 4));
            ECK(cudaMemcpyAsync(r.hws, im->hws_host.data(), nsb * 8 * 4, cudaMemcpyHostToDevice, r.st));
            (void)nsb0;
        }
        ECK(cudaStreamSynchronize(r.st));
    } else {
        r.hw = (uint8_t *)r.hw0;
        r.hb = (float *)r.hb0;
        r.hws = (float *)r.hws0;
    }
    // activations
    ECK(cudaMalloc(&r.in, (size_t)nb * EVA_IN * 2));
    ECK(cudaMalloc(&r.in_b, (size_t)nb * EVA_IN * 2));
    ECK(cudaMalloc(&r.x, (size_t)rows * D * 2));
    ECK(cudaMalloc(&r.h, (size_t)rows * D));
    const size_t qkb = (size_t)nb * NH * TP * HD;
    ECK(cudaMalloc(&r.q8, qkb));
    ECK(cudaMalloc(&r.k8, qkb));
    ECK(cudaMalloc(&r.v8, qkb));
    ECK(cudaMemsetAsync(r.q8, 0, qkb, r.st));   // padded key / query rows stay zero forever
    ECK(cudaMemsetAsync(r.k8, 0, qkb, r.st));
    ECK(cudaMemsetAsync(r.v8, 0, qkb, r.st));
    ECK(cudaMalloc(&r.h8, (size_t)rows * HIDP));
    ECK(cudaMalloc(&r.stat, (size_t)NSTAT * rows * sizeof(float2)));
    ECK(cudaMalloc(&r.pool, (size_t)nb * D * 4));
    ECK(cudaMalloc(&r.pn, (size_t)nb * D * 2));
    ECK(cudaMalloc(&r.pn8, (size_t)nb * D));
    ECK(cudaMalloc(&r.out, (size_t)nb * nt * 4));
    ECK(cudaMemsetAsync(r.x, 0, (size_t)rows * D * 2, r.st));
    ECK(cudaMemsetAsync(r.h, 0, (size_t)rows * D, r.st));
    // TMA operands
    RCK(make_operand(&r.op_in, r.in, nb * NP, K0P * 2, 128));
    RCK(make_operand(&r.op_pe, r.pe, D, K0P * 2, 256));
    RCK(make_operand(&r.op_h, r.h, rows, D, 128));
    RCK(make_operand(&r.op_h8, r.h8, rows, HIDP, 128));
    RCK(make_operand(&r.op_h_sp, r.h, rows, D, SP_BOX_ROWS));
    RCK(make_operand(&r.op_h8_sp, r.h8, rows, HIDP, SP_BOX_ROWS));
    if (im->head8) {
        r.whead.ws = r.hws;
        r.whead.n = (int)nt;
        r.whead.k = D;
        RCK(make_operand(&r.whead.op, r.hw, (int)nt, D, 128));
        RCK(make_operand(&r.op_pn, r.pn8, nb, D, 64));
    } else {
        RCK(make_operand(&r.op_hw, r.hw, (int)nt, D * 2, 128));
        RCK(make_operand(&r.op_pn, r.pn, nb, D * 2, 64));
    }
    RCK(make_attn(&r.attn, r.q8, r.k8, r.v8, nb));
    for (int s = 0; s < EVA_NBUF; s++)
        ECK(cudaEventCreateWithFlags(&r.done[s], cudaEventDisableTiming | cudaEventBlockingSync));
    for (int k = 0; k < 2; k++) {
        ECK(cudaEventCreateWithFlags(&r.in_ready[k], cudaEventDisableTiming));
        ECK(cudaEventCreateWithFlags(&r.in_free[k], cudaEventDisableTiming));
    }
    ECK(cudaHostAlloc((void **)&r.errh, EVA_NBUF * sizeof(uint32_t), cudaHostAllocPortable));
    memset(r.errh, 0, EVA_NBUF * sizeof(uint32_t));
    ECK(cudaStreamSynchronize(r.st));
    // capture the forward once per input buffer
    for (int k = 0; k < 2; k++) {
        RCK(make_operand(&r.op_in, k ? r.in_b : r.in, nb * NP, K0P * 2, 128));
        cudaGraph_t g;
        ECK(cudaStreamBeginCapture(r.st, cudaStreamCaptureModeThreadLocal));
        if (forward(im, r, e, nullptr)) {
            cudaStreamEndCapture(r.st, &g);
            return -1;
        }
        ECK(cudaStreamEndCapture(r.st, &g));
        ECK(cudaGraphInstantiate(k ? &r.graph_b : &r.graph, g, 0));
        ECK(cudaGraphDestroy(g));
        ECK(cudaGraphUpload(k ? r.graph_b : r.graph, r.st));
    }
    RCK(make_operand(&r.op_in, r.in, nb * NP, K0P * 2, 128));  // direct (profiling) forwards read buffer 0
    ECK(cudaStreamSynchronize(r.st));
    return 0;
}

int engine_up(eva *e)
{
    Impl *im = I(e);
    // weights -> pinned host memory once (every replica copies from it)
    FILE *f = fopen(im->path.c_str(), "rb");
    if (!f) {
        fprintf(stderr, "eva: cannot open %s\n", im->path.c_str());
        return -1;
    }
    uint8_t *blob = nullptr;
    ECK(cudaSetDevice(im->devices[0]));
    ECK(cudaHostAlloc((void **)&blob, im->wbytes, cudaHostAllocPortable));
    bool ok = fseek(f, 256, SEEK_SET) == 0 && fread(blob, 1, im->wbytes, f) == im->wbytes;
    fclose(f);
    if (!ok) {
        fprintf(stderr, "eva: cannot stream weights from %s\n", im->path.c_str());
        cudaFreeHost(blob);
        return -1;
    }
    if (im->head8) {
        // host copy of the head block scales (eva_head_put quantises with them); the blocks of extra rows take
        // the largest scale of the file's head
        const HeadOff ho = head_offsets(im, e->ntp);
        const size_t nsb0 = (e->ntp + 127) / 128, nsb = ((size_t)e->nt + 127) / 128;
        const float *hs = (const float *)(blob + ho.hws);
        im->hws_host.assign(hs, hs + nsb0 * 8);
        float mx = 0.f;
        for (float v : im->hws_host) mx = v > mx ? v : mx;
        im->hws_host.resize(std::max(nsb, nsb0) * 8, mx);
    }
    int rc = 0;
    for (size_t i = 0; i < im->reps.size() && !rc; i++) rc = replica_up(im, im->reps[i], e, blob);
    cudaFreeHost(blob);
    if (rc) return -1;
    // host buffers page-locked in place (portable: every device DMAs from / to them)
    for (int s = 0; s < EVA_NBUF; s++) {
        ECK(cudaHostRegister(e->hout[s], (((size_t)e->nb * e->nt * 4) + 4095) & ~(size_t)4095, cudaHostRegisterPortable));
        if (e->hpn[s]) ECK(cudaHostRegister(e->hpn[s], (size_t)e->nb * D * 2, cudaHostRegisterPortable));
    }
    im->out_reg = true;
    if (im->ipool && im->ipoolb) {
        ECK(cudaHostRegister(im->ipool, im->ipoolb, cudaHostRegisterPortable));
        im->pool_reg = true;
    }
    return 0;
}

// Contiguous shard of n inputs for replica i: [*off, *off + *cnt).
void shard(Impl *im, uint32_t n, size_t i, uint32_t *off, uint32_t *cnt)
{
    uint32_t o = 0;
    for (size_t j = 0; j < im->reps.size(); j++) {
        const uint32_t c = std::min<uint32_t>((uint32_t)im->reps[j].nb, n > o ? n - o : 0);
        if (j == i) {
            *off = o;
            *cnt = c;
            return;
        }
        o += c;
    }
    *off = o;
    *cnt = 0;
}

int open_common(eva *e, const char *weights, const std::vector<int> &devs, uint32_t nb, void *pool, size_t poolb,
                uint32_t extra)
{
    memset(e, 0, sizeof(*e));
    FILE *f = fopen(weights, "rb");
    uint32_t hdr[6] = {0, 0, 0, 0, 0, 0};
    if (!f || fread(hdr, 4, 6, f) != 6 || memcmp(hdr, "EVA2", 4) || (hdr[1] != 3 && hdr[1] != 4)) {
        fprintf(stderr, "eva: %s is not an eva02.bin v3 / v4\n", weights);
        if (f) fclose(f);
        return -1;
    }
    Impl *im = new Impl();
    im->ver = (int)hdr[1];
    im->nl = im->ver == 4 && hdr[4] ? (int)hdr[4] : 24;
    im->head8 = im->ver == 4 && (hdr[5] & 1);
    im->table.resize((size_t)im->nl * 12);
    if (fseek(f, 256, SEEK_SET) || fread(im->table.data(), 4, im->table.size(), f) != im->table.size()) {
        fprintf(stderr, "eva: %s: cannot read the scale table\n", weights);
        fclose(f);
        delete im;
        return -1;
    }
    fclose(f);
    for (float v : im->table)
        if (!std::isfinite(v)) {
            fprintf(stderr, "eva: %s: non-finite scale table\n", weights);
            delete im;
            return -1;
        }
    e->impl = im;
    im->path = weights;
    im->wbytes = hdr[3];
    im->devices = devs;
    im->ipool = pool;
    im->ipoolb = poolb;
    im->extra = extra;
    e->nt0 = hdr[2];
    e->nt = hdr[2] + extra;
    e->ntp = (hdr[2] + 7) & ~7u;
    e->nb = nb;
    const size_t ndev = devs.size();
    im->reps.resize(ndev);
    for (size_t i = 0; i < ndev; i++) {
        im->reps[i].dev = devs[i];
        im->reps[i].nb = (int)((nb + ndev - 1 - i) / ndev);  // contiguous shards, sizes differ by at most 1
    }
    for (int s = 0; s < EVA_NBUF; s++) {
        e->hout[s] = (float *)aligned_alloc(4096, (((size_t)nb * e->nt * 4) + 4095) & ~(size_t)4095);
        if (extra && e->hout[s])
            e->hpn[s] = (uint16_t *)aligned_alloc(4096, (((size_t)nb * D * 2) + 4095) & ~(size_t)4095);
        if (!e->hout[s] || (extra && !e->hpn[s])) {
            fprintf(stderr, "eva: out of host memory for the score slots\n");
            for (int t = 0; t <= s; t++) {
                free(e->hout[t]);
                free(e->hpn[t]);
            }
            delete im;
            memset(e, 0, sizeof(*e));
            return -1;
        }
    }
    im->bstatus = -1;
    im->boot_running = true;
    im->boot = std::thread([e]() {
        Impl *p = I(e);
        p->bstatus = engine_up(e);
    });
    return 0;
}

int read_head_adq(eva *e)
{
    Impl *im = I(e);
    if (!im->head8) return 0;
    const HeadOff ho = head_offsets(im, e->ntp);
    FILE *f = fopen(im->path.c_str(), "rb");
    float v = 0.f;
    const bool ok = f && fseek(f, 256 + (long)ho.hsc, SEEK_SET) == 0 && fread(&v, 4, 1, f) == 1;
    if (f) fclose(f);
    if (!ok || !(v > 0.f) || !std::isfinite(v)) {
        fprintf(stderr, "eva: %s: bad FP8 head scale\n", im->path.c_str());
        return -1;
    }
    im->head_adq = v;
    return 0;
}

}  // namespace

extern "C" {

int eva_open(eva *e, const char *weights, int device, void *pool, size_t poolb, uint32_t extra)
{
    return eva_open_ex(e, weights, &device, 1, EVA_NB, pool, poolb, extra);
}

int eva_open_ex(eva *e, const char *weights, const int *devices, int ndev, uint32_t nb, void *pool, size_t poolb,
                uint32_t extra)
{
    std::vector<int> devs;
    if (ndev < 0 || !devices) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
            memset(e, 0, sizeof(*e));
            fprintf(stderr, "eva: no CUDA device\n");
            return -1;
        }
        for (int i = 0; i < n && i < EVA_MAXDEV; i++) devs.push_back(i);
    } else {
        if (ndev == 0 || ndev > EVA_MAXDEV) {
            memset(e, 0, sizeof(*e));
            fprintf(stderr, "eva: bad device count %d\n", ndev);
            return -1;
        }
        devs.assign(devices, devices + ndev);
    }
    if (!nb) nb = EVA_NB;
    if (nb < devs.size()) {
        memset(e, 0, sizeof(*e));
        fprintf(stderr, "eva: batch %u smaller than the device count %zu\n", nb, devs.size());
        return -1;
    }
    if (open_common(e, weights, devs, nb, pool, poolb, extra)) return -1;
    if (read_head_adq(e)) {
        eva_ready(e);
        return -1;
    }
    return 0;
}

int eva_ready(eva *e)
{
    Impl *im = I(e);
    if (!im) return -1;
    if (im->up) return 0;
    if (im->boot_running) {
        im->boot.join();
        im->boot_running = false;
    }
    if (im->bstatus) return -1;
    if (cudaSetDevice(im->devices[0]) != cudaSuccess) return -1;
    im->up = true;
    return 0;
}

int eva_poll(eva *e)
{
    Impl *im = I(e);
    if (!im) return 0;
    return im->up || im->bstatus == 0 ? 1 : (im->boot_running ? 0 : 1);
}

int eva_submit(eva *e, uint32_t buf, uint16_t *const *in, uint32_t n)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    if (buf >= EVA_NBUF || n > e->nb) {
        fprintf(stderr, "eva: submit slot %u / %u inputs out of range\n", buf, n);
        return -1;
    }
    for (size_t i = 0; i < im->reps.size(); i++) {
        Replica &r = im->reps[i];
        uint32_t off, cnt;
        shard(im, n, i, &off, &cnt);
        ECK(cudaSetDevice(r.dev));
        if (cnt) {
            // inputs on the copy stream into the buffer the forward before last has finished reading, so they
            // overlap the previous submit's forward
            const int k = r.ib;
            r.ib ^= 1;
            __half *dst = k ? r.in_b : r.in;
            ECK(cudaStreamWaitEvent(r.cst, r.in_free[k], 0));
            for (uint32_t a = 0, b; a < cnt; a = b) {  // runs of adjacent pool inputs go in one copy
                for (b = a + 1; b < cnt && in[off + b] == in[off + b - 1] + EVA_IN; b++) {
                }
                ECK(cudaMemcpyAsync(dst + (size_t)a * EVA_IN, in[off + a], (size_t)(b - a) * EVA_IN * 2,
                                    cudaMemcpyHostToDevice, r.cst));
            }
            ECK(cudaEventRecord(r.in_ready[k], r.cst));
            ECK(cudaStreamWaitEvent(r.st, r.in_ready[k], 0));
            ECK(cudaGraphLaunch(k ? r.graph_b : r.graph, r.st));
            ECK(cudaEventRecord(r.in_free[k], r.st));
            ECK(cudaMemcpyAsync(e->hout[buf] + (size_t)off * e->nt, r.out, (size_t)cnt * e->nt * 4,
                                cudaMemcpyDeviceToHost, r.st));
            if (e->hpn[buf])
                ECK(cudaMemcpyAsync(e->hpn[buf] + (size_t)off * D, r.pn, (size_t)cnt * D * 2, cudaMemcpyDeviceToHost,
                                    r.st));
        }
        // the device error word after this forward (a bounded wait that ran out invalidates the batch)
        ECK(cudaMemcpyAsync(r.errh + buf, error_word(r.dev), 4, cudaMemcpyDeviceToHost, r.st));
        ECK(cudaEventRecord(r.done[buf], r.st));
    }
    return 0;
}

int eva_query(eva *e, uint32_t buf)
{
    Impl *im = I(e);
    if (!im || !im->up || buf >= EVA_NBUF) return 1;
    for (Replica &r : im->reps) {
        cudaSetDevice(r.dev);
        if (cudaEventQuery(r.done[buf]) == cudaErrorNotReady) return 0;
    }
    return 1;
}

const float *eva_wait(eva *e, uint32_t buf)
{
    Impl *im = I(e);
    if (!im || !im->up || buf >= EVA_NBUF) return nullptr;
    for (Replica &r : im->reps) {
        cudaSetDevice(r.dev);
        if (cudaEventSynchronize(r.done[buf]) != cudaSuccess) return nullptr;
        if (r.errh[buf]) {
            fprintf(stderr, "eva: device %d: a kernel's bounded wait ran out (error bits 0x%x); slot %u is invalid "
                            "(xtb_error_clear resets the device's error word)\n", r.dev, r.errh[buf], buf);
            return nullptr;
        }
    }
    return e->hout[buf];
}

int eva_head_put(eva *e, uint32_t j, const uint16_t *w, float bias)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    if (j >= e->nt) {
        fprintf(stderr, "eva: head row %u out of range (%u tags)\n", j, e->nt);
        return -1;
    }
    std::vector<uint8_t> q;
    const void *src = w;
    size_t rowb = (size_t)D * 2;
    if (im->head8) {
        // quantise with the row block's scales (saturating, like every E4M3 conversion of this library)
        q.resize(D);
        const float *s = &im->hws_host[(size_t)(j / 128) * 8];
        for (int k = 0; k < D; k++) {
            __half_raw hr;
            hr.x = w[k];
            const float v = __half2float(__half(hr)) / s[k / 128];
            q[k] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
        }
        src = q.data();
        rowb = D;
    }
    for (Replica &r : im->reps) {
        ECK(cudaSetDevice(r.dev));
        ECK(cudaMemcpyAsync(r.hw + (size_t)j * rowb, src, rowb, cudaMemcpyHostToDevice, r.st));
        ECK(cudaMemcpyAsync(r.hb + j, &bias, 4, cudaMemcpyHostToDevice, r.st));
    }
    return 0;
}

int eva_head_get(eva *e, uint16_t *w, float *bias)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    Replica &r = im->reps[0];
    ECK(cudaSetDevice(r.dev));
    ECK(cudaStreamSynchronize(r.st));
    if (im->head8) {
        std::vector<uint8_t> q((size_t)e->nt0 * D);
        ECK(cudaMemcpy(q.data(), r.hw0, q.size(), cudaMemcpyDeviceToHost));
        for (uint32_t j = 0; j < e->nt0; j++)
            for (int k = 0; k < D; k++) {
                __nv_fp8_e4m3 f;
                f.__x = q[(size_t)j * D + k];
                const __half h = __float2half_rn((float)f * im->hws_host[(size_t)(j / 128) * 8 + k / 128]);
                w[(size_t)j * D + k] = __half_raw(h).x;
            }
    } else {
        ECK(cudaMemcpy(w, r.hw0, (size_t)e->nt0 * D * 2, cudaMemcpyDeviceToHost));
    }
    ECK(cudaMemcpy(bias, r.hb0, (size_t)e->nt0 * 4, cudaMemcpyDeviceToHost));
    return 0;
}

void eva_close(eva *e)
{
    Impl *im = I(e);
    if (!im) return;
    if (im->boot_running) {
        im->boot.join();
        im->boot_running = false;
    }
    for (Replica &r : im->reps) {
        if (cudaSetDevice(r.dev) != cudaSuccess) continue;
        if (r.st) cudaStreamSynchronize(r.st);
        if (r.cst) cudaStreamSynchronize(r.cst);
        if (r.ast) cudaStreamSynchronize(r.ast);
        if (r.graph) cudaGraphExecDestroy(r.graph);
        if (r.graph_b) cudaGraphExecDestroy(r.graph_b);
        for (int s = 0; s < EVA_NBUF; s++)
            if (r.done[s]) cudaEventDestroy(r.done[s]);
        for (int k = 0; k < 2; k++) {
            if (r.in_ready[k]) cudaEventDestroy(r.in_ready[k]);
            if (r.in_free[k]) cudaEventDestroy(r.in_free[k]);
        }
        void *bufs[] = {r.in, r.in_b, r.x, r.h, r.q8, r.k8, r.v8, r.h8, r.stat, r.pool, r.pn, r.pn8, r.out, r.wts, r.sexp, r.spw,
                        r.sfimg};
        for (void *p : bufs)
            if (p) cudaFree(p);
        if (r.errh) cudaFreeHost(r.errh);
        if (r.head_copy) {
            cudaFree(r.hw);
            cudaFree(r.hb);
            if (im->head8) cudaFree(r.hws);
        }
        if (r.afork) cudaEventDestroy(r.afork);
        if (r.ajoin) cudaEventDestroy(r.ajoin);
        if (r.st) cudaStreamDestroy(r.st);
        if (r.cst) cudaStreamDestroy(r.cst);
        if (r.ast) cudaStreamDestroy(r.ast);
    }
    for (int s = 0; s < EVA_NBUF; s++) {
        if (im->out_reg) {
            cudaHostUnregister(e->hout[s]);
            if (e->hpn[s]) cudaHostUnregister(e->hpn[s]);
        }
        free(e->hout[s]);
        free(e->hpn[s]);
    }
    if (im->pool_reg) cudaHostUnregister(im->ipool);
    delete im;
    memset(e, 0, sizeof(*e));
}

int eva_forward_resident(eva *e)
{
    if (eva_ready(e)) return -1;
    for (Replica &r : I(e)->reps) {
        ECK(cudaSetDevice(r.dev));
        ECK(cudaGraphLaunch(r.graph, r.st));
    }
    return 0;
}

int eva_upload(eva *e, uint16_t *const *in, uint32_t n)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    if (n > e->nb) return -1;
    for (size_t i = 0; i < im->reps.size(); i++) {
        Replica &r = im->reps[i];
        uint32_t off, cnt;
        shard(im, n, i, &off, &cnt);
        ECK(cudaSetDevice(r.dev));
        for (uint32_t a = 0; a < cnt; a++)
            ECK(cudaMemcpyAsync(r.in + (size_t)a * EVA_IN, in[off + a], EVA_IN * 2, cudaMemcpyHostToDevice, r.st));
        ECK(cudaStreamSynchronize(r.st));
    }
    return 0;
}

int eva_download(eva *e, float *out, uint32_t n)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    if (n > e->nb) return -1;
    for (size_t i = 0; i < im->reps.size(); i++) {
        Replica &r = im->reps[i];
        uint32_t off, cnt;
        shard(im, n, i, &off, &cnt);
        ECK(cudaSetDevice(r.dev));
        ECK(cudaStreamSynchronize(r.st));
        if (cnt) ECK(cudaMemcpy(out + (size_t)off * e->nt, r.out, (size_t)cnt * e->nt * 4, cudaMemcpyDeviceToHost));
    }
    return 0;
}

void *eva_stream(eva *e, int i)
{
    Impl *im = I(e);
    if (!im || eva_ready(e) || i < 0 || (size_t)i >= im->reps.size()) return nullptr;
    return (void *)im->reps[i].st;
}

void *eva_input(eva *e, int i)
{
    Impl *im = I(e);
    if (!im || eva_ready(e) || i < 0 || (size_t)i >= im->reps.size()) return nullptr;
    return (void *)im->reps[i].in;
}

void *eva_output(eva *e, int i)
{
    Impl *im = I(e);
    if (!im || eva_ready(e) || i < 0 || (size_t)i >= im->reps.size()) return nullptr;
    return (void *)im->reps[i].out;
}

int eva_block_scale_kinds(eva *e)
{
    Impl *im = I(e);
    if (!im || eva_ready(e) || im->reps[0].L.empty()) return 0;
    int m = 0;
    for (int g = 0; g < NG; g++)
        if (im->reps[0].L[0].w[g].sf) m |= 1 << g;
    return m;
}

int eva_sparse_kinds(eva *e)
{
    if (eva_ready(e)) return -1;
    return I(e)->sp_mask;
}

int eva_launches_per_forward(eva *e)
{
    if (eva_ready(e)) return -1;
    return I(e)->reps[0].launches;
}

int eva_profile(eva *e, float *ms, int kinds)
{
    if (eva_ready(e)) return -1;
    Impl *im = I(e);
    Replica &r = im->reps[0];
    ECK(cudaSetDevice(r.dev));
    for (int w = 0; w < 2; w++)
        if (forward(im, r, e, nullptr)) return -1;  // warm
    Prof p;
    if (forward(im, r, e, &p)) return -1;
    ECK(cudaStreamSynchronize(r.st));
    for (int k = 0; k < kinds; k++) ms[k] = 0.f;
    for (size_t i = 1; i < p.ev.size(); i++) {
        float dt = 0.f;
        cudaEventElapsedTime(&dt, p.ev[i - 1], p.ev[i]);
        if (p.kind[i] >= 0 && p.kind[i] < kinds) ms[p.kind[i]] += dt;
    }
    for (cudaEvent_t ev : p.ev) cudaEventDestroy(ev);
    return P_KINDS;
}

const char *eva_prof_name(int kind) { return kind >= 0 && kind < P_KINDS ? prof_names[kind] : nullptr; }

}  // extern "C"

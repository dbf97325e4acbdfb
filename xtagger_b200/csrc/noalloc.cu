// fc2 (with the folded MLP LayerNorm) without any device allocation.
//
// Some callers cannot let a library allocate device memory: a host application that hands out all GPU memory
// from its own fixed arena and accounts for every byte, a caller on a latency-critical path that cannot afford
// cudaMalloc's implicit device-wide synchronisation, or one that must not fail on an out-of-memory at run time
// after start-up. xtb_fc2 needs device scratch beyond its inputs and outputs -- the per-row (mean, rstd) of the
// SwiGLU output, which it writes over the caller's fc1 partials. xtb_fc2_noalloc keeps that scratch in a
// file-scope static device array of fixed size instead, and leaves the caller's fc1 partials untouched.
//
// Failures: a bounded wait inside the GEMM that runs out sets a bit of the library's error word of the device,
// read with xtb_error_word() (which allocates nothing either: the error words are a static device array too) and
// cleared with xtb_error_clear().
//
// Limits and sharing: at most XTB_NOALLOC_MAX_ROWS rows (16 images of 1025 tokens; 131 KB of row statistics).
// Every GPU that loads the library holds the array until the process exits. All calls on a device share it and it
// keeps the last call's contents: every call rewrites the statistics of all the rows it uses before reading them.
// Calls whose work overlaps on the GPU (different streams, or host threads racing on one device) race on the array
// and must be serialised by the caller.
//
// Set-up: the first call on a device, with that device current, looks up the array's device address
// (cudaGetSymbolAddress), and the GEMM launcher sets its kernel's shared-memory attribute and reads how many CTAs
// fit; that first call should come before any stream capture.
#include <mutex>

#include "../../include/xtagger_b200.h"
#include "epilogues.cuh"
#include "host.h"
#include "ops.h"

using namespace xtb;

namespace {

struct NoAllocScratch {
    float2 ms[XTB_NOALLOC_MAX_ROWS];          // per-row (mean, rstd) over the 2730 SwiGLU units
};

// In host code this name is only a stand-in for the device object: host code uses the address returned by
// cudaGetSymbolAddress for the current device, never the name itself.
static __device__ __align__(256) NoAllocScratch g_noalloc;

// (mean, rstd) of every row from fc1's NSTAT partials into ms, four threads per row in the fixed order of k_rowstat
// (the same rowstat_of), so that the result is bit-identical to xtb_fc2's.
__global__ void __launch_bounds__(ROWSTAT_THREADS) k_rowstat_into(const float2 *__restrict__ stat, float2 *__restrict__ ms,
                                                                  int rows)
{
    const int t = blockIdx.x * ROWSTAT_THREADS + threadIdx.x, row = t >> 2;
    const float2 v = rowstat_of(stat, rows, row, t & 3);
    if ((t & 3) == 0 && row < rows) ms[row] = v;
}

struct DeviceScratch {
    bool ready = false;
    NoAllocScratch *ptr = nullptr;
};
std::mutex g_mu;
DeviceScratch g_dev[64];

// Once per device, with the device current: the array's device address. (The GEMM launcher sets its kernel's
// shared-memory attribute itself on first use, without allocating.)
int setup(int dev, NoAllocScratch **out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 0 || dev >= 64) {
        fprintf(stderr, "eva: xtb_fc2_noalloc: device %d out of range\n", dev);
        return -1;
    }
    DeviceScratch &d = g_dev[dev];
    if (!d.ready) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc);
        if (e != cudaSuccess || !p) {
            fprintf(stderr, "eva: xtb_fc2_noalloc: cudaGetSymbolAddress: %s\n", cudaGetErrorString(e));
            return -1;
        }
        d.ptr = (NoAllocScratch *)p;
        d.ready = true;
    }
    *out = d.ptr;
    return 0;
}

}  // namespace

extern "C" int xtb_fc2_noalloc(const uint8_t *h8, int rows, const uint8_t *w, const float *ws, float ascale, uint16_t *x,
                               const float *stat, const float *c, const float *d, void *stream)
{
    if (rows <= 0 || rows > XTB_NOALLOC_MAX_ROWS) {
        fprintf(stderr, "eva: xtb_fc2_noalloc: %d rows; the static scratch holds 1..%d rows (16 images)\n", rows,
                XTB_NOALLOC_MAX_ROWS);
        return -1;
    }
    int dev = 0;
    XTB_CK(cudaGetDevice(&dev));
    NoAllocScratch *sc = nullptr;
    if (setup(dev, &sc)) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    Operand A;
    Weight8 W;
    CUtensorMap xm;
    W.ws = ws;
    W.n = D;
    W.k = HIDP;
    if (make_operand(&A, h8, rows, HIDP, A_BOX_ROWS) || make_operand(&W.op, w, D, HIDP, weight_box_rows(W_FC2)) ||
        resid_map(&xm, (__half *)x, rows))
        return -1;
    uint32_t *err = error_word(dev);
    if (!err) return -1;
    k_rowstat_into<<<rowstat_blocks(rows), ROWSTAT_THREADS, 0, st>>>((const float2 *)stat, sc->ms, rows);
    XTB_CK(cudaGetLastError());
    if (launch_fc2_gemm(A, W, ascale, rows, xm, sc->ms, nullptr, c, d, err, st)) return -1;
    return 0;
}

#include <cudaTypedefs.h>
#include <map>
#include <mutex>
#include "host.h"

namespace xtb {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static void load_encode()
{
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
}

int make_tmap_2d_typed(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                       uint64_t pitch, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz)
{
    std::call_once(g_encode_once, load_encode);
    if (!g_encode) {
        fprintf(stderr, "eva: cuTensorMapEncodeTiled is not available from the driver\n");
        return -1;
    }
    if (((uintptr_t)base & 15) || (pitch & 15)) {
        fprintf(stderr, "eva: tensor map base / pitch not 16-byte aligned (%p, %llu)\n", base, (unsigned long long)pitch);
        return -1;
    }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, dt, 2, (void *)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "eva: cuTensorMapEncodeTiled failed (%d): cols %llu rows %llu pitch %llu box %ux%u\n", (int)r,
                (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)pitch, box_cols, box_rows);
        return -1;
    }
    return 0;
}

int make_tmap_2d(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t pitch, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swz)
{
    return make_tmap_2d_typed(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, cols, rows, pitch, box_cols, box_rows, swz);
}

int num_sms(int device)
{
    static int cache[64];
    if (device < 0 || device >= 64) return 148;
    if (!cache[device]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
        cache[device] = n;
    }
    return cache[device];
}

int max_pairs(const void *kern, int threads, size_t smem)
{
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({kern, dev});
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(dev), 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        fprintf(stderr, "eva: cudaOccupancyMaxActiveClusters failed on device %d\n", dev);
        return 0;
    }
    cache[{kern, dev}] = n;
    return n;
}

// The error words live in a static device array (zero when the library's code is loaded on a device), so that no
// entry point allocates device memory for them. In host code the name is only a stand-in for the device object:
// kernels get the address cudaGetSymbolAddress returns for the device, looked up once per device.
static __device__ __align__(256) uint32_t g_error_words[64];

uint32_t *error_word(int device)
{
    static uint32_t *words[64];
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (device < 0 || device >= 64) return nullptr;
    if (!words[device]) {
        int prev = 0;
        if (cudaGetDevice(&prev) != cudaSuccess) return nullptr;
        void *p = nullptr;
        if (cudaSetDevice(device) == cudaSuccess && cudaGetSymbolAddress(&p, g_error_words) == cudaSuccess)
            words[device] = (uint32_t *)p;
        else
            fprintf(stderr, "eva: cannot look up the error word on device %d\n", device);
        cudaSetDevice(prev);
    }
    return words[device];
}

}  // namespace xtb

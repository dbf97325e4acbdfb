// Host-side helpers shared by the launchers and the engine: error reporting in the engine's "eva: ..." style,
// TMA tensor-map encoding (through the driver entry point, so the library needs no -lcuda), SM count cache.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

namespace xtb {

#define XTB_CK(call)                                                                             \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "eva: %s: %s (%s:%d)\n", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return -1;                                                                           \
        }                                                                                        \
    } while (0)

// 2D byte matrix [rows][cols bytes] (row pitch `pitch` bytes, a multiple of 16) read in boxes of
// box_cols bytes x box_rows rows with the given swizzle. Out-of-range boxes read as zero.
int make_tmap_2d(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t pitch, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swz);
// Same for elements of another type: cols / box_cols in elements, pitch in bytes.
int make_tmap_2d_typed(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                       uint64_t pitch, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

int num_sms(int device);

// Clusters of two CTAs of `kern` (threads, dynamic shared memory) that can be resident at once on the current
// device (cudaOccupancyMaxActiveClusters), cached per (kernel, device); 0 on failure.
int max_pairs(const void *kern, int threads, size_t smem);

// Library error word on the given device (set by kernels whose bounded waits ran out): a static device array, not an
// allocation; its address is looked up on the first call for a device (not a stream operation, but keep that first
// call outside a stream capture, as the engine's bring-up and prepare_kernels() do).
uint32_t *error_word(int device);

}  // namespace xtb

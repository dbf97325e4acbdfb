// Launch harness for the reference's own FP8 flash attention (flash8<1025>, kern_common.cuh:403-543), compiled from
// the reference's header where it lies (oracle/Makefile, target `ref`, output oracle/_ref/libref_attention.so).
// TEST INFRASTRUCTURE ONLY: tests/ load it to pin the oracle's attention restatement, and this library's kernel, to
// the reference's kernel on the same inputs. Nothing in the product loads it.
//
// The including file supplies the model shapes (eva_kernels.cu:6-16 defines the same values before including the
// header). Layouts are converted here, on the host: q / k rows of this library ([img][16][1152][64], zero padding)
// become the reference's [img][16][1088][64] (its k_qkv also permutes the 64 dims of q and k, identically for
// both, which leaves every dot product unchanged, so the harness keeps them in order); v [img][16][1152][64]
// becomes the reference's per-64-key-tile transpose vt8 [img][16][17][64 dims][64 keys] (eva_kernels.cu:111).
#define D 1024
#define T 1025
#define HID 2730
#define HIDP 2736
#define K0 588
#define K0P 592
#define QKV 3072
#define NKT 17
#define SWT 352
#define TP 1088
#define FC1_GM 8
#define EVA_FP8
#include "kern_common.cuh"

#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <vector>

extern "C" __global__ void __launch_bounds__(128, 4) ref_flash(const unsigned char *__restrict__ q8,
                                                              const unsigned char *__restrict__ k8,
                                                              const unsigned char *__restrict__ v8, void *__restrict__ out,
                                                              float sinv, float vo)
{
    flash8<T>(q8, k8, v8, out, sinv, vo);
}

#define CK(x)                                                                                    \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "ref_attention: %s: %s\n", #x, cudaGetErrorString(e_));              \
            return -1;                                                                           \
        }                                                                                        \
    } while (0)

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
    ref_flash<<<dim3(NKT, 16, nimg), 128>>>(dq, dk, dv, dout, sinv, vo);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(out, dout, out_bytes, cudaMemcpyDeviceToHost));
    CK(cudaFree(dq));
    CK(cudaFree(dk));
    CK(cudaFree(dv));
    CK(cudaFree(dout));
    return 0;
}

// Inline-PTX building blocks for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads, tcgen05
// (TMEM allocation, MMA issue/commit, TMEM loads/stores) and the shared-memory / instruction descriptors the
// tensor core consumes. Everything here is written against the public PTX ISA (8.7, sm_100a).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace xtb {

// ---------------------------------------------------------------------------------------------------------------
// Error word shared by every kernel of the library. A wait that runs out of its time budget sets a bit here and the
// kernel winds down instead of spinning forever; the host reads it back after a forward (xtb_error_word()).
// ---------------------------------------------------------------------------------------------------------------
enum : uint32_t {
    XTB_ERR_WAIT_TMA = 1u,      // producer or consumer of the shared-memory ring timed out
    XTB_ERR_WAIT_TMEM = 2u,     // TMEM accumulator hand-off timed out
    XTB_ERR_WAIT_ATTN = 4u,     // attention pipeline timed out
    XTB_ERR_SHAPE = 8u,         // a launch was given a shape the kernel does not support
    XTB_ERR_SELFTEST = 16u,     // the self-test's wait ran out (xtb_selftest_wait)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// The dynamic shared memory block rounded up to 1024 bytes (128B-swizzled TMA tiles and UMMA descriptors want it).
// Pointer arithmetic on the __shared__ array itself, not an integer round trip: the compiler can then still tell that
// every pointer derived from the result is shared memory and address it as such rather than generically.
__device__ __forceinline__ uint8_t *smem_align1024(uint8_t *raw) { return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u); }

// Programmatic dependent launch: the kernels of the forward are launched so that they may start while the previous
// kernel on the stream finishes. Each of them runs its on-chip set-up (barriers, TMEM, descriptor prefetch, constant
// weights) first and then waits here until the previous kernel has completed and its memory is visible, before it
// reads or writes any activation. Without a programmatic predecessor the wait returns at once.
// Once past the wait, the kernel lets the next one launch (griddepcontrol.launch_dependents): that kernel's CTAs are
// placed as SMs free up and run their own set-up, then block in their wait until this kernel has completed. A kernel
// triggers only after its own wait, so at most one kernel ahead is in its set-up; and the trigger takes effect only
// when every CTA of this grid has issued it, so CTAs that wait never keep this grid's CTAs from being placed.
#ifndef XTB_PDL_TRIGGER
#define XTB_PDL_TRIGGER 1
#endif
__device__ __forceinline__ void griddep_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
#if XTB_PDL_TRIGGER
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

__device__ __forceinline__ uint64_t globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Wait for the phase of the given parity to complete. Bounded: after ~2 s of wall time the wait gives up, records
// `code` in the error word and returns false, so that a broken pipeline ends the kernel instead of hanging the GPU.
#ifndef XTB_WAIT_NS
#define XTB_WAIT_NS 2000000000ull
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && globaltimer() - t0 > XTB_WAIT_NS) {
            atomicOr(err, code);
            return false;
        }
    }
}

// The same with the bound given in nanoseconds.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code, uint64_t ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && globaltimer() - t0 > ns) {
            atomicOr(err, code);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (tiled bulk tensor copies, no multicast anywhere in this library)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *m)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)m) : "memory");
}

// 2D tile load: box at (x = inner coordinate, y = row) into shared memory, completion counted on bar in bytes.
// x must be a multiple of 16 bytes' worth of elements (every caller passes multiples of the 128-byte box width).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, uint64_t *bar, int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)m), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 2D tile store / reduce-add (element type from the tensor map) from shared memory, tracked by the issuing
// thread's bulk async-group. Boxes reaching past the tensor are clipped; coordinates are never negative here.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *m, const void *src, int32_t x, int32_t y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)m),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *m, const void *src, int32_t x, int32_t y)
{
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     (uint64_t)m),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completion counted in
// bytes on the mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of every committed group have been read (the buffer may be rewritten)
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16-byte asynchronous global -> shared copy (L2 only), and an arrival on an mbarrier when every cp.async this
// thread issued so far has landed (noinc: the barrier's expected count includes these arrivals).
__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t *bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, TMEM <-> registers
// ---------------------------------------------------------------------------------------------------------------
// Whole warp: allocate ncols (power of two >= 32) TMEM columns, base address written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, both operands K-major. kind::f8f6f4 (E4M3 x E4M3) or kind::f16 (fp16 x fp16).
template <bool F16>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    if (F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrive (once) on bar when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns: thread i of the warp gets TMEM lane (base lane + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v)
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v)
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float *v)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns from registers (raw 32-bit words)
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t *w)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]), "r"(w[9]),
        "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f8f6f4: A (M rows = TMEM lanes, K bytes packed 4 per 32-bit column,
// K-major) read from tensor memory, B from a shared-memory descriptor.
__device__ __forceinline__ void umma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T with A 2:4-sparse along K, kind::f8f6f4 (E4M3): per instruction K = 64
// logical elements, of which A holds the two kept bytes of every group of four (32 bytes per row) and the
// metadata at TMEM column e_tmem (one row per lane, 4 bits per group: in-group index of the first kept element in
// bits 0-1, of the second in bits 2-3; groups in K order, low nibble first; 2 columns per instruction) says where
// they sit. e_tmem must be an even column.
__device__ __forceinline__ void umma_sp(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t e_tmem, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f8f6f4 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared memory -> TMEM: 128 rows of 16 bytes (row i to lane i, 4 consecutive columns), asynchronous, ordered with
// this thread's later tcgen05.mma and tracked by its tcgen05.commit.
__device__ __forceinline__ void tmem_cp_128x128b(uint32_t taddr, uint64_t sdesc_)
{
    asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc_) : "memory");
}

// 32 lanes x 128 bits from shared memory (32 rows of 16 bytes) into the same 32-lane slice of all four lane groups
// (warpx4): four TMEM columns at taddr across the 128 lanes. The copy into a block-scaled MMA's scale factors.
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc_)
{
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc_) : "memory");
}

// D[tmem] (+)= (A[smem] x 2^sfa) (B[smem] x 2^sfb)^T, kind::mxf8f6f4 block-scaled (E4M3 operands, one UE8M0 scale
// per 32 K elements and row, read from tensor memory at sfa / sfb).
__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                        uint32_t sfb, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait with the 32 registers of an earlier tcgen05.ld tied to it, so that no use of them is scheduled before
// it (the loads write their destinations asynchronously).
__device__ __forceinline__ void tmem_wait_ld_regs(float *v)
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15]),
                   "+f"(v[16]), "+f"(v[17]), "+f"(v[18]), "+f"(v[19]), "+f"(v[20]), "+f"(v[21]), "+f"(v[22]),
                   "+f"(v[23]), "+f"(v[24]), "+f"(v[25]), "+f"(v[26]), "+f"(v[27]), "+f"(v[28]), "+f"(v[29]),
                   "+f"(v[30]), "+f"(v[31])
                 :
                 : "memory");
}
// The same with the 16 registers of a tcgen05.ld ... .x16.
__device__ __forceinline__ void tmem_wait_ld_regs16(float *v)
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------------------
// CTA pairs (clusters of two CTAs on the two SMs of a TPC, tcgen05 .cta_group::2). A kernel uses either these
// forms or the .cta_group::1 forms above for all of its tcgen05 instructions, never both.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs (converged warps): release this CTA's prior writes / acquire the peer's.
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address, in the cluster's shared window, of the object at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// Arrive on an mbarrier of either CTA of the cluster (cluster-window address). The default (CTA-scope) forms are
// enough for every hand-off of the pair GEMM: shared-memory tiles are published by the TMA's complete_tx, TMEM
// reads and writes are ordered by the tcgen05 fences around the barrier; cluster-scope acquire / release on these
// barriers made the pair GEMM three times slower.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr)
{
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t caddr, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(caddr), "r"(bytes) : "memory");
}
// 2D tile load into this CTA's shared memory whose completion is counted on an mbarrier of either CTA of the pair
// (cluster-window address). No multicast: each CTA loads only its own tiles.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *m, uint32_t bar_caddr, int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.cta_group::2 [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)m), "r"(bar_caddr), "r"(x), "r"(y)
        : "memory");
}
// One warp in each CTA of the pair, together: allocate / free ncols TMEM columns in both CTAs.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair forms of the block-scaled MMA (issued by rank 0) and of the scale-factor copy into tensor memory (issued by
// rank 0 for both CTAs of the pair).
__device__ __forceinline__ void umma_pair_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                             uint32_t sfb, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}
__device__ __forceinline__ void tmem_cp_pair_32x128b_x4(uint32_t taddr, uint64_t sdesc_)
{
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc_) : "memory");
}
// Pair MMA (issued by rank 0 for both CTAs), E4M3 x E4M3 -> f32: A rows from each CTA's own shared memory, B rows
// from both, D rows of each CTA in its own TMEM; descriptors give the (identical) shared-memory offsets.
__device__ __forceinline__ void umma_pair_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at this shared-memory offset in every CTA of `mask` when the pair MMAs issued so far
// have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar, uint16_t mask)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"(mask)
                 : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand tile written by TMA with a 128-byte (sw = 2) or 64-byte
// (sw = 4) swizzle: rows of `rowb` bytes, 8-row groups `8 * rowb` bytes apart (SBO); LBO unused for swizzled K-major.
// Bits: [0,14) start >> 4, [16,30) LBO >> 4, [32,46) SBO >> 4, [46,48) version 1, [61,64) swizzle mode.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t sbo_bytes, uint32_t swz)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;  // LBO (ignored for swizzled K-major layouts)
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;  // descriptor version for tcgen05
    d |= (uint64_t)(swz & 7u) << 61;
    return d;
}
constexpr uint32_t SWZ_128B = 2, SWZ_64B = 4;

// Descriptor of an MN-major operand tile (rows along K, each row a 64-byte run of MN elements, 64B swizzle): SBO =
// byte distance between 8-row groups along K; LBO (distance between 64-byte column groups along MN) is unused for
// a tile no wider than one swizzle atom and set to the tile's own size.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t saddr, uint32_t sbo_bytes, uint32_t swz)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((8192u >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)(swz & 7u) << 61;
    return d;
}

// Descriptor of an unswizzled tile of 16-byte rows stored back to back (8-row core matrices 128 bytes apart):
// the source of tmem_cp_128x128b.
__device__ __forceinline__ uint64_t sdesc_rows16(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((2048u >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((128u >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

// Instruction descriptor (kind::f8f6f4 with E4M3 operands, or kind::f16 with fp16 operands), fp32 accumulate,
// both operands K-major, M = 128. Bits: [4,6) D format (1 = f32), [7,10) A format, [10,13) B format,
// [15] A major, [16] B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_m128(uint32_t n)
{
    return (1u << 4) | (0u << 7) | (0u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
// Block-scaled kind::mxf8f6f4, M = 128 (E4M3 A and B, K-major, UE8M0 scales: bit 23): B's scale-factor byte id in
// bits 4-5, A's in bits 29-30 (which of the four 32-K scale bytes of a TMEM word an instruction reads).
__host__ __device__ constexpr uint32_t idesc_mx_m128(uint32_t n, uint32_t sfa_id, uint32_t sfb_id)
{
    return ((sfb_id & 3u) << 4) | ((n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) | ((sfa_id & 3u) << 29);
}
// The same for a CTA-pair MMA of M = 256.
__host__ __device__ constexpr uint32_t idesc_mx_m256(uint32_t n, uint32_t sfa_id, uint32_t sfb_id)
{
    return ((sfb_id & 3u) << 4) | ((n >> 3) << 17) | (1u << 23) | ((256u >> 4) << 24) | ((sfa_id & 3u) << 29);
}
// The same with A 2:4-sparse (bit 2; K = 64 logical elements per instruction).
__host__ __device__ constexpr uint32_t idesc_sp_m128(uint32_t n) { return idesc_m128(n) | (1u << 2); }
// The same for a CTA-pair MMA of M = 256 (128 rows per CTA).
__host__ __device__ constexpr uint32_t idesc_m256(uint32_t n)
{
    return (1u << 4) | (0u << 7) | (0u << 10) | ((n >> 3) << 17) | ((256u >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------------------------
// Numeric helpers
// ---------------------------------------------------------------------------------------------------------------
// Two floats -> packed E4M3 pair (round to nearest even, saturate to +-448; a in the low byte).
__device__ __forceinline__ uint32_t e4m3x2(float a, float b)
{
    return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float tanh_fast(float x)
{
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32 pair arithmetic (sm_100: one instruction for two lanes' worth of fp32 work).
__device__ __forceinline__ uint64_t f2_bits(float2 a) { return *reinterpret_cast<uint64_t *>(&a); }
__device__ __forceinline__ float2 bits_f2(uint64_t b) { return *reinterpret_cast<float2 *>(&b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(d);
}

// max(a, b, c) in one instruction (three-operand max.f32, sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred;
    asm volatile("{\n\t.reg .b32 r;\n\t.reg .pred p;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(pred));
    return pred != 0;
}

}  // namespace xtb

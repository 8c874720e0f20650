// Inline-PTX wrappers for the sm_100a features the kernels use: mbarriers,
// TMA tiled loads and stores (each CTA copies for itself only), tcgen05 MMA /
// TMEM, and a
// bounded wait that gives up with an error code instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace mgb {

// Error codes a kernel writes to the engine's device status word.
enum DeviceError : int {
    kErrNone = 0,
    kErrWaitProducer = 1,   // TMA producer gave up waiting for a free stage
    kErrWaitMma = 2,        // MMA issuer gave up waiting for data / TMEM
    kErrWaitEpilogue = 3,   // epilogue gave up waiting for an accumulator
    kErrWaitDrain = 4,      // exit-time drain of in-flight copies timed out
    kErrWaitDep = 5,        // gave up waiting for another CTA's tiles of the previous layer
};

// Every mbarrier wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of parity `parity` to complete.  Returns false (and
// records `code` in *err) if it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// ---- cross-CTA progress (one persistent kernel over several layers) ----

// Release / acquire on a global counter at GPU scope.
__device__ __forceinline__ void red_max_release_gpu(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.max.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Shared-memory add with acquire-release semantics at CTA scope; returns the
// old value.
__device__ __forceinline__ unsigned atom_add_acq_rel_cta(uint32_t addr, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
                 : "=r"(old)
                 : "r"(addr), "r"(v)
                 : "memory");
    return old;
}
// Orders this thread's generic-proxy global accesses with its async-proxy
// (TMA) accesses to global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Waits until *p >= target (acquire).  Returns false (and records `code` in
// *err) if that has not happened within kWaitLimitNs.
__device__ __forceinline__ bool wait_counter(const unsigned* p, unsigned target, int* err,
                                             int code) {
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 8; ++i)
            if (ld_acquire_gpu(p) >= target) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// 16-bit global load cached in L2 only, issued exactly where it is written
// (volatile), so a load meant to run ahead of other work is not sunk next to
// its use by the scheduler.
__device__ __forceinline__ uint16_t ld_cg_u16_early(const uint16_t* p) {
    uint16_t v;
    asm volatile("ld.global.cg.b16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// 16-byte global load cached in L2 only, issued where it is written.
__device__ __forceinline__ uint4 ld_cg_v4_early(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Programmatic dependent launch: let the next kernel in the stream start
// its prologue, and wait until the previous kernel's results are visible.
// Both are no-ops for kernels launched without the programmatic attribute.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Named barrier `id` over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate across the participating threads.
__device__ __forceinline__ bool bar_any(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// 2-D tiled TMA load global -> shared, completion counted on `bar`.
// Coordinates: x = innermost (element index, 16-byte aligned), y = row.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Bulk copy global -> shared of `bytes` (a multiple of 16; both addresses
// 16-byte aligned), completion counted on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst),
        "l"((uint64_t)src), "r"(bytes), "r"(bar)
        : "memory");
}

// Bulk prefetch of [addr, addr + bytes) into L2 (both 16-byte aligned).
__device__ __forceinline__ void prefetch_l2(const void* addr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((uint64_t)addr), "r"(bytes)
                 : "memory");
}

// 2-D tiled TMA store shared -> global (bulk-group completion).  Rows or
// columns outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            (uint64_t)map),
        "r"(src), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// 32-byte global load, L2 only (a whole sector per lane): r[0..7] are the
// eight 32-bit words at p, which must be 32-byte aligned.
__device__ __forceinline__ void ld_cg_v8(const void* p, uint32_t* r) {
    asm volatile("ld.global.cg.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "l"(p));
}

// Waits until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until at most N of the most recently committed bulk groups still
// read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read_n() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---- tcgen05 ---------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 or fp16
// operands, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// Warp-collective load of 32 consecutive fp32 columns for the warp's 32 TMEM
// lanes: thread i receives lane (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr));
}

// As tmem_ld_32cols for 16 columns.
__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// The same wait, naming the registers a tcgen05.ld writes: as far as the
// compiler knows they are produced here, so no use of them can be
// scheduled above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                   "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                   "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
                 :
                 : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes (64 16-bit elements), 8-row
// groups 1024 bytes apart.  Bit layout (tcgen05 matrix descriptor):
// [0,14) start >> 4, [16,30) leading byte offset >> 4 (unused for swizzled
// K-major; 1), [32,46) stride byte offset >> 4, [46,48) version 1,
// [49,52) base offset, [61,64) layout (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3fff);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands
// K-major: [4,6) D format (1 = f32), [7,10) A format, [10,13) B format
// (0 = f16, 1 = bf16), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool bf16) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

}  // namespace mgb

// oxide_tc.cuh -- Blackwell (sm_100a) asynchronous building blocks: mbarriers,
// TMA tile loads, tensor memory (TMEM) and tcgen05 matrix products, as inline
// PTX.  Every wait is bounded: tc_wait() gives up after two seconds and
// reports it, so a kernel built on these can record an error and return
// instead of hanging.
#pragma once

#include <cuda.h>  // CUtensorMap

#include "oxide_common.cuh"

namespace oxide {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarriers -----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Make the initialised barriers visible to the asynchronous proxy (TMA, tcgen05).
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Arrive and add `bytes` to the transaction count the phase waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
// A wait is declared lost after TC_WAIT_NS of wall time (the %globaltimer
// nanosecond clock), far above any legitimate wait (microseconds); the poll
// count is a second bound in case the timer does not advance.
constexpr uint64_t TC_WAIT_NS = 2000000000ull;
constexpr uint32_t TC_WAIT_POLLS = 1u << 30;
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Wait until the phase with `parity` of `bar` completes, or until `abort`
// (shared flag) is raised elsewhere or the time runs out (then raise it).
// Returns false when the wait did not complete.
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < TC_WAIT_POLLS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u) {
            if (*abort) return false;
            if (global_ns() - t0 > TC_WAIT_NS) break;
        }
    }
    *abort = 1;
    return false;
}

// The same bounded wait without the abort flag: for draining copies and
// products still in flight after an abort.
__device__ __forceinline__ bool tc_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < TC_WAIT_POLLS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > TC_WAIT_NS) return false;
    }
    return false;
}
// Warp-uniform bounded wait: lane 0 polls, every lane gets its verdict (so
// the warp stays converged for the .sync.aligned instructions that follow).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = tc_wait(bar, parity, abort) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
// Named barrier 1 over 128 threads (four warps), and the same barrier
// returning the OR of every participant's flag (a uniform decision).
__device__ __forceinline__ void nbar_sync128() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ bool nbar_or128(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v ? 1u : 0u)
        : "memory");
    return r != 0;
}

// ---- TMA -------------------------------------------------------------------------
// 2-D tiled load of the box at element coordinates (x, y) into shared memory,
// completing on `bar` with the box's byte count.  x * element size must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- proxies and tcgen05 ordering ----------------------------------------------------
// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- tensor memory ---------------------------------------------------------------------
// Warp-wide: allocate `ncols` (a power of two >= 32) TMEM columns; the base
// address is written to shared memory at dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Warp-wide: lane i reads 16 consecutive 32-bit columns of TMEM lane
// (lane base of taddr) + i.  The values are valid after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- tcgen05 matrix products ------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 layout): start address, leading and
// stride byte offsets (all >> 4), descriptor version 1, swizzle layout
// (0 none, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)(layout & 7u) << 61);
}
constexpr uint32_t UMMA_SWIZZLE_NONE = 0, UMMA_SWIZZLE_128B = 2;

// Instruction descriptor of kind::f16 with bf16 A and B, f32 accumulation,
// M x N tile; a_mn / b_mn: the operand is MN-major (else K-major).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t m, uint32_t n, bool a_mn, bool b_mn) {
    return (1u << 4)                      // D: f32
           | (1u << 7) | (1u << 10)       // A, B: bf16
           | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((n >> 3) << 17) | ((m >> 4) << 24);
}
// D[tmem] (+)= A . B, issued by one thread for the CTA; accumulate = 0
// overwrites D.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The mbarrier arrives once every tcgen05 operation this thread issued
// before it has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

}  // namespace oxide

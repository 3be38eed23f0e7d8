// oxide_bulk.cuh -- bulk asynchronous global->shared copies (the 1-D form of
// the Tensor Memory Accelerator path, cp.async.bulk) completed on shared
// memory mbarriers, for sm_90+/sm_100a.  No multicast form is used: every
// copy targets only the issuing CTA's own shared memory.
//
// Every wait is bounded by the global nanosecond timer: a wait that runs
// out records OXIDE_DEVERR_TIMEOUT in a device error word and returns false,
// so a kernel never spins forever.
#pragma once

#include <stdint.h>

namespace oxide {

constexpr unsigned OXIDE_DEVERR_TIMEOUT = 1u;
// Budget of one mbarrier wait (ns).  A healthy bulk copy lands in
// microseconds; 4 s means the copy engine or the kernel is broken.
constexpr uint64_t BULK_WAIT_NS = 4000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier shared-memory accesses (generic proxy) before
// later bulk copies (async proxy) into the same buffers.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; on timeout sets *err and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > BULK_WAIT_NS) {
            atomicOr(err, OXIDE_DEVERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Copy `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// memory into this CTA's shared memory; completion is counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

}  // namespace oxide

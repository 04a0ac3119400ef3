// Asynchronous-copy and launch-dependency helpers shared by the sa_b200
// kernels (sm_100a): mbarriers with bounded waits, 1-D bulk copies
// global -> shared memory (never with multicast), programmatic dependent
// launch controls.
#pragma once

#include <stdint.h>

namespace sa {

constexpr uint32_t kWaitLimit = 20000;       // bounded waits: at most kWaitLimit tries ...
constexpr uint32_t kWaitHintNs = 100000;     // ... each suspending the thread for up to 100 us

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Arrival without data: completes the current phase of a count-1 barrier.
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// The thread sleeps until the phase completes or the hint elapses, so a
// waiting warp takes no issue slots from the warps that compute.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}


}  // namespace sa

// tcgen05 / TMEM building blocks shared by the sm_100a tensor-core kernels:
// TMEM allocation, MMA issue with A from TMEM or shared memory, commits to
// mbarriers, TMEM loads and stores, the 128-byte-swizzle K-major shared
// memory descriptor, and a polling mbarrier wait for the short hand-offs
// between the roles of a warp-specialised kernel.
#pragma once

#include <stdint.h>

#include "sa_async.cuh"

namespace sa {

// ---- tcgen05 wrappers ----------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (f32, TMEM) (+)= A (16-bit, TMEM) * B^T (16-bit, shared memory descriptor)
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}

// D (f32, TMEM) (+)= A (16-bit, shared memory descriptor) * B^T (16-bit, shared memory descriptor)
__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile in the 128-byte-swizzle
// canonical layout: rows of 128 B, 8-row groups 1024 B apart (SBO), version 1,
// layout type 2 (SWIZZLE_128B).  The tile base is 1024-byte aligned; a k step
// of 16 elements inside the swizzle atom advances the start address by 32 B.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// One lane of the (converged) warp: the lowest active lane.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n.reg .b32 rx;\n.reg .pred px;\nelect.sync rx|px, 0xffffffff;\nselp.b32 %0, 1, 0, px;\n}\n"
        : "=r"(pred));
    return pred != 0;
}

// One poll of an mbarrier phase (try_wait without a suspend hint: the
// hand-offs between the roles are short).
__device__ __forceinline__ bool um_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t um_clock_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase that also gives up when another role of
// the kernel has aborted (*abort_flag set).  The bound is 2 s of %globaltimer;
// a wait that runs out sets the abort flag and bit 0 of *status.
constexpr uint64_t kTcWaitNs = 2000000000ull;

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status) {
    if (um_try(bar, parity)) return true;
    const uint64_t t0 = um_clock_ns();
    for (uint32_t it = 1;; ++it) {
        if (um_try(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*abort_flag) return false;
            if (um_clock_ns() - t0 > kTcWaitNs) break;
        }
    }
    *abort_flag = 1;
    if (status) atomicOr(status, 1);
    return false;
}

// The same bound, but the waiting thread sleeps (try_wait with a suspend-time
// hint of 10 us; the hardware wakes it when the phase completes), so warps that
// wait long take no issue slots from the warps that compute.
__device__ __forceinline__ bool tc_wait_sleep(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status) {
    // The abort flag and the clock are read every 16th try only: a try often returns well before
    // its hint (each return costs the waiting warp a few issue slots), and a try sleeps 10 us at
    // most, so the bound is still checked every 160 us.
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(10000u)
            : "memory");
        if (ok) return true;
        if ((it & 15) == 0) {
            if (*abort_flag) return false;
            if (it == 0) t0 = um_clock_ns();
            else if (um_clock_ns() - t0 > kTcWaitNs) break;
        }
    }
    *abort_flag = 1;
    if (status) atomicOr(status, 1);
    return false;
}

}  // namespace sa

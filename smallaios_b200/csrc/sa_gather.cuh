// Completion of the head-sharded gather inside the kernel that writes it.
//
// The kernel that stores this rank's attention heads into every rank's
// gathered-output buffer (the decode merge, or the scatter after the generic
// attention) ends with gather_complete(): the last CTA to finish publishes a
// per-step epoch into every peer's signal array over NVLink and waits until
// every peer has published the same epoch into this rank's array.  When it
// returns, every rank's heads are in this rank's buffer, so the kernels that
// follow on the stream may read it; no host barrier and no extra launch.
//
// Memory order: a CTA's peer stores are followed by a barrier and one
// system-scope acquire-release fence before the CTA is counted; the last CTA
// fences again after its count and publishes with st.release.sys; the waiter
// reads with ld.acquire.sys.  The epoch is a
// device-side counter (so a step replayed from a CUDA graph still advances
// it) compared with wrap-around arithmetic.  The wait is bounded by
// %globaltimer: after `timeout_ns` it sets bit 0 of the cache's device
// status word and returns, and the gathered output of that step is not valid.
#pragma once

#include <stdint.h>

#include "sa_internal.h"

namespace sa {

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Called by every thread of every CTA of the launch, after its stores.  Thread 0 of each CTA
// releases the CTA's stores (the barrier orders every thread's stores before its fence, whose
// cumulativity carries them) with an acquire-release fence at system scope before counting the
// CTA; the last CTA's thread 0 fences again to acquire every counted CTA's stores, and its
// publishing threads release the epoch.
__device__ __forceinline__ void gather_complete(const GatherOut &g) {
    __shared__ int s_last;
    __shared__ uint32_t s_epoch;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned nblocks = gridDim.x * gridDim.y * gridDim.z;
        asm volatile("fence.acq_rel.gpu;\n" ::: "memory");  // release: the CTA's stores before its count
        const bool last = atomicAdd(&g.state[0], 1u) == nblocks - 1;
        // acquire every counted CTA's stores: the epoch's st.release.sys below is cumulative over
        // this GPU-scope chain, so it carries all of them to the peers
        if (last) asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
        s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    if (threadIdx.x == 0) {
        g.state[0] = 0;  // the next launch counts its CTAs from zero
        s_epoch = g.state[1] + 1u;
        g.state[1] = s_epoch;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    const int p = threadIdx.x;
    if (p < g.n) {
        st_release_sys(g.sig[p] + g.rank, e);  // this rank's heads are in rank p's buffer
        const uint32_t *mine = g.sig[g.rank] + p;
        const uint64_t t0 = globaltimer_ns();
        while ((int32_t)(ld_acquire_sys(mine) - e) < 0) {  // rank p's heads are in this rank's buffer
            if (globaltimer_ns() - t0 > g.timeout_ns) {
                atomicOr(g.status, 1);
                break;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace sa

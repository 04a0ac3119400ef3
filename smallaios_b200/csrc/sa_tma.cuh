// Tensor-memory-access helpers shared by the sa_b200 kernels (sm_100a): the
// driver's tensor-map encoder (through the runtime's entry-point query, no
// libcuda link) and the 2-D tiled TMA load into this CTA's shared memory
// (never with multicast).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sa_async.cuh"

namespace sa {

// cuTensorMapEncodeTiled, or nullptr when the driver does not provide it.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 2-D tiled TMA load global -> shared (no multicast); x = inner coordinate.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

}  // namespace sa

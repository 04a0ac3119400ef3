// Device helpers shared by the tensor-core decode kernels (sm_100a):
// integer mma.sync wrappers, fragment index maps of the code layouts, the
// fixed-point constants of the q' and P digits, programmatic dependent
// launch controls.
#pragma once

#include <stdint.h>

namespace sa {
namespace dec {

constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kQMax = 8355711.0f;   // 127*65536 + 127*256 + 127
constexpr float kUMax = 16777215.0f;  // 2^24 - 1
constexpr float kLog2UMax = 23.99999991400867f;  // log2(2^24 - 1)

// ---- PTX helpers (mbarrier / bulk copy / PDL helpers are in sa_async.cuh) ----------
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Programmatic dependent launch: let the next kernel of the stream start
// early / wait until the previous kernel has completed and its writes are
// visible (a no-op when the launch carries no programmatic dependency).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Same product with a zero accumulator input (starts a sum without zeroing registers).
__device__ __forceinline__ void mma_u8u8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// ---- fragment layouts ---------------------------------------------------------
// Dimension carried by logical k (0..31) of K-chunk c for quad q in the QK
// A fragment built from one token's packed codes.
template <int BITS, int D>
__device__ __forceinline__ int k_dim(int c, int q, int k) {
    constexpr int KB = D * BITS / 8;
    constexpr int SEG = KB / 4;
    const int hi = k >> 4, e = k & 3;
    if (BITS == 4) return 2 * (q * SEG + 4 * c + e) + hi;
    return q * SEG + 8 * c + 4 * hi + e;
}

// Dimension carried by column `col` of PV n-tile `nt` (B fragment from the
// 4-token interleaved V words; word index 32*(i/4) + 4*col + i%4).
template <int BITS, int D>
__device__ __forceinline__ int v_dim(int nt, int col) {
    if (BITS == 4) {
        const int i = nt >> 1, hi = nt & 1;
        return 2 * (32 * (i >> 2) + 4 * col + (i & 3)) + hi;
    }
    return 32 * (nt >> 2) + 4 * col + (nt & 3);
}

// Inverse of v_dim: n-tile and column of dimension `dim`.
template <int BITS, int D>
__device__ __forceinline__ void v_inv(int dim, int &nt, int &col) {
    if (BITS == 4) {
        const int w = dim >> 1, hi = dim & 1;
        col = (w >> 2) & 7;
        nt = 2 * (4 * (w >> 5) + (w & 3)) + hi;
    } else {
        col = (dim >> 2) & 7;
        nt = 4 * (dim >> 5) + (dim & 3);
    }
}

}  // namespace dec
}  // namespace sa

// Device helpers shared by the tensor-core decode kernels (sm_100a):
// integer mma.sync wrappers, fragment index maps of the code layouts, the
// fixed-point constants of the q' and P digits, programmatic dependent
// launch controls.
#pragma once

#include <stdint.h>

#include <type_traits>

#include "sa_append.cuh"
#include "sa_gather.cuh"

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

// ---- stream-K records and their merge -------------------------------------------
// Warp owning flat chunk f when F chunks are cut into W ranges
// [w*F/W, (w+1)*F/W): the largest w with w*F/W <= f.
__host__ __device__ __forceinline__ int warp_of_chunk(int f, int F, int W) {
    return (int)((((int64_t)f + 1) * W - 1) / F);
}

// Floats of one partial record holding HPR query heads: value sums
// [HPR][D], then R, L, Z of each head (and HPR floats of padding).
template <int D, int HPR>
struct RecGeo {
    static constexpr int REC = HPR * D + 4 * HPR;
    static constexpr int R = HPR * D, L = HPR * D + HPR, Z = HPR * D + 2 * HPR;
};

template <typename T, int D, int HPR>
__device__ __forceinline__ void decode_merge_head(const AttendArgs &a, int ncu, int F, int W, int g, int lane,
                                                  const float (&sgw)[D / 32]);

// Merge of each unit's partial records (one warp per query head), then
// normalisation, inverse rotation and the store.  The records of unit u are
// w_lo + u .. w_hi + u, one per decode warp whose range touched the unit.
// In the head-sharded mode with signal arrays the launch also completes the
// gather (sa_gather.cuh).
template <typename T, int D, int HPR>
__global__ void __launch_bounds__(32 * HPR) decode_merge_kernel(AttendArgs a, int ncu, int F, int W) {
    constexpr int EPL = D / 32;
    const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
    // The next kernel of the stream may be scheduled now; a kernel of this library launched as a
    // programmatic dependent waits for this grid before it reads anything.
    griddep_launch_dependents();
    // signs * 1/sqrt(n) of this unit's KV head: not written by the decode, so read before the wait
    float sgw[EPL];
    {
        const float *sg = a.signs + (int64_t)(blockIdx.x % a.heads) * D + lane * EPL;
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) sgw[rr] = a.wht_scale * sg[rr];
    }
    griddep_wait();  // the decode grid's records
    if (g < a.group) decode_merge_head<T, D, HPR>(a, ncu, F, W, g, lane, sgw);
    if (a.gather.sig[0]) gather_complete(a.gather);  // every rank's heads are in this rank's buffer
}

// One query head's merge (warp g of the unit's CTA).  Up to kMergeBatch
// records (the common case: a unit spans a handful of decode warps) are merged
// with every load issued up front, so the merge costs one L2 round trip.
constexpr int kMergeBatch = 8;

template <typename T, int D, int HPR>
__device__ __forceinline__ void decode_merge_head(const AttendArgs &a, int ncu, int F, int W, int g, int lane,
                                                  const float (&sgw)[D / 32]) {
    using RG = RecGeo<D, HPR>;
    constexpr int EPL = D / 32;
    using VT = typename std::conditional<EPL == 4, float4, float2>::type;
    const int u = blockIdx.x;
    const int w_lo = warp_of_chunk(u * ncu, F, W), w_hi = warp_of_chunk(u * ncu + ncu - 1, F, W);
    const float *base = a.workspace + ((int64_t)u + w_lo) * RG::REC;  // record w_lo + u, then one per warp
    const int nrec = w_hi - w_lo + 1;
    float x[EPL], L = 0.0f, Z = 0.0f;
#pragma unroll
    for (int rr = 0; rr < EPL; rr++) x[rr] = 0.0f;
    if (nrec <= kMergeBatch) {
        float Rm = -INFINITY, Lm = 0.0f, Zm = 0.0f;
        if (lane < nrec) {
            const float *m = base + (int64_t)lane * RG::REC;
            Rm = m[RG::R + g];
            Lm = m[RG::L + g];
            Zm = m[RG::Z + g];
        }
        VT vals[kMergeBatch];
#pragma unroll
        for (int j = 0; j < kMergeBatch; j++) {
            if (j < nrec) vals[j] = *reinterpret_cast<const VT *>(base + (int64_t)j * RG::REC + g * D + lane * EPL);
        }
        const float M = warp_max(Rm);
        const float wt = Rm == -INFINITY ? 0.0f : exp2f(Rm - M);
        L = wt * Lm;
        Z = wt * Zm;
#pragma unroll
        for (int j = 0; j < kMergeBatch; j++) {
            if (j < nrec) {
                const float wj = __shfl_sync(0xffffffffu, wt, j);
                const float *t = reinterpret_cast<const float *>(&vals[j]);
#pragma unroll
                for (int rr = 0; rr < EPL; rr++) x[rr] = fmaf(wj, t[rr], x[rr]);
            }
        }
    } else {
        // lane i handles the meta of records i, i + 32, ...
        float M = -INFINITY;
        for (int i = lane; i < nrec; i += 32) M = fmaxf(M, base[(int64_t)i * RG::REC + RG::R + g]);
        M = warp_max(M);
        for (int i0 = 0; i0 < nrec; i0 += 32) {
            float wt = 0.0f;
            if (i0 + lane < nrec) {
                const float *m = base + (int64_t)(i0 + lane) * RG::REC;
                const float Rw = m[RG::R + g];
                wt = Rw == -INFINITY ? 0.0f : exp2f(Rw - M);
                L = fmaf(wt, m[RG::L + g], L);
                Z = fmaf(wt, m[RG::Z + g], Z);
            }
            const int n = min(32, nrec - i0);
#pragma unroll 8
            for (int j = 0; j < n; j++) {
                const float wj = __shfl_sync(0xffffffffu, wt, j);
                const VT tv = *reinterpret_cast<const VT *>(base + (int64_t)(i0 + j) * RG::REC + g * D + lane * EPL);
                const float *t = reinterpret_cast<const float *>(&tv);
#pragma unroll
                for (int rr = 0; rr < EPL; rr++) x[rr] = fmaf(wj, t[rr], x[rr]);
            }
        }
    }
    L = warp_sum(L);
    Z = warp_sum(Z);
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int rr = 0; rr < EPL; rr++) x[rr] = L > 0.0f ? (x[rr] + Z) * inv : 0.0f;
    warp_wht_butterfly<EPL>(x, lane, D);
    const int h = u % a.heads;
#pragma unroll
    for (int rr = 0; rr < EPL; rr++) x[rr] *= sgw[rr];
    if (a.gather.n == 0) {
        T *dst = static_cast<T *>(a.out) + ((int64_t)u * a.group + g) * D;
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) st_from_f32(dst + lane * EPL + rr, x[rr]);
    } else {
        // head-sharded: row b, global query head col0 + h*G + g of every rank's buffer
        const int64_t b = u / a.heads;
        const int64_t off = (b * a.gather.cols + a.gather.col0 + (int64_t)h * a.group + g) * D + lane * EPL;
        for (int r = 0; r < a.gather.n; r++) {
            T *dst = static_cast<T *>(a.gather.p[r]) + off;
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) st_from_f32(dst + rr, x[rr]);
        }
    }
}

}  // namespace dec
}  // namespace sa

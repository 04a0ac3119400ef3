// Shared device/host helpers for the sa_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sa_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "sa_b200 kernels are written for sm_100a (B200) only"
#endif

namespace sa {

// ---- error reporting (host) ----------------------------------------------
int set_error(int status, const char *fmt, ...);
int check_cuda(cudaError_t e, const char *what);

// ---- dtype access ---------------------------------------------------------
template <typename T> struct DT;
template <> struct DT<float> {
    static __device__ __forceinline__ float to_f32(float v) { return v; }
    static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <> struct DT<__half> {
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};
template <> struct DT<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float ld_f32(const T *p) { return DT<T>::to_f32(*p); }
template <typename T> __device__ __forceinline__ void st_from_f32(T *p, float v) { *p = DT<T>::from_f32(v); }

// ---- exact-rounding scalar helpers matching the reference's Rust ---------
// `x as i32` (saturating, NaN -> 0): cvt.rzi.s32.f32 clamps and maps NaN to 0.
__device__ __forceinline__ float rust_round_f32(float x) {
    // kv_compression.rs:27-37 round_f32: half away from zero via trunc+frac.  Branch-free: tr is
    // never -0 (it comes from an integer), so tr + 0 is tr and tr - 1 is tr + (-1).
    const float tr = __int2float_rn(__float2int_rz(x));
    const float frac = __fsub_rn(x, tr);
    return __fadd_rn(tr, frac >= 0.5f ? 1.0f : (frac <= -0.5f ? -1.0f : 0.0f));
}

// a / b correctly rounded (the value __fdiv_rn returns) from y = RN(1/b), for 2^-90 <= b <= 2^100
// and 2^-100 <= a <= 256 b (or a = 0): every product and residual then stays in the normal range.
// For 0 < a < 2^-100 the quotient is below 2^-10 and the result is within far less than 1/2 of it,
// so a code rounded from it is the same.  Markstein's method (P. Markstein, IBM J. Res. Dev.
// 34(1), 1990): q0 = RN(a*y) is within two ulps of a/b; each step forms the exact residual
// r = a - b*q with an FMA and corrects q to RN(q + r*y).  The first step makes q faithful, and
// from a faithful q and y = RN(1/b) the second returns RN(a/b) (Markstein's theorem).
__device__ __forceinline__ float div_rn_markstein(float a, float b, float y) {
    const float q0 = __fmul_rn(a, y);
    const float r0 = __fmaf_rn(-q0, b, a);
    const float q1 = __fmaf_rn(r0, y, q0);
    const float r1 = __fmaf_rn(-q1, b, a);
    return __fmaf_rn(r1, y, q1);
}

// ---- warp helpers ---------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// In-warp Walsh-Hadamard butterfly over a vector of D = 32*EPL (or D < 32 with
// one element on each of the first D lanes), element e = lane*EPL + r.
// Same stage order (h = 1, 2, 4, ...) and operand order as
// wht_butterfly_normalize (kv_compression.rs:81-107): x[j] = a + b,
// x[j + h] = a - b, all rounded separately.
template <int EPL>
__device__ __forceinline__ void warp_wht_butterfly(float (&x)[EPL], int lane, int d) {
#pragma unroll
    for (int h = 1; h < EPL; h <<= 1) {
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            if ((r & h) == 0) {
                float a = x[r], b = x[r + h];
                x[r] = __fadd_rn(a, b);
                x[r + h] = __fsub_rn(a, b);
            }
        }
    }
    const int lanes_used = d / EPL;  // power of two
    for (int lm = 1; lm < lanes_used; lm <<= 1) {
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            float other = __shfl_xor_sync(0xffffffffu, x[r], lm);
            x[r] = (lane & lm) ? __fsub_rn(other, x[r]) : __fadd_rn(x[r], other);
        }
    }
}

}  // namespace sa

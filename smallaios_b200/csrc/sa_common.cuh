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
    // kv_compression.rs:27-37 round_f32: half away from zero via trunc+frac.
    float tr = __int2float_rn(__float2int_rz(x));
    float frac = __fsub_rn(x, tr);
    if (frac >= 0.5f) return __fadd_rn(tr, 1.0f);
    if (frac <= -0.5f) return __fsub_rn(tr, 1.0f);
    return tr;
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

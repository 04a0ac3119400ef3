// MatMulNBits (ORT com.microsoft.MatMulNBits contract), int4 weights with
// per-(column, k-block) scales and optional packed zero points.
//
// GEMV path (m <= 8 rows per pass): one warp per output column streams that
// column's packed codes with 128-bit loads (16 bytes = 32 codes per lane per
// step) and keeps the activation rows in registers/L1.  The block scale is
// factored out of the inner sum: y = sum_blk s_blk * (sum_k a_k*(q_k - zp)),
// so each code costs one integer extract and one FMA.  HBM-bound: the codes
// and scales are read exactly once.
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kGemvWarps = 8;

template <typename T>
__device__ __forceinline__ float scale_at(const T *s, int64_t i) {
    return DT<T>::to_f32(s[i]);
}

// grid.x covers columns (one warp each); rows [m0, m0 + MT) of A.
template <typename T, int MT>
__global__ void __launch_bounds__(32 * kGemvWarps)
    mnb_gemv_kernel(const T *__restrict__ a, const uint8_t *__restrict__ b, const T *__restrict__ scales,
                    const uint8_t *__restrict__ zps, const T *__restrict__ bias, T *__restrict__ y, int64_t m,
                    int64_t m0, int64_t n, int64_t k, int block_size) {
    const int lane = threadIdx.x & 31;
    const int64_t col = (int64_t)blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (col >= n) return;
    const int64_t nblk = k / block_size;
    const int64_t row_bytes = k / 2;
    const int64_t zp_row = (nblk * 4 + 7) / 8;
    const uint8_t *bcol = b + col * row_bytes;
    float acc[MT];
#pragma unroll
    for (int r = 0; r < MT; r++) acc[r] = 0.0f;

    // Each lane owns 32 consecutive k per step (16 bytes of codes); a block of
    // block_size >= 16 codes spans whole 16-element halves of that chunk.
    for (int64_t k0 = (int64_t)lane * 32; k0 < k; k0 += 32 * 32) {
        const uint4 w = *reinterpret_cast<const uint4 *>(bcol + k0 / 2);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        float part[MT][2];
#pragma unroll
        for (int r = 0; r < MT; r++) part[r][0] = part[r][1] = 0.0f;
        float zf[2];
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int64_t blk = (k0 + hlf * 16) / block_size;
            uint32_t zp = 8u;
            if (zps) {
                const uint8_t zb = zps[col * zp_row + blk / 2];
                zp = (blk & 1) ? (uint32_t)(zb >> 4) : (uint32_t)(zb & 15u);
            }
            zf[hlf] = (float)zp;
        }
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
            const int hlf = wi >> 1;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float qv = (float)((words[wi] >> (4 * j)) & 15u) - zf[hlf];
                const int64_t kk = k0 + wi * 8 + j;
#pragma unroll
                for (int r = 0; r < MT; r++) {
                    if (m0 + r < m) part[r][hlf] += ld_f32(a + (m0 + r) * k + kk) * qv;
                }
            }
        }
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int64_t blk = (k0 + hlf * 16) / block_size;
            const float s = scale_at(scales, col * nblk + blk);
#pragma unroll
            for (int r = 0; r < MT; r++) acc[r] += s * part[r][hlf];
        }
    }
#pragma unroll
    for (int r = 0; r < MT; r++) {
        float v = warp_sum(acc[r]);
        if (lane == 0 && m0 + r < m) {
            if (bias) v += ld_f32(bias + col);
            st_from_f32(y + (m0 + r) * n + col, v);
        }
    }
}

template <typename T>
int launch_t(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, const void *bias, void *y,
             int64_t m, int64_t n, int64_t k, int block_size, cudaStream_t stream) {
    if (k % 32 != 0) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: K must be a multiple of 32");
    if ((reinterpret_cast<uintptr_t>(b) & 15) != 0 || ((k / 2) % 16) != 0)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: packed B rows must be 16-byte aligned");
    const int64_t blocks = (n + kGemvWarps - 1) / kGemvWarps;
    for (int64_t m0 = 0; m0 < m; m0 += 8) {
        const int64_t mt = m - m0;
        dim3 grid((unsigned)blocks), block(32 * kGemvWarps);
        const T *A = static_cast<const T *>(a);
        const T *S = static_cast<const T *>(scales);
        const T *Bi = static_cast<const T *>(bias);
        T *Y = static_cast<T *>(y);
        if (mt == 1)
            mnb_gemv_kernel<T, 1><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else if (mt <= 2)
            mnb_gemv_kernel<T, 2><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else if (mt <= 4)
            mnb_gemv_kernel<T, 4><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else
            mnb_gemv_kernel<T, 8><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        count_launch();
        int rc = check_cuda(cudaGetLastError(), "MatMulNBits gemv launch");
        if (rc != SA_OK) return rc;
    }
    return SA_OK;
}

}  // namespace

int launch_matmul_nbits(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, const void *bias,
                        void *y, int dtype, int64_t m, int64_t n, int64_t k, int block_size, cudaStream_t stream) {
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_t<float>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        case SA_DTYPE_FLOAT16: return launch_t<__half>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        case SA_DTYPE_BFLOAT16:
            return launch_t<__nv_bfloat16>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: dtype %d not supported", dtype);
    }
}

}  // namespace sa

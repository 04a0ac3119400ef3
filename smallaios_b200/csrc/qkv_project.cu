// Epilogue kernel of the fused QKV projection when the projection itself ran
// as separate MatMulNBits launches (the mma.sync / GEMV shapes): one warp per
// (head, row) finishes the head vector (RoPE of q in place, quantize-on-append
// of k and v).  The tcgen05 projection runs the same routine in its own
// epilogue instead (matmul_nbits_umma.cu).
#include "sa_qkv.cuh"

namespace sa {

namespace {

template <typename T, int EPL>
__global__ void __launch_bounds__(32) qkv_finish_kernel(QkvArgs a) {
    __shared__ uint8_t s_codes[256];
    qkv_finish_vector<T, EPL>(a, blockIdx.y, blockIdx.x, threadIdx.x, s_codes);
}

template <typename T>
int launch_t(const QkvArgs &a, cudaStream_t stream) {
    const dim3 grid((unsigned)(a.q_heads + 2 * a.ap.heads), (unsigned)a.ap.batch);
    switch (a.ap.head_dim) {
        case 16: qkv_finish_kernel<T, 1><<<grid, 32, 0, stream>>>(a); break;
        case 32: qkv_finish_kernel<T, 1><<<grid, 32, 0, stream>>>(a); break;
        case 64: qkv_finish_kernel<T, 2><<<grid, 32, 0, stream>>>(a); break;
        case 128: qkv_finish_kernel<T, 4><<<grid, 32, 0, stream>>>(a); break;
        case 256: qkv_finish_kernel<T, 8><<<grid, 32, 0, stream>>>(a); break;
        default: return set_error(SA_ERR_UNSUPPORTED, "qkv_project_append: head_dim %d", a.ap.head_dim);
    }
    count_launch();
    return check_cuda(cudaGetLastError(), "qkv finish launch");
}

}  // namespace

int launch_qkv_finish(const QkvArgs &a, cudaStream_t stream) {
    switch (a.ap.dtype) {
        case SA_DTYPE_FLOAT: return launch_t<float>(a, stream);
        case SA_DTYPE_FLOAT16: return launch_t<__half>(a, stream);
        default: return launch_t<__nv_bfloat16>(a, stream);
    }
}

}  // namespace sa

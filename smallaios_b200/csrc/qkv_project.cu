// Finishing kernel of the fused QKV projection: one warp per (head, row)
// finishes the head vector (RoPE of q in place, quantize-on-append of k and
// v) once the projection (the tcgen05 kernel writing q / k / v directly, or
// three MatMulNBits launches) has stored it.
#include "sa_qkv.cuh"

namespace sa {

namespace {

template <typename T, int EPL>
__global__ void __launch_bounds__(32) qkv_finish_kernel(QkvArgs a) {
    __shared__ uint8_t s_codes[256];
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the projection's outputs (a no-op without PDL)
    qkv_finish_vector<T, EPL>(a, blockIdx.y, blockIdx.x, threadIdx.x, s_codes);
}

// Launched as a programmatic dependent of the projection kernel before it, so
// its warps are resident (and waiting) when the projection completes.
template <typename T>
int launch_t(const QkvArgs &a, cudaStream_t stream) {
    void (*kern)(QkvArgs);
    switch (a.ap.head_dim) {
        case 16:
        case 32: kern = qkv_finish_kernel<T, 1>; break;
        case 64: kern = qkv_finish_kernel<T, 2>; break;
        case 128: kern = qkv_finish_kernel<T, 4>; break;
        case 256: kern = qkv_finish_kernel<T, 8>; break;
        default: return set_error(SA_ERR_UNSUPPORTED, "qkv_project_append: head_dim %d", a.ap.head_dim);
    }
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.q_heads + 2 * a.ap.heads), (unsigned)a.ap.batch);
    cfg.blockDim = dim3(32);
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    count_launch();
    return check_cuda(e, "qkv finish launch");
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

// Quantize-on-append kernel: one warp per (row, token, head, K|V) vector
// (encode_append_vector in sa_append.cuh does the bit-exact work).
#include "sa_append.cuh"

namespace sa {

namespace {

constexpr int kAppendWarps = 4;

template <typename T, int EPL>
__global__ void __launch_bounds__(32 * kAppendWarps) kv_append_kernel(AppendArgs a) {
    __shared__ uint8_t s_codes[kAppendWarps][256];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t vec = (int64_t)blockIdx.x * kAppendWarps + warp;
    const int64_t nvec = (int64_t)a.batch * a.seq_len * a.heads * 2;
    if (vec >= nvec) return;
    const int which = (int)(vec & 1);  // 0 = K, 1 = V
    int64_t rest = vec >> 1;
    const int h = (int)(rest % a.heads);
    rest /= a.heads;
    const int s = (int)(rest % a.seq_len);
    const int b = (int)(rest / a.seq_len);
    encode_append_vector<T, EPL>(a, b, s, h, which, lane, s_codes[warp]);
}

template <typename T>
int launch_t(const AppendArgs &a, cudaStream_t stream) {
    const int64_t nvec = (int64_t)a.batch * a.seq_len * a.heads * 2;
    if (nvec == 0) return SA_OK;
    const int64_t blocks = (nvec + kAppendWarps - 1) / kAppendWarps;
    if (blocks > 0x7fffffff) return set_error(SA_ERR_UNSUPPORTED, "kv_append: too many vectors");
    dim3 grid((unsigned)blocks), block(32 * kAppendWarps);
    switch (a.head_dim) {
        case 16: kv_append_kernel<T, 1><<<grid, block, 0, stream>>>(a); break;
        case 32: kv_append_kernel<T, 1><<<grid, block, 0, stream>>>(a); break;
        case 64: kv_append_kernel<T, 2><<<grid, block, 0, stream>>>(a); break;
        case 128: kv_append_kernel<T, 4><<<grid, block, 0, stream>>>(a); break;
        case 256: kv_append_kernel<T, 8><<<grid, block, 0, stream>>>(a); break;
        default: return set_error(SA_ERR_UNSUPPORTED, "kv_append: head_dim %d not supported", a.head_dim);
    }
    count_launch();
    return check_cuda(cudaGetLastError(), "kv_append launch");
}

}  // namespace

int launch_kv_append(const AppendArgs &a, cudaStream_t stream) {
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_t<float>(a, stream);
        case SA_DTYPE_FLOAT16: return launch_t<__half>(a, stream);
        case SA_DTYPE_BFLOAT16: return launch_t<__nv_bfloat16>(a, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "kv_append: dtype %d not supported", a.dtype);
    }
}

}  // namespace sa

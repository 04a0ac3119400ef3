// Quantize-on-append kernel: one warp per (row, token, head, K|V) vector
// (encode_append_vector in sa_append.cuh does the bit-exact work).
#include "sa_append.cuh"

namespace sa {

namespace {

constexpr int kAppendWarps = 4;

// IDX = uint32_t when every vector index fits 32 bits (the common case: 64-bit division costs
// tens of instructions per warp), else int64_t.
template <typename T, int EPL, typename IDX>
__global__ void __launch_bounds__(32 * kAppendWarps) kv_append_kernel(AppendArgs a) {
    __shared__ uint8_t s_codes[kAppendWarps][256];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const IDX vec = (IDX)blockIdx.x * kAppendWarps + warp;
    const IDX nvec = (IDX)a.batch * a.seq_len * a.heads * 2;
    if (vec >= nvec) return;
    const int which = (int)(vec & 1);  // 0 = K, 1 = V
    IDX rest = vec >> 1;
    const int h = (int)(rest % (IDX)a.heads);
    rest /= (IDX)a.heads;
    const int s = (int)(rest % (IDX)a.seq_len);
    const int b = (int)(rest / (IDX)a.seq_len);
    encode_append_vector<T, EPL>(a, b, s, h, which, lane, s_codes[warp]);
}

template <typename T, int EPL>
void launch_epl(const AppendArgs &a, dim3 grid, dim3 block, bool small, cudaStream_t stream) {
    if (small) kv_append_kernel<T, EPL, uint32_t><<<grid, block, 0, stream>>>(a);
    else kv_append_kernel<T, EPL, int64_t><<<grid, block, 0, stream>>>(a);
}

template <typename T>
int launch_t(const AppendArgs &a, cudaStream_t stream) {
    const int64_t nvec = (int64_t)a.batch * a.seq_len * a.heads * 2;
    if (nvec == 0) return SA_OK;
    const int64_t blocks = (nvec + kAppendWarps - 1) / kAppendWarps;
    if (blocks > 0x7fffffff) return set_error(SA_ERR_UNSUPPORTED, "kv_append: too many vectors");
    dim3 grid((unsigned)blocks), block(32 * kAppendWarps);
    const bool small = blocks * kAppendWarps < ((int64_t)1 << 32);
    switch (a.head_dim) {
        case 16: launch_epl<T, 1>(a, grid, block, small, stream); break;
        case 32: launch_epl<T, 1>(a, grid, block, small, stream); break;
        case 64: launch_epl<T, 2>(a, grid, block, small, stream); break;
        case 128: launch_epl<T, 4>(a, grid, block, small, stream); break;
        case 256: launch_epl<T, 8>(a, grid, block, small, stream); break;
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

// Quantize-on-append: RoPE (K only) + PolarQuant encode + bit packing, one
// warp per (row, token, head, K|V) vector.  Bit-exact with
// PolarQuantizer::encode (kv_compression.rs:216-267) on the f32 value of the
// input: every float operation below is an explicitly rounded intrinsic in
// the reference's order, so nvcc cannot contract or reassociate it.
#include "sa_common.cuh"
#include "sa_internal.h"

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
    const int d = a.head_dim;
    const int64_t pos = a.pos0 + s;
    const bool active = lane * EPL < d;

    const T *src = static_cast<const T *>(which ? a.value : a.key) +
                   (((int64_t)b * a.seq_len + s) * a.heads + h) * d;
    float x[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = active ? ld_f32(src + lane * EPL + r) : 0.0f;

    // RoPE on K (rotate_rope_block, ops/microsoft.rs:137-160): y0 = c*x0 - s*x1,
    // y1 = s*x0 + c*x1, each product rounded before the add.
    if (which == 0 && a.do_rotary && active) {
        const int half = d / 2;
        const float *cr = a.cos_cache + pos * half;
        const float *sr = a.sin_cache + pos * half;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            int pair, partner;
            bool first;
            if (a.interleaved) {
                pair = e >> 1;
                first = (e & 1) == 0;
                partner = first ? e + 1 : e - 1;
            } else {
                first = e < half;
                pair = first ? e : e - half;
                partner = first ? e + half : e - half;
            }
            const float c = cr[pair], sn = sr[pair];
            const float xo = ld_f32(src + partner);
            x[r] = first ? __fsub_rn(__fmul_rn(c, x[r]), __fmul_rn(sn, xo))
                         : __fadd_rn(__fmul_rn(sn, xo), __fmul_rn(c, x[r]));
        }
    }

    // apply_signs + butterfly + 1/sqrt_approx(n) (kv_compression.rs:81-123).
    const float *sg = a.signs + (int64_t)h * d;
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = __fmul_rn(x[r], active ? sg[lane * EPL + r] : 1.0f);
    warp_wht_butterfly<EPL>(x, lane, d);
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = __fmul_rn(x[r], a.wht_scale);

    // min / max with strict comparisons in index order: the first occurrence
    // wins, as in the sequential loop of encode (this matters for +-0).
    float mn = INFINITY, mx = -INFINITY;
    int imn = 0x7fffffff, imx = 0x7fffffff;
    if (active) {
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            if (x[r] < mn) { mn = x[r]; imn = e; }
            if (x[r] > mx) { mx = x[r]; imx = e; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float omn = __shfl_xor_sync(0xffffffffu, mn, o);
        const int oimn = __shfl_xor_sync(0xffffffffu, imn, o);
        const float omx = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oimx = __shfl_xor_sync(0xffffffffu, imx, o);
        if (omn < mn || (omn == mn && oimn < imn)) { mn = omn; imn = oimn; }
        if (omx > mx || (omx == mx && oimx < imx)) { mx = omx; imx = oimx; }
    }

    const uint32_t levels = (1u << a.bits) - 1u;
    const float range = __fsub_rn(mx, mn);
    const float scale = range > 0.0f ? __fdiv_rn(range, (float)levels) : 1.0f;
    const float zp = mn;
#pragma unroll
    for (int r = 0; r < EPL; r++) {
        if (active) {
            uint32_t q = 0u;
            if (scale > 0.0f) q = __float2uint_rz(rust_round_f32(__fdiv_rn(__fsub_rn(x[r], zp), scale)));
            s_codes[warp][lane * EPL + r] = (uint8_t)(q < levels ? q : levels);
        }
    }
    __syncwarp();

    // pack_bits (kv_compression.rs:294-312): LSB-first contiguous bit stream.
    const int cb = a.code_bytes;
    const int64_t row = ((int64_t)b * a.heads + h);
    for (int j = lane; j < cb; j += 32) {
        uint32_t byte = 0;
#pragma unroll
        for (int bit = 0; bit < 8; bit++) {
            const int g = 8 * j + bit;
            const int e = g / a.bits, eb = g % a.bits;
            if (e < d) byte |= ((uint32_t)(s_codes[warp][e] >> eb) & 1u) << bit;
        }
        if (which == 0) {
            a.k_codes[(row * a.capacity + pos) * cb + j] = (uint8_t)byte;
        } else {
            a.v_codes[((row * (a.capacity / kVGroup) + pos / kVGroup) * cb + j) * kVGroup + pos % kVGroup] =
                (uint8_t)byte;
        }
    }
    if (lane == 0) {
        float *meta = (which == 0 ? a.k_meta : a.v_meta) + (row * a.capacity + pos) * 2;
        meta[0] = scale;
        meta[1] = zp;
    }
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

// Quantize-on-append kernels: one warp per (row, KV head, position quad) for the common code
// widths, one warp per (row, token, head, K|V) vector otherwise (polar_encode_warp and
// encode_append_vector in sa_append.cuh do the bit-exact work).
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

// The bulk append, one warp per (row, KV head, position quad): the K and V vectors of the up to
// four appended positions p with the same p >> 2, one after the other.  The (row, head) split,
// the signs and the pointers are set up once for up to eight vectors, and the V codes of a full
// quad leave as 32-bit words: the V layout interleaves the four tokens of a quad byte by byte
// (v_byte_offset), so code byte j of the quad's four tokens is one aligned word.  For 8-bit
// codes, or 4-bit codes with two or more elements per lane, without QJL residuals; other
// appends take kv_append_kernel.
template <typename T, int EPL>
__global__ void __launch_bounds__(32 * kAppendWarps)
    kv_append_quad_kernel(AppendArgs a, uint32_t nquads, uint32_t nwarps) {
    const int lane = threadIdx.x & 31;
    const uint32_t wid = blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
    if (wid >= nwarps) return;
    const uint32_t bh = wid / nquads, qi = wid - bh * nquads;
    const uint32_t b = bh / (uint32_t)a.heads, h = bh - b * (uint32_t)a.heads;
    const int d = a.head_dim;
    const bool active = lane * EPL < d;
    const int64_t qbase = ((a.pos0 >> 2) + qi) * 4;  // first position of the quad
    const int64_t p_lo = qbase > a.pos0 ? qbase : a.pos0;
    const int64_t p_end = a.pos0 + a.seq_len, p_hi = qbase + 4 < p_end ? qbase + 4 : p_end;
    const bool full = p_lo == qbase && p_hi == qbase + 4;
    float sg[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) sg[r] = active ? a.signs[(int64_t)h * d + lane * EPL + r] : 1.0f;
    const uint32_t levels = (1u << a.bits) - 1u;
    const int cb = a.code_bytes, nb = a.bits == 8 ? EPL : EPL / 2;  // code bytes per lane and vector
    const int64_t row = (int64_t)b * a.heads + h;
    const int64_t in_stride = (int64_t)a.heads * d;  // input elements from one token to the next
    const int64_t in0 = ((int64_t)b * a.seq_len + (p_lo - a.pos0)) * in_stride + (int64_t)h * d + lane * EPL;
    uint8_t *vdst = a.v_codes + row * a.capacity * cb;
    uint64_t vword[4] = {0, 0, 0, 0};  // this lane's V code bytes of the quad's tokens
    // K and V inputs of the current position; the next position's are loaded before this one is
    // encoded, so their latency overlaps the work
    float xn[2][EPL];
    auto load_kv = [&](int64_t p, float (&dst)[2][EPL]) {
#pragma unroll
        for (int which = 0; which < 2; which++) {
            if (active && p < p_hi) {
                load_elems<T, EPL>(static_cast<const T *>(which ? a.value : a.key) + in0 + (p - p_lo) * in_stride,
                                   dst[which]);
            } else {
#pragma unroll
                for (int r = 0; r < EPL; r++) dst[which][r] = 0.0f;
            }
        }
    };
    load_kv(p_lo, xn);
    for (int64_t p = p_lo; p < p_hi; p++) {
        float x[2][EPL];
#pragma unroll
        for (int which = 0; which < 2; which++)
#pragma unroll
            for (int r = 0; r < EPL; r++) x[which][r] = xn[which][r];
        load_kv(p + 1, xn);
        if (a.do_rotary) rope_lane<EPL>(x[0], lane, d, p, a.cos_cache, a.sin_cache, a.interleaved);
        uint32_t qc[2][EPL];
        float scale[2], zp[2];
        polar_encode_warp<EPL, 2>(x, sg, active, lane, d, a.wht_scale, levels, qc, scale, zp);
        const int64_t vec = row * a.capacity + p;
#pragma unroll
        for (int which = 0; which < 2; which++) {
            // pack_bits (kv_compression.rs:294-312): this lane's elements are whole bytes
            uint64_t word = 0;
            if (a.bits == 8) {
#pragma unroll
                for (int r = 0; r < EPL; r++) word |= (uint64_t)qc[which][r] << (8 * r);
            } else {
#pragma unroll
                for (int r = 0; r + 1 < EPL; r += 2)
                    word |= (uint64_t)(qc[which][r] | (qc[which][r + 1] << 4)) << (4 * r);
            }
            if (which == 0) {
                if (active) {
                    uint8_t *dst = a.k_codes + vec * cb + lane * nb;  // cb = 32 * nb: aligned to nb bytes
                    if (nb == 8) *reinterpret_cast<uint64_t *>(dst) = word;
                    else if (nb == 4) *reinterpret_cast<uint32_t *>(dst) = (uint32_t)word;
                    else if (nb == 2) *reinterpret_cast<uint16_t *>(dst) = (uint16_t)word;
                    else *dst = (uint8_t)word;
                }
            } else if (full) {
                const int t = (int)(p - qbase);  // selects, not an indexed store: vword stays in registers
#pragma unroll
                for (int i = 0; i < 4; i++) vword[i] = t == i ? word : vword[i];
            } else if (active) {
                for (int i = 0; i < nb; i++) vdst[v_byte_offset(p, lane * nb + i, cb)] = (uint8_t)(word >> (8 * i));
            }
            if (lane == 0)
                *reinterpret_cast<float2 *>((which ? a.v_meta : a.k_meta) + vec * 2) =
                    make_float2(scale[which], zp[which]);
        }
    }
    if (full && active) {
        for (int i = 0; i < nb; i++) {
            const uint32_t w32 = (uint32_t)((vword[0] >> (8 * i)) & 0xffu) |
                                 ((uint32_t)((vword[1] >> (8 * i)) & 0xffu) << 8) |
                                 ((uint32_t)((vword[2] >> (8 * i)) & 0xffu) << 16) |
                                 ((uint32_t)((vword[3] >> (8 * i)) & 0xffu) << 24);
            *reinterpret_cast<uint32_t *>(vdst + v_byte_offset(qbase, lane * nb + i, cb)) = w32;
        }
    }
}

template <typename T, int EPL>
void launch_epl(const AppendArgs &a, dim3 grid, dim3 block, bool small, cudaStream_t stream) {
    if (small) kv_append_kernel<T, EPL, uint32_t><<<grid, block, 0, stream>>>(a);
    else kv_append_kernel<T, EPL, int64_t><<<grid, block, 0, stream>>>(a);
}

template <typename T, int EPL>
void launch_quad(const AppendArgs &a, uint32_t nquads, uint32_t nwarps, cudaStream_t stream) {
    kv_append_quad_kernel<T, EPL>
        <<<(nwarps + kAppendWarps - 1) / kAppendWarps, 32 * kAppendWarps, 0, stream>>>(a, nquads, nwarps);
}

template <typename T>
int launch_t(const AppendArgs &a, cudaStream_t stream) {
    const int64_t nvec = (int64_t)a.batch * a.seq_len * a.heads * 2;
    if (nvec == 0) return SA_OK;
    // the position-quad kernel: 8-bit codes, or 4-bit with two or more elements per lane, no QJL
    const int epl = a.head_dim <= 32 ? 1 : a.head_dim / 32;
    const int64_t nquads = ((a.pos0 + a.seq_len + 3) >> 2) - (a.pos0 >> 2);
    const int64_t nwarps = (int64_t)a.batch * a.heads * nquads;
    if ((a.bits == 8 || (a.bits == 4 && epl >= 2)) && a.k_qjl_bits == nullptr && a.v_qjl_bits == nullptr &&
        nwarps + kAppendWarps < ((int64_t)1 << 32)) {
        switch (a.head_dim) {
            case 16: case 32: launch_quad<T, 1>(a, (uint32_t)nquads, (uint32_t)nwarps, stream); break;
            case 64: launch_quad<T, 2>(a, (uint32_t)nquads, (uint32_t)nwarps, stream); break;
            case 128: launch_quad<T, 4>(a, (uint32_t)nquads, (uint32_t)nwarps, stream); break;
            case 256: launch_quad<T, 8>(a, (uint32_t)nquads, (uint32_t)nwarps, stream); break;
            default: return set_error(SA_ERR_UNSUPPORTED, "kv_append: head_dim %d not supported", a.head_dim);
        }
        count_launch();
        return check_cuda(cudaGetLastError(), "kv_append launch");
    }
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

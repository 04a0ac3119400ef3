// Low-rank K (KVCacheConfig::kv_lowrank_k; LowRankKeyDecomposer,
// kv_compression.rs:451-690) on the GPU.
//
// CompressedKVCache::write_kv (:842-853) decomposes the first K row of a
// sequence alone (decompose(k, 1, D): rank min(r, 1, D) = 1, :483) and
// updates for every later row: the row's projection on V^T is appended to
// U*S, and every 512th update re-decomposes the reconstruction U*S.V^T
// (reorthogonalize, :564-579, which keeps rank min(1, rows, D) = 1).  So the
// cache's low-rank state is one V^T row and one U*S coefficient per row.
//
//  - lowrank_append_kernel: one CTA per (KV head, batch row) replays that
//    over the appended rows in position order, bit-exact: every sum runs in
//    the reference's element order with explicitly rounded multiplies and
//    adds; the projections between two re-decompositions run in parallel (one
//    thread per row), the power iteration (:583-671) has one thread per row
//    for u = A.v, one per column for v = A^T.u, one for the norms.
//  - lowrank_attend_kernel: attention with keys read as read_k returns them
//    (:870-882): k_t = U*S[t] * V^T, so q . k_t = U*S[t] * (q . V^T); values
//    from the PolarQuant codes, accumulated in the rotated domain and rotated
//    back once.  One block of four warps per query row, each warp every fourth
//    token.
#include "sa_append.cuh"

namespace sa {

namespace {

constexpr int kLrThreads = 256;   // >= head_dim: one thread per column of V^T
constexpr int kLrAttWarps = 4;

// sqrt_approx (operators.rs:3311-3320): ten Newton steps from s = x.
__device__ __forceinline__ float lr_sqrt_approx(float x) {
    if (x <= 0.0f) return 0.0f;
    float s = x;
#pragma unroll 1
    for (int i = 0; i < 10; i++) s = __fmul_rn(0.5f, __fadd_rn(s, __fdiv_rn(x, s)));
    return s;
}

// Element e of appended K row s as write_kv receives it (RoPE applied like the append).
template <typename T>
__device__ __forceinline__ float lr_key(const AppendArgs &a, int b, int s, int h, int e) {
    const int d = a.head_dim;
    const T *src = static_cast<const T *>(a.key) + (((int64_t)b * a.seq_len + s) * a.heads + h) * d;
    const float x = ld_f32(src + e);
    return a.do_rotary ? rope_element(src, x, e, d, a.pos0 + s, a.cos_cache, a.sin_cache, a.interleaved) : x;
}

// normalize_vec (:683-690) of the shared vector v[0..n): the norm (norm_vec, :674-681) by one
// thread in element order, then the divisions.
__device__ void lr_normalize(float *v, int n, float *s_scalar) {
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int j = 0; j < n; j++) s = __fadd_rn(s, __fmul_rn(v[j], v[j]));
        s_scalar[0] = lr_sqrt_approx(s);
    }
    __syncthreads();
    const float nn = s_scalar[0];
    if (nn > 1e-30f)
        for (int j = threadIdx.x; j < n; j += blockDim.x) v[j] = __fdiv_rn(v[j], nn);
    __syncthreads();
}

// power_iteration_svd (:583-671) at rank 1 on the m x n matrix A(i, j): ten rounds of
// u = A.v, v = A^T.u, normalize(v) from the alternating start vector; then u = A.v,
// sigma = norm(u), U*S = (u / sigma) * sigma and V^T = v, or both zero when sigma < 1e-12.
// `u` is global scratch of m floats; us_out / vt_out are written only after the last read of A.
template <typename F>
__device__ void lr_power_iteration(F A, int64_t m, int n, float *u, float *s_v, float *s_scalar, float *us_out,
                                   float *vt_out) {
    const int tid = threadIdx.x;
    for (int j = tid; j < n; j += blockDim.x) s_v[j] = (j % 2 == 0) ? 1.0f : -1.0f;
    __syncthreads();
    lr_normalize(s_v, n, s_scalar);
    for (int it = 0;; it++) {
        for (int64_t i = tid; i < m; i += blockDim.x) {
            float dot = 0.0f;
            for (int j = 0; j < n; j++) dot = __fadd_rn(dot, __fmul_rn(A(i, j), s_v[j]));
            u[i] = dot;
        }
        __syncthreads();
        if (it == 10) break;
        if (tid < n) {
            float acc = 0.0f;
            for (int64_t i = 0; i < m; i++) acc = __fadd_rn(acc, __fmul_rn(A(i, tid), u[i]));
            s_v[tid] = acc;  // s_v is not read again until after the barrier below
        }
        __syncthreads();
        lr_normalize(s_v, n, s_scalar);
    }
    if (tid == 0) {
        float s = 0.0f;
        for (int64_t i = 0; i < m; i++) s = __fadd_rn(s, __fmul_rn(u[i], u[i]));
        s_scalar[1] = lr_sqrt_approx(s);
    }
    __syncthreads();
    const float sigma = s_scalar[1];
    const bool keep = !(sigma < 1e-12f);
    for (int64_t i = tid; i < m; i += blockDim.x) us_out[i] = keep ? __fmul_rn(__fdiv_rn(u[i], sigma), sigma) : 0.0f;
    for (int j = tid; j < n; j += blockDim.x) vt_out[j] = keep ? s_v[j] : 0.0f;
    __syncthreads();
}

// grid (KV heads, batch), kLrThreads threads, (3 * head_dim + 4) floats of shared memory.
template <typename T>
__global__ void __launch_bounds__(kLrThreads) lowrank_append_kernel(AppendArgs a) {
    extern __shared__ float lr_sm[];
    const int d = a.head_dim, h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    float *s_vt = lr_sm, *s_v = lr_sm + d, *s_k = lr_sm + 2 * d, *s_scalar = lr_sm + 3 * d;
    const int64_t unit = (int64_t)b * a.heads + h;
    float *vt = a.lr_vt + unit * d;
    float *us = a.lr_us + unit * a.capacity;
    float *u = a.lr_scratch + unit * a.capacity;

    int s = 0;
    if (a.pos0 == 0) {
        // the sequence's first row: decompose(k, 1, D)
        for (int e = tid; e < d; e += blockDim.x) s_k[e] = lr_key<T>(a, b, 0, h, e);
        __syncthreads();
        lr_power_iteration([&](int64_t, int j) { return s_k[j]; }, 1, d, u, s_v, s_scalar, us, s_vt);
        s = 1;
    } else {
        for (int e = tid; e < d; e += blockDim.x) s_vt[e] = vt[e];
        __syncthreads();
    }
    while (s < a.seq_len) {
        // rows up to (and including) the next one whose update re-decomposes: row r is update
        // number r since the decomposition of row 0, and every 512th update re-decomposes
        const int64_t r0 = a.pos0 + s;  // >= 1
        const int64_t rb = (r0 + 511) / 512 * 512;
        const int64_t end64 = rb - a.pos0 + 1;
        const int e_end = end64 < (int64_t)a.seq_len ? (int)end64 : a.seq_len;
        for (int i = s + tid; i < e_end; i += blockDim.x) {
            float dot = 0.0f;
            for (int c = 0; c < d; c++) dot = __fadd_rn(dot, __fmul_rn(lr_key<T>(a, b, i, h, c), s_vt[c]));
            us[a.pos0 + i] = dot;
        }
        __syncthreads();
        const int64_t last = a.pos0 + e_end - 1;
        if (last == rb) {
            // reorthogonalize: power iteration on the reconstruction (0 + U*S[i] * V^T[j], :502-526)
            lr_power_iteration([&](int64_t i, int j) { return __fadd_rn(0.0f, __fmul_rn(us[i], s_vt[j])); },
                               last + 1, d, u, s_v, s_scalar, us, s_vt);
        }
        s = e_end;
    }
    for (int e = tid; e < d; e += blockDim.x) vt[e] = s_vt[e];
}

// Code of dimension e of token t (pack_bits order, in the 16-token-block V layout).
__device__ __forceinline__ uint32_t lr_v_code(const uint8_t *vc, int64_t t, int e, int bits, int cb) {
    const int bit = e * bits, j0 = bit >> 3, sh = bit & 7;
    uint32_t w = vc[v_byte_offset(t, j0, cb)];
    if (sh + bits > 8) w |= (uint32_t)vc[v_byte_offset(t, j0 + 1, cb)] << 8;
    return (w >> sh) & ((1u << bits) - 1u);
}

// grid B * S * Hq blocks, one per (row, query token, query head); the block's kLrAttWarps warps
// take every kLrAttWarps-th token and their sums are added at the end.
template <typename T, int EPL>
__global__ void __launch_bounds__(32 * kLrAttWarps) lowrank_attend_kernel(AttendArgs a) {
    __shared__ float s_red[kLrAttWarps];
    __shared__ float s_acc[kLrAttWarps][256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = a.head_dim, G = a.group, hq_all = a.heads * G;
    const int64_t qi = blockIdx.x;
    const int hq = (int)(qi % hq_all);
    const int s = (int)((qi / hq_all) % a.seq_len);
    const int b = (int)(qi / ((int64_t)hq_all * a.seq_len));
    const int h = hq / G;
    const int64_t unit = (int64_t)b * a.heads + h;
    const bool active = lane * EPL < d;
    const int64_t pos = a.pos0 + s;  // attends tokens 0..pos
    const int64_t row = ((int64_t)b * a.seq_len + s) * hq_all + hq;
    const T *src = static_cast<const T *>(a.query) + row * d;
    const float *vt = a.lr_vt + unit * d;
    const float *us = a.lr_us + unit * a.capacity;

    // q (RoPE at its position) . V^T (every warp computes it)
    float qv = 0.0f;
    if (active) {
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            float x = ld_f32(src + e);
            if (a.do_rotary) x = rope_element(src, x, e, d, pos, a.cos_cache, a.sin_cache, a.interleaved);
            qv = fmaf(x, vt[e], qv);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qv += __shfl_xor_sync(0xffffffffu, qv, o);
    const float c = qv * a.scale * 1.4426950408889634f;  // score of token t, base 2: U*S[t] * c

    float mx = -INFINITY;
    for (int64_t t = threadIdx.x; t <= pos; t += 32 * kLrAttWarps) mx = fmaxf(mx, us[t] * c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kLrAttWarps; w++) mx = fmaxf(mx, s_red[w]);

    // sum_t p_t (code * scale + zp) in the rotated domain; lanes own EPL dimensions, this warp
    // every kLrAttWarps-th token
    const int cb = a.code_bytes;
    const uint8_t *vc = a.v_codes + unit * a.capacity * (int64_t)cb;
    const float2 *vm = reinterpret_cast<const float2 *>(a.v_meta) + unit * a.capacity;
    float acc[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) acc[r] = 0.0f;
    float l = 0.0f;
    for (int64_t t = warp; t <= pos; t += kLrAttWarps) {
        const float p = exp2f(us[t] * c - mx);
        const float2 m = vm[t];
        l += p;
        if (active) {
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                const float code = (float)lr_v_code(vc, t, lane * EPL + r, a.bits, cb);
                acc[r] = fmaf(p, fmaf(code, m.x, m.y), acc[r]);
            }
        }
    }
    __syncthreads();  // s_red is read: reuse it for the weight sums
    if (lane == 0) s_red[warp] = l;
    if (active) {
#pragma unroll
        for (int r = 0; r < EPL; r++) s_acc[warp][lane * EPL + r] = acc[r];
    }
    __syncthreads();
    if (warp != 0) return;
    float lt = 0.0f;
#pragma unroll
    for (int w = 0; w < kLrAttWarps; w++) lt += s_red[w];
    const float inv = 1.0f / lt;  // lt >= 1: the maximum term is exp2(0)
    float x[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) {
        float v = 0.0f;
        if (active) {
#pragma unroll
            for (int w = 0; w < kLrAttWarps; w++) v += s_acc[w][lane * EPL + r];
        }
        x[r] = v * inv;
    }
    warp_wht_butterfly<EPL>(x, lane, d);
    if (active) {
        T *dst = static_cast<T *>(a.out) + row * d;
        const float *sg = a.signs + (int64_t)h * d;
#pragma unroll
        for (int r = 0; r < EPL; r++)
            st_from_f32(dst + lane * EPL + r, x[r] * a.wht_scale * sg[lane * EPL + r]);
    }
}

template <typename T>
int append_t(const AppendArgs &a, cudaStream_t stream) {
    if (a.head_dim > kLrThreads) return set_error(SA_ERR_UNSUPPORTED, "lowrank append: head_dim %d", a.head_dim);
    const size_t smem = (3 * (size_t)a.head_dim + 4) * sizeof(float);
    lowrank_append_kernel<T><<<dim3((unsigned)a.heads, (unsigned)a.batch), kLrThreads, smem, stream>>>(a);
    count_launch();
    return check_cuda(cudaGetLastError(), "lowrank append launch");
}

template <typename T>
int attend_t(const AttendArgs &a, cudaStream_t stream) {
    const int64_t n = (int64_t)a.batch * a.seq_len * a.heads * a.group;
    const int64_t blocks = n;  // one block per query row
    if (blocks > 0x7fffffff) return set_error(SA_ERR_UNSUPPORTED, "lowrank attend: %lld queries", (long long)n);
    const dim3 grid((unsigned)blocks), block(32 * kLrAttWarps);
    switch (a.head_dim) {
        case 16:
        case 32: lowrank_attend_kernel<T, 1><<<grid, block, 0, stream>>>(a); break;
        case 64: lowrank_attend_kernel<T, 2><<<grid, block, 0, stream>>>(a); break;
        case 128: lowrank_attend_kernel<T, 4><<<grid, block, 0, stream>>>(a); break;
        case 256: lowrank_attend_kernel<T, 8><<<grid, block, 0, stream>>>(a); break;
        default: return set_error(SA_ERR_UNSUPPORTED, "lowrank attend: head_dim %d", a.head_dim);
    }
    count_launch();
    return check_cuda(cudaGetLastError(), "lowrank attend launch");
}

}  // namespace

int launch_lowrank_append(const AppendArgs &a, cudaStream_t stream) {
    if (a.batch == 0 || a.seq_len == 0) return SA_OK;
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return append_t<float>(a, stream);
        case SA_DTYPE_FLOAT16: return append_t<__half>(a, stream);
        case SA_DTYPE_BFLOAT16: return append_t<__nv_bfloat16>(a, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "lowrank append: dtype %d not supported", a.dtype);
    }
}

int launch_lowrank_attend(const AttendArgs &a, cudaStream_t stream) {
    if (a.batch == 0 || a.seq_len == 0) return SA_OK;
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return attend_t<float>(a, stream);
        case SA_DTYPE_FLOAT16: return attend_t<__half>(a, stream);
        case SA_DTYPE_BFLOAT16: return attend_t<__nv_bfloat16>(a, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "lowrank attend: dtype %d not supported", a.dtype);
    }
}

}  // namespace sa

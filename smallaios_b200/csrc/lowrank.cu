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
//    It also writes what attention reads of the state: the K metadata
//    {scale 0, zero point U*S[t]} per row and V^T rotated like the queries.
//    read_k returns k_t = U*S[t] * V^T (:870-882), so q . k_t = U*S[t] *
//    (q' . R(V^T)): the attention kernels' own identity q.k = scale*(q'.c) +
//    zp*sum(q') with that metadata and q'.R(V^T) in place of sum(q').
#include "sa_append.cuh"

namespace sa {

namespace {

constexpr int kLrThreads = 256;   // >= head_dim: one thread per column of V^T

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
                                   float *kmeta_out, float *vt_out) {
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
    for (int64_t i = tid; i < m; i += blockDim.x) {
        const float v = keep ? __fmul_rn(__fdiv_rn(u[i], sigma), sigma) : 0.0f;
        us_out[i] = v;
        kmeta_out[2 * i] = 0.0f;  // {scale 0, zero point U*S[i]}: the K metadata attention reads
        kmeta_out[2 * i + 1] = v;
    }
    for (int j = tid; j < n; j += blockDim.x) vt_out[j] = keep ? s_v[j] : 0.0f;
    __syncthreads();
}

// out = H.S.v / sqrt(n) by one warp (signs, butterfly, normaliser): the rotation of the queries.
template <int EPL>
__device__ void lr_rotate(const float *v, const float *sg, float wht_scale, int d, float *out) {
    const int lane = threadIdx.x & 31;
    const bool active = lane * EPL < d;
    float x[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = active ? v[lane * EPL + r] * sg[lane * EPL + r] : 0.0f;
    warp_wht_butterfly<EPL>(x, lane, d);
    if (active)
#pragma unroll
        for (int r = 0; r < EPL; r++) out[lane * EPL + r] = x[r] * wht_scale;
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
    float *kmeta = a.lr_kmeta + unit * a.capacity * 2;

    int s = 0;
    if (a.pos0 == 0) {
        // the sequence's first row: decompose(k, 1, D)
        for (int e = tid; e < d; e += blockDim.x) s_k[e] = lr_key<T>(a, b, 0, h, e);
        __syncthreads();
        lr_power_iteration([&](int64_t, int j) { return s_k[j]; }, 1, d, u, s_v, s_scalar, us, kmeta, s_vt);
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
            kmeta[2 * (a.pos0 + i)] = 0.0f;
            kmeta[2 * (a.pos0 + i) + 1] = dot;
        }
        __syncthreads();
        const int64_t last = a.pos0 + e_end - 1;
        if (last == rb) {
            // reorthogonalize: power iteration on the reconstruction (0 + U*S[i] * V^T[j], :502-526)
            lr_power_iteration([&](int64_t i, int j) { return __fadd_rn(0.0f, __fmul_rn(us[i], s_vt[j])); },
                               last + 1, d, u, s_v, s_scalar, us, kmeta, s_vt);
        }
        s = e_end;
    }
    for (int e = tid; e < d; e += blockDim.x) vt[e] = s_vt[e];
    // V^T rotated like the queries, for the attention kernels' zero-point term
    __syncthreads();
    if (tid < 32) {
        float *vtr = a.lr_vtr + unit * d;
        const float *sg = a.signs + (int64_t)h * d;
        switch (d) {
            case 16:
            case 32: lr_rotate<1>(s_vt, sg, a.wht_scale, d, vtr); break;
            case 64: lr_rotate<2>(s_vt, sg, a.wht_scale, d, vtr); break;
            case 128: lr_rotate<4>(s_vt, sg, a.wht_scale, d, vtr); break;
            default: lr_rotate<8>(s_vt, sg, a.wht_scale, d, vtr); break;
        }
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

}  // namespace sa

// The decoder-layer glue around the attention and MatMulNBits: RMSNorm with an
// optional fused residual add (com.microsoft.SimplifiedLayerNormalization /
// SkipSimplifiedLayerNormalization, onnx-rt/src/ops/microsoft.rs:441-540, on
// op_rms_normalization, onnx-rt/src/ops/generative.rs:517-580), and SwiGLU
// (Silu(gate) * up, the Silu + Mul pair GraphBuilder::swiglu emits,
// onnx-rt/src/model_loader/graph_builder.rs:366-369; Silu as in
// onnx-rt/src/ops/activations.rs:37-39).  Both are HBM-bound row kernels
// with coalesced loads and f32 arithmetic, rounding once to the activation
// type at the store (RMSNorm: one CTA per row; SwiGLU: a row per grid.y).
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kGlueThreads = 256;

template <typename T>
__device__ __forceinline__ float glue_ld(const T *p, int64_t i) {
    return ld_f32(p + i);
}

// Both kernels run as programmatic dependent launches: the next kernel may be scheduled at
// once (it waits for this grid before it reads what this grid writes), and this grid waits
// for the previous one before it touches global memory.
__device__ __forceinline__ void glue_pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}

template <typename K, typename... Args>
cudaError_t glue_launch(K kern, dim3 grid, cudaStream_t stream, Args... args) {
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kGlueThreads);
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// pre = x (+ skip) (+ bias); y = pre / sqrt(mean(pre^2) + eps) * w.
// `pre` (optional) receives the rounded pre-sum: the residual of the next add.
template <typename T>
__global__ void __launch_bounds__(kGlueThreads)
    rms_norm_kernel(const T *__restrict__ x, const T *__restrict__ skip, const T *__restrict__ bias,
                    const T *__restrict__ w, T *__restrict__ y, T *__restrict__ pre, int cols, float eps) {
    __shared__ float s_red[kGlueThreads / 32];
    const int64_t base = (int64_t)blockIdx.x * cols;
    const int tid = threadIdx.x;
    glue_pdl_enter();
    float ss = 0.0f;
    for (int i = tid; i < cols; i += kGlueThreads) {
        float v = glue_ld(x, base + i);
        if (skip) v += glue_ld(skip, base + i);
        if (bias) v += glue_ld(bias, i);
        if (pre) st_from_f32(pre + base + i, v);
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) s_red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
        float t = tid < kGlueThreads / 32 ? s_red[tid] : 0.0f;
        t = warp_sum(t);
        if (tid == 0) s_red[0] = t;
    }
    __syncthreads();
    const float rinv = 1.0f / sqrtf(s_red[0] / (float)cols + eps);
    for (int i = tid; i < cols; i += kGlueThreads) {
        float v = glue_ld(x, base + i);
        if (skip) v += glue_ld(skip, base + i);
        if (bias) v += glue_ld(bias, i);
        st_from_f32(y + base + i, v * rinv * glue_ld(w, i));
    }
}

// y[r][j] = silu(gate[r][j]) * up[r][j], silu(g) = g / (1 + exp(-g)).
template <typename T>
__global__ void __launch_bounds__(kGlueThreads)
    silu_mul_kernel(const T *__restrict__ gate, const T *__restrict__ up, int64_t ld_in, T *__restrict__ y,
                    int64_t rows, int cols) {
    glue_pdl_enter();
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)  // grid.y is capped at 65535 rows
        for (int j = blockIdx.x * kGlueThreads + threadIdx.x; j < cols; j += gridDim.x * kGlueThreads) {
            const float g = glue_ld(gate, r * ld_in + j), u = glue_ld(up, r * ld_in + j);
            st_from_f32(y + r * cols + j, g / (1.0f + expf(-g)) * u);
        }
}

// The same RMSNorm with the row held in registers between its two passes (one read of x and
// skip instead of two) and 16-byte accesses: for rows of up to 256 * U 16-byte units whose
// pointers and length keep every unit aligned.  Each thread sums the squares of its elements in
// its own order (as the scalar kernel does, with another split of the row).
template <typename T, int U>
__global__ void __launch_bounds__(kGlueThreads)
    rms_norm_vec_kernel(const T *__restrict__ x, const T *__restrict__ skip, const T *__restrict__ bias,
                        const T *__restrict__ w, T *__restrict__ y, T *__restrict__ pre, int cols, float eps) {
    constexpr int V = 16 / (int)sizeof(T);
    union Vec {
        uint4 v;
        T t[V];
    };
    __shared__ float s_red[kGlueThreads / 32];
    const int64_t base = (int64_t)blockIdx.x * cols;
    const int tid = threadIdx.x;
    glue_pdl_enter();
    float v[U][V];
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < U; u++) {
        const int j = (u * kGlueThreads + tid) * V;
        if (j < cols) {
            Vec a, b, c;
            a.v = *reinterpret_cast<const uint4 *>(x + base + j);
            if (skip) b.v = *reinterpret_cast<const uint4 *>(skip + base + j);
            if (bias) c.v = *reinterpret_cast<const uint4 *>(bias + j);
            Vec p;
#pragma unroll
            for (int i = 0; i < V; i++) {
                float t = DT<T>::to_f32(a.t[i]);
                if (skip) t += DT<T>::to_f32(b.t[i]);
                if (bias) t += DT<T>::to_f32(c.t[i]);
                v[u][i] = t;
                p.t[i] = DT<T>::from_f32(t);
                ss = fmaf(t, t, ss);
            }
            if (pre) *reinterpret_cast<uint4 *>(pre + base + j) = p.v;
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) s_red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
        float t = tid < kGlueThreads / 32 ? s_red[tid] : 0.0f;
        t = warp_sum(t);
        if (tid == 0) s_red[0] = t;
    }
    __syncthreads();
    const float rinv = 1.0f / sqrtf(s_red[0] / (float)cols + eps);
#pragma unroll
    for (int u = 0; u < U; u++) {
        const int j = (u * kGlueThreads + tid) * V;
        if (j < cols) {
            Vec wv, o;
            wv.v = *reinterpret_cast<const uint4 *>(w + j);
#pragma unroll
            for (int i = 0; i < V; i++) o.t[i] = DT<T>::from_f32(v[u][i] * rinv * DT<T>::to_f32(wv.t[i]));
            *reinterpret_cast<uint4 *>(y + base + j) = o.v;
        }
    }
}

// The same SwiGLU, 16 bytes of each operand per thread (16 / sizeof(T) elements): for rows whose
// start and length keep every 16-byte unit aligned.  One thread per unit, grid.y = row.
template <typename T>
__global__ void __launch_bounds__(kGlueThreads)
    silu_mul_vec_kernel(const T *__restrict__ gate, const T *__restrict__ up, int64_t ld_in, T *__restrict__ y,
                        int64_t rows, int cols) {
    constexpr int V = 16 / (int)sizeof(T);
    glue_pdl_enter();
    const int j = (blockIdx.x * kGlueThreads + threadIdx.x) * V;
    if (j >= cols) return;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {  // grid.y is capped at 65535 rows
        union U {
            uint4 v;
            T t[V];
        } g, u, o;
        g.v = *reinterpret_cast<const uint4 *>(gate + r * ld_in + j);
        u.v = *reinterpret_cast<const uint4 *>(up + r * ld_in + j);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const float gf = DT<T>::to_f32(g.t[i]), uf = DT<T>::to_f32(u.t[i]);
            o.t[i] = DT<T>::from_f32(gf / (1.0f + expf(-gf)) * uf);
        }
        *reinterpret_cast<uint4 *>(y + r * cols + j) = o.v;
    }
}

template <typename T, int U>
cudaError_t launch_rms_vec(const void *x, const void *skip, const void *bias, const void *w, void *y, void *pre,
                           int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
    return glue_launch(rms_norm_vec_kernel<T, U>, dim3((unsigned)rows), stream, static_cast<const T *>(x),
                       static_cast<const T *>(skip), static_cast<const T *>(bias), static_cast<const T *>(w),
                       static_cast<T *>(y), static_cast<T *>(pre), (int)cols, eps);
}

template <typename T>
int launch_rms_t(const void *x, const void *skip, const void *bias, const void *w, void *y, void *pre, int64_t rows,
                 int64_t cols, float eps, cudaStream_t stream) {
    constexpr int V = 16 / (int)sizeof(T);
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(skip) |
                         reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(w) |
                         reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(pre);
    const int64_t units = cols / V;
    if ((al & 15) == 0 && cols % V == 0 && units <= 8 * kGlueThreads) {
        const int64_t per = (units + kGlueThreads - 1) / kGlueThreads;  // units per thread: 1..8
        cudaError_t e;
        if (per <= 1) e = launch_rms_vec<T, 1>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        else if (per <= 2) e = launch_rms_vec<T, 2>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        else if (per <= 4) e = launch_rms_vec<T, 4>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        else e = launch_rms_vec<T, 8>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        count_launch();
        return check_cuda(e, "rms_norm launch");
    }
    const cudaError_t e = glue_launch(rms_norm_kernel<T>, dim3((unsigned)rows), stream, static_cast<const T *>(x),
                                      static_cast<const T *>(skip), static_cast<const T *>(bias),
                                      static_cast<const T *>(w), static_cast<T *>(y), static_cast<T *>(pre), (int)cols,
                                      eps);
    count_launch();
    return check_cuda(e, "rms_norm launch");
}

template <typename T>
int launch_silu_t(const void *gate, const void *up, int64_t ld_in, void *y, int64_t rows, int64_t cols,
                  cudaStream_t stream) {
    constexpr int V = 16 / (int)sizeof(T);
    const uintptr_t al = reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
                         reinterpret_cast<uintptr_t>(y);
    const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
    if ((al & 15) == 0 && cols % V == 0 && ld_in % V == 0) {
        const int64_t units = cols / V;
        const cudaError_t e = glue_launch(silu_mul_vec_kernel<T>,
                                          dim3((unsigned)((units + kGlueThreads - 1) / kGlueThreads), gy), stream,
                                          static_cast<const T *>(gate), static_cast<const T *>(up), ld_in,
                                          static_cast<T *>(y), rows, (int)cols);
        count_launch();
        return check_cuda(e, "silu_mul launch");
    }
    const int64_t blocks = (cols + kGlueThreads - 1) / kGlueThreads;
    const unsigned bx = (unsigned)(blocks < 64 ? blocks : 64);
    const cudaError_t e = glue_launch(silu_mul_kernel<T>, dim3(bx, gy), stream, static_cast<const T *>(gate),
                                      static_cast<const T *>(up), ld_in, static_cast<T *>(y), rows, (int)cols);
    count_launch();
    return check_cuda(e, "silu_mul launch");
}

}  // namespace

int launch_rms_norm(const void *x, const void *skip, const void *bias, const void *w, void *y, void *pre, int dtype,
                    int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_rms_t<float>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        case SA_DTYPE_FLOAT16: return launch_rms_t<__half>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
        default: return launch_rms_t<__nv_bfloat16>(x, skip, bias, w, y, pre, rows, cols, eps, stream);
    }
}

int launch_silu_mul(const void *gate, const void *up, int64_t ld_in, void *y, int dtype, int64_t rows, int64_t cols,
                    cudaStream_t stream) {
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_silu_t<float>(gate, up, ld_in, y, rows, cols, stream);
        case SA_DTYPE_FLOAT16: return launch_silu_t<__half>(gate, up, ld_in, y, rows, cols, stream);
        default: return launch_silu_t<__nv_bfloat16>(gate, up, ld_in, y, rows, cols, stream);
    }
}

}  // namespace sa

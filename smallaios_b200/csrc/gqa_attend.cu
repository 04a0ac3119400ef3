// GroupQueryAttention over the PolarQuant-compressed cache: generic split-K
// kernel (any bits in {3,4,8}, head_dim 16..256, any group size <= 8, any
// number of query tokens).  The fast decode kernel for the common shapes
// lives in gqa_decode_mma.cu; this one covers everything else.
//
// Math (rotated domain).  The reference decodes every cached vector,
// k_hat = S.H.(c*scale + zp)/sqrt(n) (PolarQuantizer::decode,
// kv_compression.rs:270-286), and runs SDPA on k_hat (ops/microsoft.rs:
// 241-319).  S.H/sqrt(n) is orthogonal and symmetric, so
//   q . k_hat          = q' . (c*scale + zp) = scale*(q'.c) + zp*sum(q'),
//   sum_t p_t v_hat_t  = S.H.(sum_t p_t (c_t*scale_t + zp_t))/sqrt(n),
// with q' = H.S.q/sqrt(n), the same rotation encode applies.  The kernel
// rotates q once, streams codes without ever decoding a vector, and applies
// the inverse rotation once per output row.
#include "sa_common.cuh"
#include "sa_gather.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;

struct Layout {
    int d, bits, cb, cap, heads, group;
};

// Code of element e of a K token row (pack_bits order, contiguous bytes).
__device__ __forceinline__ uint32_t code_at(const uint8_t *row, int e, int bits, int cb) {
    const int bo = e * bits;
    const int j = bo >> 3, sh = bo & 7;
    uint32_t w = row[j];
    if (sh + bits > 8 && j + 1 < cb) w |= (uint32_t)row[j + 1] << 8;
    return (w >> sh) & ((1u << bits) - 1u);
}

// Code of element e of V token t (bytes placed by v_byte_offset).
__device__ __forceinline__ uint32_t v_code_at(const uint8_t *vrow, int64_t t, int e, int bits, int cb) {
    const int bo = e * bits;
    const int j = bo >> 3, sh = bo & 7;
    uint32_t w = vrow[v_byte_offset(t, j, cb)];
    if (sh + bits > 8 && j + 1 < cb) w |= (uint32_t)vrow[v_byte_offset(t, j + 1, cb)] << 8;
    return (w >> sh) & ((1u << bits) - 1u);
}

template <typename T, int EPL>
__device__ __forceinline__ void rope_and_rotate(const T *src, float (&x)[EPL], int lane, int d, int64_t pos,
                                                const AttendArgs &a, const float *sg) {
    const bool active = lane * EPL < d;
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = active ? ld_f32(src + lane * EPL + r) : 0.0f;
    if (a.do_rotary && active) {
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
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] *= active ? sg[lane * EPL + r] : 1.0f;
    warp_wht_butterfly<EPL>(x, lane, d);
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] *= a.wht_scale;
}

// Inverse rotation of one output vector held as EPL values per lane and
// store to out (dtype T).
template <typename T, int EPL>
__device__ __forceinline__ void unrotate_store(float (&x)[EPL], int lane, int d, const float *sg, float wht_scale,
                                               T *dst) {
    warp_wht_butterfly<EPL>(x, lane, d);
    if (lane * EPL < d) {
#pragma unroll
        for (int r = 0; r < EPL; r++) st_from_f32(dst + lane * EPL + r, x[r] * wht_scale * sg[lane * EPL + r]);
    }
}

// grid = (splits, heads, batch*seq_len), block = 32*kWarps.
template <typename T, int EPL, int MAXG>
__global__ void __launch_bounds__(32 * kWarps) attend_split_kernel(AttendArgs a, int n_splits, int tokens_per_split) {
    extern __shared__ float smem[];
    const int d = a.head_dim, G = a.group;
    float *s_q = smem;                                   // [G][d] rotated queries
    float *s_qsum = s_q + MAXG * d;                      // [G]
    float *s_acc = s_qsum + MAXG;                        // [kWarps][G][d]
    float *s_mlz = s_acc + kWarps * MAXG * d;            // [kWarps][G][3]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
    const int b = row / a.seq_len, s = row % a.seq_len;
    const int64_t qpos = a.pos0 + s;
    const int64_t total = qpos + 1;  // causal: keys [0, qpos]
    const float *sg = a.signs + (int64_t)h * d;
    const int qheads = a.heads * G;

    // Prologue: RoPE + rotation of the G query heads of this KV head.
    for (int g = warp; g < G; g += kWarps) {
        const T *src = static_cast<const T *>(a.query) + ((int64_t)row * qheads + h * G + g) * d;
        float x[EPL];
        rope_and_rotate<T, EPL>(src, x, lane, d, qpos, a, sg);
        float part = 0.0f;
        if (lane * EPL < d) {
            const float *vtr = a.lr_vtr ? a.lr_vtr + ((int64_t)b * a.heads + h) * d : nullptr;
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                s_q[g * d + lane * EPL + r] = x[r];
                part += vtr ? x[r] * vtr[lane * EPL + r] : x[r];  // sum(q'), or q'.V^T with low-rank K
            }
        }
        part = warp_sum(part);
        if (lane == 0) s_qsum[g] = part;
    }
    __syncthreads();

    float q[MAXG][EPL], acc[MAXG][EPL], m[MAXG], l[MAXG], z[MAXG];
    const bool active = lane * EPL < d;
#pragma unroll
    for (int g = 0; g < MAXG; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
        z[g] = 0.0f;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            q[g][r] = (g < G && active) ? s_q[g * d + lane * EPL + r] : 0.0f;
            acc[g][r] = 0.0f;
        }
    }

    const int64_t hrow = (int64_t)b * a.heads + h;
    const uint8_t *kc = a.k_codes + hrow * a.capacity * a.code_bytes;
    const uint8_t *vc = a.v_codes + hrow * a.capacity * a.code_bytes;
    const float *km = a.k_meta + hrow * a.capacity * 2;
    const float *vm = a.v_meta + hrow * a.capacity * 2;
    const int64_t t_begin = (int64_t)split * tokens_per_split;
    int64_t t_end = t_begin + tokens_per_split;
    if (t_end > total) t_end = total;

    for (int64_t t = t_begin + warp; t < t_end; t += kWarps) {
        const uint8_t *krow = kc + t * a.code_bytes;
        float ck[EPL], cv[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            ck[r] = active ? (float)code_at(krow, e, a.bits, a.code_bytes) : 0.0f;
            cv[r] = active ? (float)v_code_at(vc, t, e, a.bits, a.code_bytes) : 0.0f;
        }
        const float kscale = km[t * 2], kzp = km[t * 2 + 1];
        const float vscale = vm[t * 2], vzp = vm[t * 2 + 1];
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
            if (g >= G) break;
            float dot = 0.0f;
#pragma unroll
            for (int r = 0; r < EPL; r++) dot += ck[r] * q[g][r];
            dot = warp_sum(dot);
            const float sc = (kscale * dot + kzp * s_qsum[g]) * a.scale * kLog2e;
            const float mn = fmaxf(m[g], sc);
            const float alpha = exp2f(m[g] - mn);
            const float p = exp2f(sc - mn);
            m[g] = mn;
            l[g] = l[g] * alpha + p;
            z[g] = z[g] * alpha + p * vzp;
            const float pv = p * vscale;
#pragma unroll
            for (int r = 0; r < EPL; r++) acc[g][r] = acc[g][r] * alpha + pv * cv[r];
        }
    }

    // Merge the warps of this CTA.
    for (int g = 0; g < G; g++) {
        if (lane == 0) {
            s_mlz[(warp * MAXG + g) * 3 + 0] = m[g];
            s_mlz[(warp * MAXG + g) * 3 + 1] = l[g];
            s_mlz[(warp * MAXG + g) * 3 + 2] = z[g];
        }
        if (active) {
#pragma unroll
            for (int r = 0; r < EPL; r++) s_acc[(warp * MAXG + g) * d + lane * EPL + r] = acc[g][r];
        }
    }
    __syncthreads();

    for (int g = warp; g < G; g += kWarps) {
        float M = -INFINITY;
        for (int w = 0; w < kWarps; w++) M = fmaxf(M, s_mlz[(w * MAXG + g) * 3]);
        float L = 0.0f, Z = 0.0f, wts[kWarps];
        for (int w = 0; w < kWarps; w++) {
            const float mw = s_mlz[(w * MAXG + g) * 3];
            wts[w] = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
            L += wts[w] * s_mlz[(w * MAXG + g) * 3 + 1];
            Z += wts[w] * s_mlz[(w * MAXG + g) * 3 + 2];
        }
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            float A = 0.0f;
            if (active)
                for (int w = 0; w < kWarps; w++) A += wts[w] * s_acc[(w * MAXG + g) * d + lane * EPL + r];
            x[r] = A;
        }
        if (n_splits == 1) {
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
            for (int r = 0; r < EPL; r++) x[r] = L > 0.0f ? (x[r] + Z) * inv : 0.0f;
            T *dst = static_cast<T *>(a.out) + ((int64_t)row * qheads + h * G + g) * d;
            unrotate_store<T, EPL>(x, lane, d, sg, a.wht_scale, dst);
        } else {
            float *ws = a.workspace + ((((int64_t)row * a.heads + h) * n_splits + split) * G + g) * (d + 4);
            if (active) {
#pragma unroll
                for (int r = 0; r < EPL; r++) ws[lane * EPL + r] = x[r];
            }
            if (lane == 0) {
                ws[d] = M;
                ws[d + 1] = L;
                ws[d + 2] = Z;
            }
        }
    }
}

// Merge split-K partials, normalise, inverse-rotate, store.
// grid = (heads*group, batch*seq_len), block = 32.
template <typename T, int EPL>
__global__ void __launch_bounds__(32) attend_combine_kernel(AttendArgs a, int n_splits) {
    const int lane = threadIdx.x;
    const int d = a.head_dim, G = a.group;
    const int hg = blockIdx.x, row = blockIdx.y;
    const int h = hg / G, g = hg % G;
    const float *base = a.workspace + (((int64_t)row * a.heads + h) * n_splits * G + g) * (d + 4);
    const int64_t sstride = (int64_t)G * (d + 4);
    float M = -INFINITY;
    for (int sp = 0; sp < n_splits; sp++) M = fmaxf(M, base[sp * sstride + d]);
    float L = 0.0f, Z = 0.0f, x[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = 0.0f;
    const bool active = lane * EPL < d;
    for (int sp = 0; sp < n_splits; sp++) {
        const float *p = base + sp * sstride;
        const float ms = p[d];
        const float w = (ms == -INFINITY) ? 0.0f : exp2f(ms - M);
        L += w * p[d + 1];
        Z += w * p[d + 2];
        if (active) {
#pragma unroll
            for (int r = 0; r < EPL; r++) x[r] += w * p[lane * EPL + r];
        }
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = L > 0.0f ? (x[r] + Z) * inv : 0.0f;
    const int qheads = a.heads * G;
    T *dst = static_cast<T *>(a.out) + ((int64_t)row * qheads + h * G + g) * d;
    unrotate_store<T, EPL>(x, lane, d, a.signs + (int64_t)h * d, a.wht_scale, dst);
}

template <int MAXG>
size_t split_smem_bytes(int d) {
    return sizeof(float) * ((size_t)MAXG * d + MAXG + (size_t)kWarps * MAXG * d + (size_t)kWarps * MAXG * 3);
}

template <typename T, int EPL, int MAXG>
int launch_generic(const AttendArgs &a, int n_splits, int tps, cudaStream_t stream) {
    const size_t smem = split_smem_bytes<MAXG>(a.head_dim);
    auto kern = attend_split_kernel<T, EPL, MAXG>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "gqa_attend smem attribute");
    }
    const int64_t rows = (int64_t)a.batch * a.seq_len;
    if (rows > 65535 || a.heads * a.group > 65535)  // grid y/z limits of the split and combine launches
        return set_error(SA_ERR_UNSUPPORTED,
                         "gqa_attend: batch*seq_len = %lld query rows exceed the 65535 rows one call of the "
                         "general attention kernel takes; split the call into chunks of fewer rows",
                         (long long)rows);
    dim3 grid(n_splits, a.heads, (unsigned)rows);
    kern<<<grid, 32 * kWarps, smem, stream>>>(a, n_splits, tps);
    count_launch();
    int rc = check_cuda(cudaGetLastError(), "gqa_attend split launch");
    if (rc != SA_OK || n_splits == 1) return rc;
    attend_combine_kernel<T, EPL><<<dim3(a.heads * a.group, (unsigned)rows), 32, 0, stream>>>(a, n_splits);
    count_launch();
    return check_cuda(cudaGetLastError(), "gqa_attend combine launch");
}

template <typename T, int EPL>
int launch_by_group(const AttendArgs &a, int n_splits, int tps, cudaStream_t stream) {
    if (a.group <= 1) return launch_generic<T, EPL, 1>(a, n_splits, tps, stream);
    if (a.group <= 2) return launch_generic<T, EPL, 2>(a, n_splits, tps, stream);
    if (a.group <= 4) return launch_generic<T, EPL, 4>(a, n_splits, tps, stream);
    if (a.group <= 8) return launch_generic<T, EPL, 8>(a, n_splits, tps, stream);
    return set_error(SA_ERR_UNSUPPORTED, "gqa_attend: group size %d > 8 not supported", a.group);
}

template <typename T>
int launch_by_dim(const AttendArgs &a, int n_splits, int tps, cudaStream_t stream) {
    switch (a.head_dim) {
        case 16:
        case 32: return launch_by_group<T, 1>(a, n_splits, tps, stream);
        case 64: return launch_by_group<T, 2>(a, n_splits, tps, stream);
        case 128: return launch_by_group<T, 4>(a, n_splits, tps, stream);
        case 256: return launch_by_group<T, 8>(a, n_splits, tps, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "gqa_attend: head_dim %d not supported", a.head_dim);
    }
}

}  // namespace

// Split-K partition: enough CTAs for a few waves, at least 256 tokens each,
// within the workspace.
void choose_splits(const AttendArgs &a, int64_t total, int *n_splits, int *tps) {
    const int64_t units = (int64_t)a.batch * a.seq_len * a.heads;
    int64_t want = (4LL * a.sm_count + units - 1) / units;
    int64_t by_len = (total + 255) / 256;
    int64_t n = want < by_len ? want : by_len;
    if (n > kMaxSplits) n = kMaxSplits;
    const int64_t per_split = (int64_t)a.group * (a.head_dim + 4);
    const int64_t by_ws = per_split > 0 ? (int64_t)(a.workspace_floats / (size_t)(units * per_split)) : 0;
    if (n > by_ws) n = by_ws;
    if (n < 1) n = 1;
    int64_t t = (total + n - 1) / n;
    n = (total + t - 1) / t;
    *n_splits = (int)n;
    *tps = (int)t;
}

// Split merge + normalisation + inverse rotation for a workspace filled by
// any split kernel (same partial format).
int launch_gqa_combine(const AttendArgs &a, int n_splits, cudaStream_t stream) {
    const dim3 grid(a.heads * a.group, a.batch * a.seq_len);
    switch (a.dtype) {
        case SA_DTYPE_FLOAT:
            if (a.head_dim == 64) attend_combine_kernel<float, 2><<<grid, 32, 0, stream>>>(a, n_splits);
            else attend_combine_kernel<float, 4><<<grid, 32, 0, stream>>>(a, n_splits);
            break;
        case SA_DTYPE_FLOAT16:
            if (a.head_dim == 64) attend_combine_kernel<__half, 2><<<grid, 32, 0, stream>>>(a, n_splits);
            else attend_combine_kernel<__half, 4><<<grid, 32, 0, stream>>>(a, n_splits);
            break;
        default:
            if (a.head_dim == 64) attend_combine_kernel<__nv_bfloat16, 2><<<grid, 32, 0, stream>>>(a, n_splits);
            else attend_combine_kernel<__nv_bfloat16, 4><<<grid, 32, 0, stream>>>(a, n_splits);
            break;
    }
    count_launch();
    return check_cuda(cudaGetLastError(), "gqa_attend combine launch");
}

// Head-sharded output of the generic path: rows of attn_out [B][S][q_local*D]
// copied into every gather buffer at the rank's columns (16-byte copies; the
// column offset is col0*D elements, a multiple of 16 bytes for D >= 16).
__global__ void __launch_bounds__(256) gather_scatter_kernel(const uint4 *src, GatherOut g, int row_vecs,
                                                             int64_t dst_row_vecs, int64_t col_vecs) {
    const int64_t row = blockIdx.x;
    const uint4 *s = src + row * row_vecs;
    for (int i = threadIdx.x; i < row_vecs; i += blockDim.x) {
        const uint4 x = s[i];
        for (int r = 0; r < g.n; r++) static_cast<uint4 *>(g.p[r])[row * dst_row_vecs + col_vecs + i] = x;
    }
    if (g.sig[0]) gather_complete(g);
}

int launch_gather_scatter(const AttendArgs &a, cudaStream_t stream) {
    const int esz = a.dtype == SA_DTYPE_FLOAT ? 4 : 2;
    const int64_t local_q = (int64_t)a.heads * a.group;
    const int row_vecs = (int)(local_q * a.head_dim * esz / 16);
    const int64_t dst_row_vecs = (int64_t)a.gather.cols * a.head_dim * esz / 16;
    const int64_t col_vecs = (int64_t)a.gather.col0 * a.head_dim * esz / 16;
    const unsigned rows = (unsigned)((int64_t)a.batch * a.seq_len);
    gather_scatter_kernel<<<rows, 256, 0, stream>>>(static_cast<const uint4 *>(a.out), a.gather, row_vecs, dst_row_vecs,
                                                   col_vecs);
    count_launch();
    return check_cuda(cudaGetLastError(), "gqa gather scatter launch");
}

int launch_gqa_attend_generic(const AttendArgs &a, cudaStream_t stream) {
    const int64_t total = a.pos0 + a.seq_len;
    int n_splits, tps;
    choose_splits(a, total, &n_splits, &tps);
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_by_dim<float>(a, n_splits, tps, stream);
        case SA_DTYPE_FLOAT16: return launch_by_dim<__half>(a, n_splits, tps, stream);
        case SA_DTYPE_BFLOAT16: return launch_by_dim<__nv_bfloat16>(a, n_splits, tps, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "gqa_attend: dtype %d not supported", a.dtype);
    }
}

}  // namespace sa

// ---------------------------------------------------------------------------
// Allocation-free attention entry point.
//
// Some callers may not allocate device memory once they are running: a
// real-time partition that reserves every buffer at start-up so that an
// inference step has a bounded, failure-free memory footprint, or a host
// whose memory is owned by its own pool and must not see a cudaMalloc /
// cudaFree from a library.  sa_gqa_attend needs a cache handle, and that
// handle owns a split-K workspace the library allocated.  This entry point
// instead takes the caller's cache buffers directly (an sa_kv_layer_view the
// caller fills in) and keeps its split-K partials in the fixed array below,
// which the CUDA module reserves on every GPU that loads the library and keeps
// until the process exits.  It never calls cudaMalloc, cudaFree or any
// allocating routine.
// ---------------------------------------------------------------------------
namespace sa {
namespace {

constexpr size_t kStaticScratchFloats = SA_STATIC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// Split-K partials of the allocation-free path.  Host code must not pass this
// name to a kernel: on the host it is only a stand-in for the symbol, so its
// device address is looked up with cudaGetSymbolAddress once per device.
static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];

struct StaticScratchSlot {
    float *ptr;
    int sm_count;
};
static StaticScratchSlot g_scratch_slots[kMaxDevices];
static int g_scratch_ready[kMaxDevices];  // 0 = not set up, 1 = ready

// One-time set-up on the current device (the first call on each device does
// it): resolve the array's device address and the SM count.  Concurrent
// first calls on one device may both resolve it; they store the same values.
int static_scratch_for_current_device(StaticScratchSlot *slot) {
    int dev = -1;
    int rc = check_cuda(cudaGetDevice(&dev), "gqa_attend_no_alloc: cudaGetDevice");
    if (rc != SA_OK) return rc;
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(SA_ERR_UNSUPPORTED, "gqa_attend_no_alloc: device %d beyond %d", dev, kMaxDevices);
    if (__atomic_load_n(&g_scratch_ready[dev], __ATOMIC_ACQUIRE)) {
        *slot = g_scratch_slots[dev];
        return SA_OK;
    }
    StaticScratchSlot s;
    s.ptr = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(reinterpret_cast<void **>(&s.ptr), g_static_scratch),
                    "gqa_attend_no_alloc: cudaGetSymbolAddress(static scratch)");
    if (rc != SA_OK) return rc;
    if (s.ptr == nullptr) return set_error(SA_ERR_CUDA, "gqa_attend_no_alloc: static scratch has no device address");
    s.sm_count = 0;
    rc = check_cuda(cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev),
                    "gqa_attend_no_alloc: SM count");
    if (rc != SA_OK) return rc;
    if (s.sm_count <= 0) s.sm_count = 148;
    g_scratch_slots[dev] = s;
    __atomic_store_n(&g_scratch_ready[dev], 1, __ATOMIC_RELEASE);
    *slot = s;
    return SA_OK;
}

}  // namespace
}  // namespace sa

extern "C" int sa_gqa_attend_no_alloc(const sa_kv_layer_view *layer, int64_t past_len, const void *query,
                                      void *attn_out, int32_t dtype, int32_t batch, int32_t seq_len,
                                      int32_t group, int32_t has_scale, float scale, const float *cos_cache,
                                      const float *sin_cache, int32_t cache_rows, int32_t do_rotary,
                                      int32_t rotary_interleaved, sa_stream_t stream) {
    using namespace sa;
    if (!layer) return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend_no_alloc: NULL layer view");
    const sa_kv_layer_view &v = *layer;
    if (!v.k_codes || !v.v_codes || !v.k_meta || !v.v_meta || !v.signs)
        return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend_no_alloc: NULL pointer in the layer view");
    const int d = v.head_dim;
    if (d < 16 || d > 256 || (d & (d - 1)) != 0)
        return set_error(SA_ERR_UNSUPPORTED, "gqa_attend_no_alloc: head_dim %d not a power of two in 16..256", d);
    if (v.bits != 3 && v.bits != 4 && v.bits != 8)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "bits must be 3, 4, or 8");
    if (v.code_bytes != d * v.bits / 8)
        return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend_no_alloc: code_bytes %d != head_dim*bits/8", v.code_bytes);
    if (v.kv_heads <= 0 || v.batch <= 0 || v.capacity <= 0 || v.capacity % kVBlock != 0 || v.code_bytes % 4 != 0)
        return set_error(SA_ERR_SHAPE_MISMATCH,
                         "gqa_attend_no_alloc: kv_heads/batch must be > 0, capacity a positive multiple of 16 and "
                         "code_bytes a multiple of 4");
    if (group < 1 || group > 8)
        return set_error(SA_ERR_UNSUPPORTED, "gqa_attend_no_alloc: group size %d outside 1..8", group);
    if (dtype != SA_DTYPE_FLOAT && dtype != SA_DTYPE_FLOAT16 && dtype != SA_DTYPE_BFLOAT16)
        return set_error(SA_ERR_UNSUPPORTED, "gqa_attend_no_alloc: dtype %d not supported", dtype);
    if (batch != v.batch)
        return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend_no_alloc: batch %d != view batch %d", batch, v.batch);
    if (seq_len < 0 || past_len < 0)
        return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend_no_alloc: negative seq_len/past_len");
    if (seq_len == 0) return SA_OK;
    if (!query || !attn_out) return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend_no_alloc: NULL query/attn_out");
    if (past_len + seq_len > v.capacity)
        return set_error(SA_ERR_CAPACITY, "gqa_attend_no_alloc: %lld tokens exceed the view capacity %d",
                         (long long)(past_len + seq_len), v.capacity);
    if (do_rotary) {
        if (!cos_cache || !sin_cache)
            return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend_no_alloc: do_rotary=1 but cos/sin cache missing");
        if (past_len + seq_len - 1 >= cache_rows)
            return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend_no_alloc: position %lld out of cache range %d",
                             (long long)(past_len + seq_len - 1), cache_rows);
    }

    AttendArgs a{};
    a.query = query;
    a.out = attn_out;
    a.dtype = dtype;
    a.batch = batch;
    a.seq_len = seq_len;
    a.heads = v.kv_heads;
    a.group = group;
    a.head_dim = d;
    a.bits = v.bits;
    a.code_bytes = v.code_bytes;
    a.capacity = v.capacity;
    a.pos0 = past_len;
    a.k_codes = v.k_codes;
    a.v_codes = v.v_codes;
    a.k_meta = v.k_meta;
    a.v_meta = v.v_meta;
    a.signs = v.signs;
    a.wht_scale = v.wht_scale;
    a.scale = has_scale ? scale : 1.0f / host_sqrt_f32((float)d);
    a.cos_cache = cos_cache;
    a.sin_cache = sin_cache;
    a.cache_rows = cache_rows;
    a.do_rotary = do_rotary ? 1 : 0;
    a.interleaved = rotary_interleaved ? 1 : 0;
    if (v.lr_kmeta && v.lr_vtr) {
        // low-rank K: {0, U*S[t]} metadata and the rotated V^T
        a.k_meta = v.lr_kmeta;
        a.lr_vtr = v.lr_vtr;
    }

    StaticScratchSlot slot;
    int rc = static_scratch_for_current_device(&slot);
    if (rc != SA_OK) return rc;
    a.workspace = slot.ptr;
    a.workspace_floats = kStaticScratchFloats;
    a.sm_count = slot.sm_count;

    // The split count the library would pick with unlimited scratch; a problem
    // that wants a split but cannot fit even two splits' partials is rejected.
    const int64_t total = past_len + seq_len;
    AttendArgs unlimited = a;
    unlimited.workspace_floats = (size_t)1 << 60;
    int want_splits = 1, tps = 0;
    choose_splits(unlimited, total, &want_splits, &tps);
    const size_t per_split = (size_t)batch * seq_len * v.kv_heads * group * (d + 4);
    if (want_splits > 1 && 2 * per_split > kStaticScratchFloats)
        return set_error(SA_ERR_CAPACITY,
                         "gqa_attend_no_alloc: split-K partials need %zu bytes (2 splits of %zu), above the "
                         "static scratch maximum of %zu bytes",
                         2 * per_split * sizeof(float), per_split * sizeof(float), (size_t)SA_STATIC_SCRATCH_BYTES);
    int n_splits = 1;
    choose_splits(a, total, &n_splits, &tps);
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_by_dim<float>(a, n_splits, tps, static_cast<cudaStream_t>(stream));
        case SA_DTYPE_FLOAT16: return launch_by_dim<__half>(a, n_splits, tps, static_cast<cudaStream_t>(stream));
        default: return launch_by_dim<__nv_bfloat16>(a, n_splits, tps, static_cast<cudaStream_t>(stream));
    }
}

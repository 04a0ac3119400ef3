// com.microsoft.RotaryEmbedding as a standalone operator, for graphs that emit
// separate RotaryEmbedding nodes on Q and K ahead of GroupQueryAttention with
// do_rotary = 0 (onnx-rt/src/model_loader/gemma.rs:13-36; dispatched by
// dispatch_rotary_embedding, onnx-rt/src/cuda/gpu_executor.rs:814-850, onto
// rotary_gpu, onnx-rt/src/cuda/kernels/rotary.rs:274-346).
//
// Arithmetic is rotate_rope_block's (onnx-rt/src/ops/microsoft.rs:137-162):
// y0 = c*x0 - s*x1, y1 = s*x0 + c*x1, each product and sum rounded to f32 on
// its own (no fused multiply-add), so f32 outputs are bit-exact with the CPU
// op and with the RoPE the cache append and the attention prologue apply.
// Half-precision inputs are widened, rotated in f32 and rounded once.
//
// Positions.  Without position_ids, token s of a row uses table row
// start + s (the GPU executor's rule: the cache's current position, or the
// first position id, plus the token index).  With position_ids (a DEVICE
// int32/int64 array of seq_len or batch*seq_len entries) token (b, s) uses
// position_ids[s] or position_ids[b*seq_len + s] (rope_position_for,
// ops/microsoft.rs:112-120), read on the device: no host round trip.  A
// position outside the table is a device-side check failure: the row is
// passed through unrotated and bit 0 of *device_status (when given) is set.
//
// Layouts: rank-4 (B, H, S, D) and rank-3 (B, S, H*D), the two rotary_gpu
// accepts.  rotary_dim < head_dim rotates the first rotary_dim elements and
// passes the rest through (apply_rope_in_place's partial RoPE).
//
// One thread per (row, pair): pair j of a split-half row reads x[j] and
// x[j + half], so consecutive threads read consecutive words on both halves;
// interleaved rows read the adjacent pair.  The kernel is HBM-bound (a read
// and a write of every element plus a table row per token) and, at decode
// sizes, launch-latency-bound.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kRotThreads = 256;

struct RotaryArgs {
    const void *x;
    void *y;
    const void *cos_t, *sin_t;
    const void *position_ids;
    int *device_status;
    int64_t rows;           // batch * heads * seq_len
    int64_t start;          // first position when position_ids is NULL
    int64_t table_rows;
    int64_t pos_count;      // entries of position_ids
    int batch, heads, seq_len, head_dim, rotary_dim;
    int layout;             // 0: (B, H, S, D); 1: (B, S, H*D)
    int interleaved;
    int pos_is_i64;
    int per_row_items;      // rotary_dim/2 pairs + pass-through elements copied when y != x
};

template <typename TT>
__device__ __forceinline__ float table_ld(const TT *t, int64_t i) {
    return ld_f32(t + i);
}

template <typename T, typename TT>
__global__ void __launch_bounds__(kRotThreads) rotary_kernel(RotaryArgs a) {
    const T *x = static_cast<const T *>(a.x);
    T *y = static_cast<T *>(a.y);
    const TT *cs = static_cast<const TT *>(a.cos_t);
    const TT *sn = static_cast<const TT *>(a.sin_t);
    const int half = a.rotary_dim >> 1;
    const int64_t total = a.rows * a.per_row_items;
    for (int64_t i = (int64_t)blockIdx.x * kRotThreads + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * kRotThreads) {
        const int64_t row = i / a.per_row_items;
        const int j = (int)(i - row * a.per_row_items);
        const int64_t base = row * a.head_dim;
        if (j >= half) {  // pass-through element of a partial rotation (out of place only)
            const int64_t e = base + a.rotary_dim + (j - half);
            y[e] = x[e];
            continue;
        }
        int s, b;
        if (a.layout == 0) {
            s = (int)(row % a.seq_len);
            b = (int)(row / ((int64_t)a.heads * a.seq_len));
        } else {
            s = (int)((row / a.heads) % a.seq_len);
            b = (int)(row / ((int64_t)a.heads * a.seq_len));
        }
        int64_t pos;
        if (a.position_ids) {
            const int64_t pi = a.pos_count == a.seq_len ? s : (int64_t)b * a.seq_len + s;
            pos = a.pos_is_i64 ? static_cast<const int64_t *>(a.position_ids)[pi]
                               : (int64_t) static_cast<const int32_t *>(a.position_ids)[pi];
        } else {
            pos = a.start + s;
        }
        const int64_t i0 = base + (a.interleaved ? 2 * j : j);
        const int64_t i1 = base + (a.interleaved ? 2 * j + 1 : j + half);
        if (pos < 0 || pos >= a.table_rows) {
            if (a.device_status) atomicOr(a.device_status, 1);
            y[i0] = x[i0];
            y[i1] = x[i1];
            continue;
        }
        const float c = table_ld(cs, pos * half + j), sv = table_ld(sn, pos * half + j);
        const float x0 = ld_f32(x + i0), x1 = ld_f32(x + i1);
        st_from_f32(y + i0, __fsub_rn(__fmul_rn(c, x0), __fmul_rn(sv, x1)));
        st_from_f32(y + i1, __fadd_rn(__fmul_rn(sv, x0), __fmul_rn(c, x1)));
    }
}

template <typename T>
int launch_rotary_t(const RotaryArgs &a, int table_dtype, cudaStream_t stream) {
    const int64_t total = a.rows * a.per_row_items;
    int64_t blocks = (total + kRotThreads - 1) / kRotThreads;
    if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 CTAs per SM
    if (table_dtype == SA_DTYPE_BFLOAT16)
        rotary_kernel<T, __nv_bfloat16><<<(unsigned)blocks, kRotThreads, 0, stream>>>(a);
    else
        rotary_kernel<T, float><<<(unsigned)blocks, kRotThreads, 0, stream>>>(a);
    count_launch();
    return check_cuda(cudaGetLastError(), "rotary_embedding launch");
}

}  // namespace

}  // namespace sa

extern "C" {

int sa_rotary_embedding(const void *x, void *y, int32_t dtype, int32_t layout, int64_t batch, int64_t num_heads,
                        int64_t seq_len, int32_t head_dim, const void *cos_cache, const void *sin_cache,
                        int32_t table_dtype, int64_t table_rows, int32_t table_cols, const void *position_ids,
                        int32_t position_dtype, int64_t position_count, int64_t start_position,
                        int32_t interleaved, int32_t rotary_dim, int32_t *device_status, sa_stream_t stream) {
    using namespace sa;
    if (dtype != SA_DTYPE_FLOAT && dtype != SA_DTYPE_FLOAT16 && dtype != SA_DTYPE_BFLOAT16)
        return set_error(SA_ERR_UNSUPPORTED, "rotary_gpu: unsupported dtype %d (need Float, Float16 or BFloat16)",
                         dtype);
    if (table_dtype != SA_DTYPE_FLOAT && table_dtype != SA_DTYPE_BFLOAT16)
        return set_error(SA_ERR_UNSUPPORTED, "rotary_gpu: cos/sin tables must be Float or BFloat16");
    if (layout != 0 && layout != 1) return set_error(SA_ERR_SHAPE_MISMATCH, "rotary_gpu: x must be rank-3 or rank-4");
    if (batch < 0 || seq_len < 0 || num_heads <= 0)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "RotaryEmbedding: num_heads must be > 0 (got %lld)",
                         (long long)num_heads);
    if (head_dim <= 0 || head_dim % 2 != 0)
        return set_error(SA_ERR_SHAPE_MISMATCH, "rotary_gpu: head_dim must be a positive even integer");
    const int rdim = rotary_dim <= 0 ? head_dim : rotary_dim;
    if (rdim > head_dim)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "apply_rope_in_place: rotary_dim must be in 1..=head_dim");
    if (rdim % 2 != 0) return set_error(SA_ERR_INVALID_ATTRIBUTE, "apply_rope_in_place: rotary_dim must be even");
    if (table_cols != rdim / 2)
        return set_error(SA_ERR_SHAPE_MISMATCH, "apply_rope_in_place: cache inner dim %d != rotary_dim/2 = %d",
                         table_cols, rdim / 2);
    if (table_rows < 0) return set_error(SA_ERR_SHAPE_MISMATCH, "rotary_gpu: negative table length");
    const int64_t rows = batch * num_heads * seq_len;
    if (rows == 0) return SA_OK;
    if (position_ids) {
        if (position_dtype != 7 && position_dtype != 6)  // TensorProto INT64 / INT32
            return set_error(SA_ERR_SHAPE_MISMATCH, "RotaryEmbedding: position_ids must be int32 or int64");
        if (position_count != seq_len && position_count != batch * seq_len)
            return set_error(SA_ERR_SHAPE_MISMATCH, "apply_rope_in_place: position_ids length %lld != B*Sq = %lld",
                             (long long)position_count, (long long)(batch * seq_len));
    } else if (start_position < 0 || start_position + seq_len > table_rows) {
        return set_error(SA_ERR_SHAPE_MISMATCH, "rotary_gpu: position + seq_len exceeds cos/sin table length "
                         "(%lld + %lld > %lld)", (long long)start_position, (long long)seq_len,
                         (long long)table_rows);
    }
    if (!x || !y || !cos_cache || !sin_cache)
        return set_error(SA_ERR_INVALID_ARGUMENT, "rotary_embedding: NULL input, output or table");
    RotaryArgs a;
    a.x = x;
    a.y = y;
    a.cos_t = cos_cache;
    a.sin_t = sin_cache;
    a.position_ids = position_ids;
    a.device_status = device_status;
    a.rows = rows;
    a.start = start_position;
    a.table_rows = table_rows;
    a.pos_count = position_count;
    a.batch = (int)batch;
    a.heads = (int)num_heads;
    a.seq_len = (int)seq_len;
    a.head_dim = head_dim;
    a.rotary_dim = rdim;
    a.layout = layout;
    a.interleaved = interleaved ? 1 : 0;
    a.pos_is_i64 = position_dtype == 7 ? 1 : 0;
    a.per_row_items = rdim / 2 + (x != y ? head_dim - rdim : 0);
    if (batch > 0x7fffffff || seq_len > 0x7fffffff || num_heads > 0x7fffffff)
        return set_error(SA_ERR_SHAPE_MISMATCH, "rotary_embedding: dimension too large");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_rotary_t<float>(a, table_dtype, st);
        case SA_DTYPE_FLOAT16: return launch_rotary_t<__half>(a, table_dtype, st);
        default: return launch_rotary_t<__nv_bfloat16>(a, table_dtype, st);
    }
}

}  // extern "C"

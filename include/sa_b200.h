/*
 * sa_b200.h -- C ABI of the B200-native (sm_100a) LLM decode hot path of the
 * SmallAIOS onnx-rt runtime.
 *
 * The path: com.microsoft.GroupQueryAttention over a PolarQuant-compressed
 * KV cache (quantize-on-append with fused RoPE on K, attention dequantizing
 * inside the kernel) and the block-quantized int4 MatMulNBits GEMV/GEMM.
 *
 * Conventions (replacing the reference's Rust FFI, onnx-rt/src/cuda/ffi.rs):
 *   - every entry point returns an int status (sa_status); 0 is success.
 *     On failure sa_last_error_string() describes it (thread-local).
 *   - all tensor arguments are caller-owned DEVICE pointers, row-major,
 *     in the layouts onnx-rt uses ((B, S, heads*D) for Q/K/V/out).
 *   - every compute call takes an explicit CUDA stream (cudaStream_t passed
 *     as a plain pointer; NULL is the legacy default stream) and is fully
 *     asynchronous: no host synchronisation, no allocation.
 *   - dtype codes are ONNX TensorProto data types (onnx-rt/src/tensor.rs).
 *   - calls on distinct cache handles are thread-safe; calls on one handle
 *     must be serialised by the caller (the reference holds it behind a
 *     Mutex, onnx-rt/src/session.rs:377).
 */
#ifndef SA_B200_H
#define SA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SA_B200_VERSION 1

typedef void *sa_stream_t; /* cudaStream_t */

/* Status codes.  The reference maps CUDA failures to CudaError
 * (onnx-rt/src/cuda/mod.rs:51-100) and operator failures to OpError
 * (onnx-rt/src/operators.rs); the codes keep that split. */
typedef enum sa_status {
    SA_OK = 0,
    SA_ERR_INVALID_ATTRIBUTE = 1, /* OpError::InvalidAttribute */
    SA_ERR_SHAPE_MISMATCH = 2,    /* OpError::ShapeMismatch */
    SA_ERR_UNSUPPORTED = 3,       /* OpError::UnsupportedOp / unsupported dtype or layout */
    SA_ERR_CAPACITY = 4,          /* kv_cache_append:position_overflow (kv_cache.rs:246-251) */
    SA_ERR_OUT_OF_MEMORY = 5,     /* CudaError::AllocFailed */
    SA_ERR_CUDA = 6,              /* CudaError::RuntimeError / KernelLaunchFailed */
    SA_ERR_DEVICE_CHECK = 7,      /* a device-side bounds check recorded a violation */
    SA_ERR_TIMEOUT = 8,           /* a bounded device-side wait gave up */
    SA_ERR_INVALID_ARGUMENT = 9   /* NULL handle/pointer, negative size */
} sa_status;

/* ONNX TensorProto.DataType codes (onnx-rt/src/tensor.rs DataType). */
typedef enum sa_dtype {
    SA_DTYPE_FLOAT = 1,
    SA_DTYPE_FLOAT16 = 10,
    SA_DTYPE_BFLOAT16 = 16
} sa_dtype;

/* Thread-local description of the last failure on this thread. */
const char *sa_last_error_string(void);
/* Static name of a status code. */
const char *sa_status_string(int status);
/* SA_B200_VERSION of the loaded library. */
int sa_version(void);
/* Diagnostic: number of kernels this library has launched in this process
 * (all devices, all threads).  Lets a harness count its launches. */
uint64_t sa_kernel_launches(void);

/* ======================================================================
 * Compressed KV cache.
 *
 * Replaces GpuKvCache (onnx-rt/src/cuda/kv_cache.rs:111-388: allocate,
 * append, advance_position, view_pending, reset) and carries the
 * compression state of CompressedKVCache (onnx-rt/src/kv_compression.rs:
 * 742-925): one PolarQuantizer per (layer, kv_head) seeded with
 * seed * 0x9E3779B97F4A7C15 + (layer * num_kv_heads + head) (:776-779),
 * shared by K and V and by every sequence of the batch.
 *
 * Layout in HBM, per layer (b = batch row, h = local KV head, t = token,
 * CB = head_dim * bits / 8 code bytes per vector, T = capacity rounded up to
 * a multiple of 64):
 *   k_codes  uint8 [B][H][T][CB]        pack_bits order per token (bit-exact
 *                                       with PolarQuantizer::encode)
 *   v_codes  uint8 [B][H][T*CB]         the same bytes, arranged for the
 *                                       tensor-core fragments: in 16-token
 *                                       blocks of 16*CB bytes, byte j of token
 *                                       t sits at (t/16)*16*CB + (k/16)*64 +
 *                                       ((t/4)%4)*16 + k%16, k = 4*j + t%4
 *                                       (CB must be a multiple of 4)
 *   k_meta   float [B][H][T][2]         {scale, zero_point} per K vector
 *   v_meta   float [B][H][T][2]         {scale, zero_point} per V vector
 * With qjl_residual set, every append also stores the QJL residual of each
 * vector (QJLResidualEncoder::encode, kv_compression.rs:365-395, of the
 * input against PolarQuantizer::decode of its own codes, as write_kv does at
 * :826-840), bit-exact:
 *   k_qjl_bits / v_qjl_bits  uint8 [B][H][T][D/8]  sign bits, bit i of the
 *                                       vector = bit i%8 of byte i/8 (1 when
 *                                       residual i >= 0): the bytes of the
 *                                       reference's little-endian u64 words
 *   k_qjl_mag  / v_qjl_mag   float [B][H][T]       c_magnitude = sum|r| / D
 * The reference never reads them back (read_k / read_v, :862-899), and
 * neither does attention here.
 * With lowrank_k > 0 (KVCacheConfig::kv_lowrank_k) the cache also keeps the
 * low-rank K state of LowRankKeyDecomposer (:451-671), bit-exact, as
 * write_kv builds it (:842-853): the first K row of a sequence is decomposed
 * alone, so the rank is min(lowrank_k, 1, D) = 1 from then on; every later
 * row appends its projection, and every 512th update re-decomposes the
 * reconstruction by power iteration:
 *   lr_vt  float [B][H][D]   the rank-1 V^T row
 *   lr_us  float [B][H][T]   U*S, one coefficient per written row
 * read_k then returns the reconstruction lr_us[t] * lr_vt (:862-886), so
 * attention on such a cache scores keys as lr_us[t] * (q . lr_vt); V still
 * comes from the PolarQuant codes.  The attention kernels get this from the
 * same identity they use for the codes, q.k = scale*(q'.c) + zp*sum(q'):
 * with {scale 0, zp lr_us[t]} as K metadata (lr_kmeta) and q'.lr_vtr in
 * place of sum(q').  The state follows writes in position order from 0;
 * rewinding below a re-decomposition point is not supported.
 * ====================================================================== */
typedef struct sa_kv_cache sa_kv_cache;

typedef struct sa_kv_cache_config {
    int32_t num_layers;    /* KVCacheConfig::num_layers */
    int32_t batch;         /* sequences decoded together (the reference is batch 1) */
    int32_t num_heads;     /* query heads of the model (sizes the split-K workspace) */
    int32_t num_kv_heads;  /* KVCacheConfig::num_kv_heads, model total */
    int32_t kv_head_begin; /* first KV head held here (KV-head sharding); 0 if unsharded */
    int32_t kv_head_count; /* KV heads held here; num_kv_heads if unsharded */
    int32_t head_dim;      /* KVCacheConfig::head_dim: power of two, 16..256 */
    int32_t max_seq_len;   /* GpuKvCache::max_seq_len */
    int32_t bits;          /* KVCacheConfig::kv_quant_bits: 3, 4 or 8 */
    uint64_t seed;         /* KVCacheConfig::seed (default 0xDEADBEEFCAFE1234) */
    int32_t qjl_residual;  /* KVCacheConfig::kv_qjl_residual: nonzero stores QJL residuals */
    int32_t lowrank_k;     /* KVCacheConfig::kv_lowrank_k: 0 = None, > 0 keeps low-rank K */
} sa_kv_cache_config;

/* Raw device pointers of one layer (GpuKvCache::view_at, kv_cache.rs:336-378). */
typedef struct sa_kv_layer_view {
    uint8_t *k_codes;
    uint8_t *v_codes;
    float *k_meta;
    float *v_meta;
    const float *signs;        /* [H][D] the +-1 sign vector of each local head, as float */
    int32_t batch;
    int32_t kv_heads;          /* local heads H */
    int32_t head_dim;
    int32_t bits;
    int32_t code_bytes;        /* CB */
    int32_t capacity;          /* T (padded capacity, tokens) */
    float wht_scale;           /* 1 / sqrt_approx(head_dim), kv_compression.rs:100 */
    uint8_t *k_qjl_bits;       /* QJL residual sign bits, NULL unless qjl_residual */
    uint8_t *v_qjl_bits;
    float *k_qjl_mag;          /* QJL residual c_magnitude, NULL unless qjl_residual */
    float *v_qjl_mag;
    float *lr_vt;              /* low-rank K state, NULL unless lowrank_k (attention then uses it) */
    float *lr_us;
    float *lr_kmeta;           /* [B][H][T][2] {0, lr_us[t]}: the K metadata attention reads */
    float *lr_vtr;             /* [B][H][D] lr_vt rotated like the queries (signs, WHT, 1/sqrt(n)) */
} sa_kv_layer_view;

/* GpuKvCache::allocate (kv_cache.rs:129-193) + CompressedKVCache::new
 * (kv_compression.rs:766-807).  Allocates every layer and the split-K
 * workspace on the current device, zero-filled.  This is the only call that
 * allocates device memory. */
int sa_kv_cache_create(const sa_kv_cache_config *config, sa_kv_cache **out);
/* Frees the cache (DeviceBuffer drop, onnx-rt/src/cuda/memory.rs). NULL is ok. */
int sa_kv_cache_destroy(sa_kv_cache *cache);
/* GpuKvCache::reset (kv_cache.rs:386): position back to 0, memory kept. */
int sa_kv_cache_reset(sa_kv_cache *cache);
/* GpuKvCache::current_position (kv_cache.rs:201). */
int sa_kv_cache_position(const sa_kv_cache *cache, int64_t *position);
/* Rewind or move the committed position (0 <= position <= max_seq_len). */
int sa_kv_cache_set_position(sa_kv_cache *cache, int64_t position);
/* GpuKvCache::advance_position (kv_cache.rs:281), by n tokens. */
int sa_kv_cache_advance(sa_kv_cache *cache, int64_t n);
/* The layer's device pointers and layout. */
int sa_kv_cache_layer_view(const sa_kv_cache *cache, int32_t layer, sa_kv_layer_view *view);
/* Head-sharded output (one rank of a KV-head-sharded layer).  Afterwards every
 * attention call on `cache` stores the output of this rank's query heads into
 * each of the `n` buffers -- this GPU's and its peers', all addressable from
 * this process (IPC / virtual-memory peer mappings) -- at columns
 * [q_head_offset*D, (q_head_offset + q_local)*D) of a [batch][seq_len]
 * [q_heads_total*D] tensor, instead of writing attn_out (whose contents are
 * then unspecified).  This replaces the all-gather of attn_out that follows
 * the local operator in the head-sharded mode: the decode kernel's epilogue
 * writes every rank's copy over NVLink.  q_heads_total must equal the cache's
 * num_heads and q_head_offset its kv_head_begin * group.  n = 0 turns it off.
 * At most 8 buffers.
 *
 * Completing the gather.  With signals == NULL the caller runs a cross-rank
 * barrier after each call before any rank reads its buffer.  With `signals`
 * (rank i's array of 10 uint32 words, zeroed before first use and mapped
 * here like the buffers; this rank is index `rank`), the writing kernel
 * completes it on the device: its last CTA publishes a step epoch into every
 * peer's array (st.release.sys over NVLink) and waits until every peer has
 * published it into this rank's (ld.acquire.sys), so the kernels that follow
 * on the stream see the whole gathered tensor -- no host barrier, no extra
 * launch, and a CUDA graph of the step stays valid (the epoch lives on the
 * device).  The wait is bounded by timeout_us: when it runs out the kernel
 * sets bit 0 of the device status (sa_kv_cache_device_status) and returns.
 * Either way every rank makes the same calls in the same order, and
 * alternates buffers between steps (at least two) so that no rank writes a
 * buffer a peer may still be reading.  This has no counterpart in the
 * reference, which runs on one device (onnx-rt/src/cuda/mod.rs:653-690). */
int sa_kv_cache_set_gather(sa_kv_cache *cache, void *const *buffers, uint32_t *const *signals, int32_t n,
                           int32_t rank, int32_t q_head_offset, int32_t q_heads_total, int64_t timeout_us);
/* Copy of the cache configuration. */
int sa_kv_cache_get_config(const sa_kv_cache *cache, sa_kv_cache_config *config);
/* CompressedKVCache::memory_bytes (kv_compression.rs:928-957) of the rows
 * written so far, summed over the batch's sequences and the KV heads held
 * here (the reference's per-block accounting, :166-168, :352-354, :442-444),
 * and the bytes this cache holds on the device.  Either pointer may be NULL. */
int sa_kv_cache_memory_bytes(const sa_kv_cache *cache, uint64_t *reference_bytes, uint64_t *device_bytes);
/* Device-side status of the kernels that used this cache: 0, or bit 0 set when
 * a bounded wait inside a kernel gave up (the kernel then stopped and its
 * output is not valid).  Synchronises with the device; `clear` resets it.
 * The reference has no device-side waits; this reports the safety net that
 * replaces a hang. */
int sa_kv_cache_device_status(sa_kv_cache *cache, int32_t *status, int32_t clear);

/* Quantize-on-append: GpuKvCache::append (kv_cache.rs:233-277) fused with
 * CompressedKVCache::write_kv (kv_compression.rs:814-854) and with the K half of
 * gqa_apply_rotary (ops/microsoft.rs:1004-1050).  With the cache's qjl_residual
 * option it also stores each vector's QJL residual (:826-840), and with
 * lowrank_k it updates the low-rank K state (:842-853), as write_kv does.
 *
 * key/value: (batch, seq_len, kv_head_count * head_dim) in `dtype`.  Token s
 * is written at position (cache position + s); RoPE on K uses that position
 * as the cos/sin row.  The codes, scale and zero_point of every vector are
 * bit-exact with PolarQuantizer::encode applied to the f32 value of the
 * (rotated) input.  Does not advance the position. */
int sa_kv_append(sa_kv_cache *cache, int32_t layer, const void *key, const void *value,
                 int32_t dtype, int32_t batch, int32_t seq_len,
                 const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                 int32_t do_rotary, int32_t rotary_interleaved, sa_stream_t stream);

/* Attention of seq_len query tokens over the compressed cache: query token s
 * sits at position p + s (p = cache position) and attends causally to cache
 * tokens [0, p + s] -- scaled_dot_product_attention with causal mask and
 * past_sk = p (ops/microsoft.rs:380-438), reading K/V through
 * PolarQuantizer::decode semantics (computed in the rotated domain).
 *
 * query/attn_out: (batch, seq_len, q_heads_local * head_dim), q_heads_local =
 * (num_heads / num_kv_heads) * kv_head_count.  RoPE is applied to the query
 * in the kernel prologue when do_rotary is set.  has_scale selects the
 * `scale` attribute, else 1/sqrt(head_dim) (sqrt_f32, ops/microsoft.rs:54).
 * Positions beyond the appended tokens are never read. */
int sa_gqa_attend(sa_kv_cache *cache, int32_t layer, const void *query, void *attn_out,
                  int32_t dtype, int32_t batch, int32_t seq_len, int64_t num_heads,
                  int32_t has_scale, float scale,
                  const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                  int32_t do_rotary, int32_t rotary_interleaved, sa_stream_t stream);

/* The operator: com.microsoft.GroupQueryAttention with the cache as past
 * K/V -- op_group_query_attention (ops/microsoft.rs:1082-1196) as the GPU
 * executor dispatches it with a cache (dispatch_gqa / gqa_with_cache,
 * onnx-rt/src/cuda/gpu_executor.rs:917-968): validates the attributes like
 * gqa_validate (:933-985), appends key/value (sa_kv_append) and runs
 * sa_gqa_attend.  num_heads / kv_num_heads are the node attributes (model
 * totals).  local_window_size must be -1 (the CPU op rejects windows,
 * ops/microsoft.rs:1089-1094).  Only attn_out is produced: present K/V live in
 * the cache (gpu_executor.rs:965-967).  Does not advance the position. */
int sa_group_query_attention(sa_kv_cache *cache, int32_t layer,
                             const void *query, const void *key, const void *value,
                             void *attn_out, int32_t dtype, int32_t batch, int32_t seq_len,
                             int64_t num_heads, int64_t kv_num_heads,
                             int32_t has_scale, float scale, int64_t local_window_size,
                             int32_t do_rotary, int32_t rotary_interleaved,
                             const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                             sa_stream_t stream);

/* Allocation-free variant of sa_gqa_attend.  It has no counterpart in the
 * reference.
 *
 * It serves callers that may not allocate device memory while they run.
 * Examples are a real-time partition that reserves every buffer at start-up
 * so that an inference step has a bounded, failure-free footprint, or a host
 * whose memory belongs to its own pool.  sa_gqa_attend needs a cache handle,
 * and that handle owns a library-allocated split-K workspace.  This call
 * instead reads the caller's cache buffers, described by `layer` in the
 * layout documented above (for example filled by sa_kv_cache_layer_view, or
 * pointing into memory the caller manages).  It keeps its split-K partials
 * in a fixed array of SA_STATIC_SCRATCH_BYTES that the library's CUDA module
 * reserves on every GPU that loads it, until the process exits.  It calls no
 * cudaMalloc, cudaFree or allocating routine.
 *
 *   - past_len tokens are cached before query token 0.  Query token s attends
 *     to [0, past_len + s].  group = query heads per KV head (1..8).  The other
 *     arguments mean what they mean for sa_gqa_attend.
 *   - The first call on each device resolves the array's device address
 *     (cudaGetSymbolAddress) with that device current.  Make that first call
 *     before any stream capture.
 *   - Limit: the partials take batch * seq_len * kv_heads * group *
 *     (head_dim + 4) floats per split.  The call uses as many splits as fit.
 *     When the problem wants splits and two do not fit, it returns
 *     SA_ERR_CAPACITY with the sizes in sa_last_error_string().
 *   - Every call on a device shares the one array, and the array keeps the
 *     last call's contents.  Each call writes every partial before it reads
 *     it, so nothing needs clearing.  Calls that overlap on the GPU (other
 *     streams or threads) race on it: serialise them. */
#define SA_STATIC_SCRATCH_BYTES (8u << 20)
int sa_gqa_attend_no_alloc(const sa_kv_layer_view *layer, int64_t past_len, const void *query,
                           void *attn_out, int32_t dtype, int32_t batch, int32_t seq_len,
                           int32_t group, int32_t has_scale, float scale,
                           const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                           int32_t do_rotary, int32_t rotary_interleaved, sa_stream_t stream);

/* ======================================================================
 * MatMulNBits (ONNX Runtime com.microsoft.MatMulNBits contract; absent from
 * the reference, which would register it next to MatMul in
 * dispatch_gpu_node, onnx-rt/src/cuda/gpu_executor.rs:490-514).
 *
 *   a            (m, k) in dtype
 *   b            uint8 (n, ceil(k/block_size), block_size*bits/8), low nibble first
 *   scales       (n, ceil(k/block_size)) in dtype
 *   zero_points  NULL (=> 2^(bits-1)) or uint8 (n, ceil(ceil(k/block_size)*bits/8)), packed
 *   bias         NULL or (n) in dtype
 *   y            (m, n) in dtype
 * y[i][j] = sum_k a[i][k] * (code[j][k] - zp[j][k/bs]) * scale[j][k/bs] (+ bias[j]),
 * accumulated in f32.  bits must be 4; block_size a power of two >= 16.
 * b and scales are weights (ONNX initializers): the 16-bit tensor-core kernels
 * are programmatic dependent launches that start streaming them before the
 * kernel ahead of them on the stream has finished, so no kernel enqueued just
 * before the call may still be writing them (a copy or a synchronised stream
 * is fine).  a, bias and y are only touched after that kernel completes.
 * ====================================================================== */
int sa_matmul_nbits(const void *a, const uint8_t *b, const void *scales,
                    const uint8_t *zero_points, const void *bias, void *y,
                    int32_t dtype, int64_t m, int64_t n, int64_t k,
                    int32_t bits, int32_t block_size, sa_stream_t stream);

/* Prepacked MatMulNBits weights (decode, m <= 8).  Model weights are
 * constant, so the host repacks each one once at load time -- as ONNX
 * Runtime's MatMulNBits PrePack does -- into a layout whose every chunk the
 * kernel streams is one contiguous 9 KB run: per 32 output columns and per
 * 512 k, the columns' codes (pre-swizzled for conflict-free fragment loads)
 * followed by their scales.  Supported: 4-bit codes, block 32, fp16/bf16
 * scales and activations, default zero point (8), n a multiple of 32 and k a
 * multiple of 1024.
 *
 * sa_matmul_nbits_packed_bytes: size of the packed form; 0 if the shape,
 * dtype or block size has no packed path.
 * sa_matmul_nbits_prepack: writes the packed form of (b, scales) -- the same
 * arguments as sa_matmul_nbits -- into `packed` (16-byte aligned, device).
 * sa_matmul_nbits_packed: y = a . dequant(b)^T (+ bias) from the packed form;
 * same numerics as sa_matmul_nbits (exact products, f32 accumulate). */
int64_t sa_matmul_nbits_packed_bytes(int64_t n, int64_t k, int32_t bits, int32_t block_size, int32_t dtype);
int sa_matmul_nbits_prepack(const uint8_t *b, const void *scales, void *packed, int32_t dtype,
                            int64_t n, int64_t k, int32_t bits, int32_t block_size, sa_stream_t stream);
int sa_matmul_nbits_packed(const void *a, const void *packed, const void *bias, void *y, int32_t dtype,
                           int64_t m, int64_t n, int64_t k, int32_t bits, int32_t block_size,
                           sa_stream_t stream);

/* Fused QKV projection of a decode step: MatMulNBits + RotaryEmbedding +
 * quantize-on-append in one operator.  It replaces the node sequence the
 * reference's graph runs before the attention proper: the Q/K/V MatMulNBits
 * projections, then the rotary and present-K/V concat of
 * op_group_query_attention (onnx-rt/src/ops/microsoft.rs:1082-1196, rotary
 * :1004-1050, kv_concat :762-794), with the rotary in the projection's
 * epilogue.
 *
 *   x         (batch, hidden) activations, fp16 or bf16 (one token per row)
 *   w_codes   packed QKV weights, uint8 (n, hidden/32, 16), n = (Hq + 2*Hkv)*D:
 *             rows [0, Hq*D) are Wq, then Hkv*D rows of Wk, then Wv; Hq, Hkv
 *             are this cache's heads (its KV-head shard and their query heads)
 *   w_scales  (n, hidden/32) in dtype; block 32, default zero point 8
 *   q_out     (batch, Hq*D): x.Wq^T rounded to dtype, then RoPE at the cache
 *             position (when do_rotary), rounded to dtype
 *   k_out, v_out  (batch, Hkv*D): x.Wk^T, x.Wv^T rounded to dtype (no RoPE)
 * and appends RoPE(k_out) (when do_rotary) and v_out to `layer` at the cache
 * position, bit-exact with sa_kv_append of (k_out, v_out).  The position is
 * not advanced (sa_kv_cache_advance after the step).  Attention then runs
 * with sa_gqa_attend(q_out, do_rotary = 0).  batch 17..128 with
 * Hq*D and Hkv*D multiples of 128 and hidden a multiple of 256 is one
 * tcgen05 launch whose epilogue does the rotary and the append; other shapes
 * run the three projections, then one epilogue launch. */
int sa_qkv_project_append(sa_kv_cache *cache, int32_t layer, const void *x, const uint8_t *w_codes,
                          const void *w_scales, int32_t dtype, int32_t batch, int64_t hidden,
                          const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                          int32_t do_rotary, int32_t rotary_interleaved, void *q_out, void *k_out,
                          void *v_out, sa_stream_t stream);

/* ======================================================================
 * Decoder-layer glue (the ops around GQA and MatMulNBits in a decoder
 * layer, onnx-rt/src/model_loader/gemma.rs:13-36).
 *
 * sa_rms_norm: com.microsoft.SkipSimplifiedLayerNormalization
 * (onnx-rt/src/ops/microsoft.rs:491-540) over rows of `cols`:
 *   pre = x + skip (+ bias);  y = pre / sqrt(mean(pre^2) + epsilon) * weight
 * with f32 arithmetic.  skip == NULL gives SimplifiedLayerNormalization /
 * RMSNormalization (microsoft.rs:447-480, generative.rs:517-580); `pre`
 * may be NULL (not stored).  x, skip, y, pre: (rows, cols); weight, bias:
 * (cols), all of dtype.
 *
 * sa_silu_mul: SwiGLU, Silu(gate) * up (GraphBuilder::swiglu,
 * graph_builder.rs:366-369): y[r][j] = gate[r][j] / (1 + exp(-gate[r][j])) *
 * up[r][j], gate and up rows `ld_in` elements apart (ld_in = cols for
 * separate tensors, 2*cols for one packed gate|up projection), y (rows, cols).
 * ====================================================================== */
int sa_rms_norm(const void *x, const void *skip, const void *bias, const void *weight, void *y, void *pre,
                int32_t dtype, int64_t rows, int64_t cols, float epsilon, sa_stream_t stream);
int sa_silu_mul(const void *gate, const void *up, int64_t ld_in, void *y, int32_t dtype, int64_t rows,
                int64_t cols, sa_stream_t stream);

/* ======================================================================
 * com.microsoft.RotaryEmbedding as its own node: replaces dispatch_rotary_
 * embedding -> rotary_gpu (onnx-rt/src/cuda/gpu_executor.rs:814-850,
 * onnx-rt/src/cuda/kernels/rotary.rs:274-346) for graphs that rotate Q and
 * K in separate RotaryEmbedding nodes ahead of GroupQueryAttention with
 * do_rotary = 0 (onnx-rt/src/model_loader/gemma.rs:13-36).
 *
 * x, y: layout 0 = (batch, num_heads, seq_len, head_dim) (rank 4), layout 1 =
 * (batch, seq_len, num_heads * head_dim) (rank 3); y may equal x (in place).
 * Tables cos/sin: (table_rows, table_cols) of table_dtype (Float, or BFloat16
 * widened in the kernel as the executor's cast does), table_cols =
 * rotary_dim / 2.  rotary_dim <= 0 means head_dim; elements at or past
 * rotary_dim pass through (apply_rope_in_place, ops/microsoft.rs:190-231).
 * Pairs (x[i], x[i + rotary_dim/2]), or (x[2i], x[2i+1]) when interleaved;
 * y0 = c*x0 - s*x1, y1 = s*x0 + c*x1 with every product and sum rounded to
 * f32 (rotate_rope_block, ops/microsoft.rs:137-162), so f32 outputs are
 * bit-exact with the CPU op.
 *
 * Positions: with position_ids == NULL, token s uses table row
 * start_position + s (the executor passes the cache's current position:
 * pick_rotary_position, gpu_executor.rs:761-773; the caller checks
 * start_position + seq_len <= table_rows on the host, no D2H read).  With a
 * DEVICE position_ids array of position_dtype INT64 (7) or INT32 (6) and
 * position_count = seq_len or batch * seq_len entries, token (b, s) uses
 * position_ids[s] or position_ids[b * seq_len + s] (rope_position_for,
 * ops/microsoft.rs:112-120); the reference GPU path reads only the first id
 * back to the host instead.  A position id outside [0, table_rows) cannot be
 * reported by the call's status: that row is passed through unrotated and
 * bit 0 of *device_status is set when device_status (a device int) is given.
 * ====================================================================== */
int sa_rotary_embedding(const void *x, void *y, int32_t dtype, int32_t layout, int64_t batch, int64_t num_heads,
                        int64_t seq_len, int32_t head_dim, const void *cos_cache, const void *sin_cache,
                        int32_t table_dtype, int64_t table_rows, int32_t table_cols, const void *position_ids,
                        int32_t position_dtype, int64_t position_count, int64_t start_position,
                        int32_t interleaved, int32_t rotary_dim, int32_t *device_status, sa_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SA_B200_H */

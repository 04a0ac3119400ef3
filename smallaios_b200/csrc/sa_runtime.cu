// Host runtime of libsa_b200: error reporting, the compressed KV cache
// (GpuKvCache / CompressedKVCache replacement) and argument validation of
// every C-ABI entry point.  Kernels live in the other translation units.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

static thread_local char g_err[512] = "no error";
static unsigned long long g_launches = 0;

void count_launch(int n) { __atomic_fetch_add(&g_launches, (unsigned long long)n, __ATOMIC_RELAXED); }

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return status;
}

int check_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return SA_OK;
    if (e == cudaErrorMemoryAllocation)
        return set_error(SA_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return set_error(SA_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

// operators.rs:3311-3320, computed on the host in f32 exactly as the
// reference does (each operation rounded to f32).
float host_sqrt_approx(float x) {
    if (x <= 0.0f) return 0.0f;
    volatile float s = x;
    for (int i = 0; i < 10; i++) {
        volatile float q = x / s;
        volatile float t = s + q;
        s = 0.5f * t;
    }
    return s;
}

// ops/microsoft.rs:54-62 sqrt_f32 (16 Newton steps).
float host_sqrt_f32(float x) {
    if (x <= 0.0f) return 0.0f;
    volatile float g = x;
    for (int i = 0; i < 16; i++) {
        volatile float q = x / g;
        volatile float t = g + q;
        g = 0.5f * t;
    }
    return g;
}

// Xorshift64 (kv_compression.rs:44-68) and the PolarQuantizer sign draw
// (:207-210), seeded per (layer, head) as CompressedKVCache::new (:776-779).
static void make_signs(uint64_t seed, int dim, float *out) {
    uint64_t st = seed == 0 ? 0x5EEDDEADBEEFCAFEULL : seed;
    for (int i = 0; i < dim; i++) {
        uint64_t x = st;
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        st = x;
        out[i] = (x & 1) == 0 ? 1.0f : -1.0f;
    }
}

int launch_gqa_attend_generic(const AttendArgs &a, cudaStream_t stream);


}  // namespace sa

using namespace sa;

extern "C" {

const char *sa_last_error_string(void) { return g_err; }

const char *sa_status_string(int status) {
    switch (status) {
        case SA_OK: return "SA_OK";
        case SA_ERR_INVALID_ATTRIBUTE: return "SA_ERR_INVALID_ATTRIBUTE";
        case SA_ERR_SHAPE_MISMATCH: return "SA_ERR_SHAPE_MISMATCH";
        case SA_ERR_UNSUPPORTED: return "SA_ERR_UNSUPPORTED";
        case SA_ERR_CAPACITY: return "SA_ERR_CAPACITY";
        case SA_ERR_OUT_OF_MEMORY: return "SA_ERR_OUT_OF_MEMORY";
        case SA_ERR_CUDA: return "SA_ERR_CUDA";
        case SA_ERR_DEVICE_CHECK: return "SA_ERR_DEVICE_CHECK";
        case SA_ERR_TIMEOUT: return "SA_ERR_TIMEOUT";
        case SA_ERR_INVALID_ARGUMENT: return "SA_ERR_INVALID_ARGUMENT";
        default: return "SA_ERR_UNKNOWN";
    }
}

int sa_version(void) { return SA_B200_VERSION; }

uint64_t sa_kernel_launches(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

static bool is_pow2(int n) { return n > 0 && (n & (n - 1)) == 0; }

int sa_kv_cache_create(const sa_kv_cache_config *cfg, sa_kv_cache **out) {
    if (!cfg || !out) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_create: NULL argument");
    *out = nullptr;
    const sa_kv_cache_config c = *cfg;
    // GpuKvCache::allocate zero_dim check (kv_cache.rs:147-152).
    if (c.num_layers <= 0 || c.batch <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 0 || c.max_seq_len <= 0)
        return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_allocate:zero_dim");
    // PolarQuantizer::new asserts (kv_compression.rs:197-205).
    if (!is_pow2(c.head_dim)) return set_error(SA_ERR_INVALID_ATTRIBUTE, "dim must be a power of two");
    if (c.bits != 3 && c.bits != 4 && c.bits != 8)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "bits must be 3, 4, or 8");
    if (c.head_dim < 16 || c.head_dim > 256)
        return set_error(SA_ERR_UNSUPPORTED, "kv_cache_create: head_dim %d outside 16..256", c.head_dim);
    if ((c.head_dim * c.bits / 8) % 4 != 0)
        return set_error(SA_ERR_UNSUPPORTED, "kv_cache_create: head_dim %d at %d bits packs to %d bytes, not a "
                         "multiple of 4 (the V layout interleaves 4-byte words)", c.head_dim, c.bits,
                         c.head_dim * c.bits / 8);
    if (c.num_heads <= 0 || c.num_heads % c.num_kv_heads != 0)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "num_heads must be a positive multiple of num_kv_heads");
    if (c.kv_head_count <= 0 || c.kv_head_begin < 0 || c.kv_head_begin + c.kv_head_count > c.num_kv_heads)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "kv head range [%d, %d) outside [0, %d)", c.kv_head_begin,
                         c.kv_head_begin + c.kv_head_count, c.num_kv_heads);
    if (c.lowrank_k < 0) return set_error(SA_ERR_INVALID_ATTRIBUTE, "kv_lowrank_k must be >= 0 (0 = None)");
    if ((int64_t)c.max_seq_len > (int64_t)0x7fffffff - kCapacityAlign)
        return set_error(SA_ERR_INVALID_ARGUMENT, "max_seq_len too large");

    kv_cache_impl *k = new kv_cache_impl();
    memset(k, 0, sizeof(*k));
    k->cfg = c;
    if (cudaGetDevice(&k->device) != cudaSuccess) {
        delete k;
        return check_cuda(cudaGetLastError(), "cudaGetDevice");
    }
    cudaDeviceGetAttribute(&k->sm_count, cudaDevAttrMultiProcessorCount, k->device);
    if (k->sm_count <= 0) k->sm_count = 148;
    k->capacity = (c.max_seq_len + kCapacityAlign - 1) / kCapacityAlign * kCapacityAlign;
    k->code_bytes = c.head_dim * c.bits / 8;
    k->group = c.num_heads / c.num_kv_heads;
    k->wht_scale = 1.0f / host_sqrt_approx((float)c.head_dim);
    const size_t L = c.num_layers, B = c.batch, H = c.kv_head_count, T = k->capacity, D = c.head_dim;
    k->layer_codes_bytes = B * H * T * k->code_bytes;
    k->layer_meta_floats = B * H * T * 2;
    k->workspace_floats = B * H * (size_t)kMaxSplits * k->group * (D + 4);
    const size_t dec_ws = decode_workspace_floats(k->sm_count, (int64_t)(B * H), (int)D, k->group);
    if (dec_ws > k->workspace_floats) k->workspace_floats = dec_ws;
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t codes = up(L * k->layer_codes_bytes);
    const size_t meta = up(L * k->layer_meta_floats * sizeof(float));
    const size_t signs = up(L * H * D * sizeof(float));
    const size_t ws = up(k->workspace_floats * sizeof(float));
    const size_t qp = up(B * H * decode_qprep_words(k->group) * sizeof(uint32_t));
    const size_t st = 256;
    // QJL residuals (KVCacheConfig::kv_qjl_residual): D/8 sign bytes and one magnitude per vector
    k->layer_qjl_bytes = c.qjl_residual ? B * H * T * (D / 8) : 0;
    k->layer_qjl_floats = c.qjl_residual ? B * H * T : 0;
    const size_t qjl_bits = up(L * k->layer_qjl_bytes);
    const size_t qjl_mag = up(L * k->layer_qjl_floats * sizeof(float));
    // low-rank K (KVCacheConfig::kv_lowrank_k): V^T row, U*S column and the power iteration's u
    k->layer_lr_vt_floats = c.lowrank_k > 0 ? B * H * D : 0;
    k->layer_lr_us_floats = c.lowrank_k > 0 ? B * H * T : 0;
    const size_t lr_vt = up(L * k->layer_lr_vt_floats * sizeof(float));
    const size_t lr_us = up(L * k->layer_lr_us_floats * sizeof(float));
    k->base_bytes = 2 * codes + 2 * meta + signs + ws + qp + st + 2 * qjl_bits + 2 * qjl_mag + 2 * lr_vt + 4 * lr_us;
    const size_t k_bytes = k->base_bytes;
    cudaError_t e = cudaMalloc(&k->base, k->base_bytes);
    if (e != cudaSuccess) {
        delete k;
        cudaGetLastError();
        return set_error(SA_ERR_OUT_OF_MEMORY, "kv_cache_create: cudaMalloc(%zu bytes) failed: %s",
                         k_bytes, cudaGetErrorString(e));
    }
    uint8_t *p = static_cast<uint8_t *>(k->base);
    k->k_codes = p;
    p += codes;
    k->v_codes = p;
    p += codes;
    k->k_meta = reinterpret_cast<float *>(p);
    p += meta;
    k->v_meta = reinterpret_cast<float *>(p);
    p += meta;
    k->signs = reinterpret_cast<float *>(p);
    p += signs;
    k->workspace = reinterpret_cast<float *>(p);
    p += ws;
    k->qprep = reinterpret_cast<uint32_t *>(p);
    p += qp;
    k->dev_status = reinterpret_cast<int *>(p);
    p += st;
    if (c.qjl_residual) {
        k->k_qjl_bits = p;
        p += qjl_bits;
        k->v_qjl_bits = p;
        p += qjl_bits;
        k->k_qjl_mag = reinterpret_cast<float *>(p);
        p += qjl_mag;
        k->v_qjl_mag = reinterpret_cast<float *>(p);
        p += qjl_mag;
    }
    if (c.lowrank_k > 0) {
        k->lr_vt = reinterpret_cast<float *>(p);
        p += lr_vt;
        k->lr_us = reinterpret_cast<float *>(p);
        p += lr_us;
        k->lr_scratch = reinterpret_cast<float *>(p);
        p += lr_us;
        k->lr_kmeta = reinterpret_cast<float *>(p);  // two floats per row: 2 * lr_us bytes
        p += 2 * lr_us;
        k->lr_vtr = reinterpret_cast<float *>(p);
    }
    // Zero-initialise like GpuKvCache::allocate (kv_cache.rs:171-175).
    e = cudaMemset(k->base, 0, k->base_bytes);
    if (e == cudaSuccess) {
        std::vector<float> hs(L * H * D);
        for (size_t l = 0; l < L; l++)
            for (size_t h = 0; h < H; h++) {
                const uint64_t hseed = c.seed * 0x9E3779B97F4A7C15ULL +
                                       (uint64_t)(l * (uint64_t)c.num_kv_heads + (uint64_t)(c.kv_head_begin + h));
                make_signs(hseed, (int)D, &hs[(l * H + h) * D]);
            }
        e = cudaMemcpy(k->signs, hs.data(), hs.size() * sizeof(float), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        int rc = check_cuda(e, "kv_cache_create init");
        cudaFree(k->base);
        delete k;
        return rc;
    }
    *out = reinterpret_cast<sa_kv_cache *>(k);
    return SA_OK;
}

int sa_kv_cache_destroy(sa_kv_cache *cache) {
    if (!cache) return SA_OK;
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != k->device) cudaSetDevice(k->device);
    cudaError_t e = cudaFree(k->base);
    if (dev >= 0 && dev != k->device) cudaSetDevice(dev);
    delete k;
    return check_cuda(e, "kv_cache_destroy cudaFree");
}

int sa_kv_cache_reset(sa_kv_cache *cache) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_reset: NULL cache");
    reinterpret_cast<kv_cache_impl *>(cache)->position = 0;
    return SA_OK;
}

int sa_kv_cache_position(const sa_kv_cache *cache, int64_t *position) {
    if (!cache || !position) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_position: NULL argument");
    *position = reinterpret_cast<const kv_cache_impl *>(cache)->position;
    return SA_OK;
}

int sa_kv_cache_set_position(sa_kv_cache *cache, int64_t position) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_position: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    if (position < 0 || position > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "kv_cache_set_position: %lld outside [0, %d]", (long long)position,
                         k->cfg.max_seq_len);
    k->position = position;
    return SA_OK;
}

int sa_kv_cache_advance(sa_kv_cache *cache, int64_t n) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_advance: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    if (n < 0 || k->position + n > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "kv_cache_advance:position_overflow");
    k->position += n;
    return SA_OK;
}

int sa_kv_cache_device_status(sa_kv_cache *cache, int32_t *status, int32_t clear) {
    if (!cache || !status) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_device_status: NULL argument");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    int v = 0;
    int rc = check_cuda(cudaMemcpy(&v, k->dev_status, sizeof(int), cudaMemcpyDeviceToHost),
                        "kv_cache_device_status read");
    if (rc != SA_OK) return rc;
    *status = v;
    if (clear && v) rc = check_cuda(cudaMemset(k->dev_status, 0, sizeof(int)), "kv_cache_device_status clear");
    return rc;
}

int sa_kv_cache_set_gather(sa_kv_cache *cache, void *const *buffers, uint32_t *const *signals, int32_t n,
                           int32_t rank, int32_t q_head_offset, int32_t q_heads_total, int64_t timeout_us) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    if (n == 0) {
        k->gather = GatherOut{};
        return SA_OK;
    }
    if (n < 0 || n > kMaxGather || !buffers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: %d buffers (1..%d)", n, kMaxGather);
    const int local_q = k->cfg.kv_head_count * k->group;
    if (q_heads_total != k->cfg.num_heads || q_head_offset < 0 || q_head_offset + local_q > q_heads_total ||
        q_head_offset != k->cfg.kv_head_begin * k->group)
        return set_error(SA_ERR_SHAPE_MISMATCH,
                         "kv_cache_set_gather: query heads [%d, %d) of %d do not match the cache's KV heads "
                         "[%d, %d) of %d",
                         q_head_offset, q_head_offset + local_q, q_heads_total, k->cfg.kv_head_begin,
                         k->cfg.kv_head_begin + k->cfg.kv_head_count, k->cfg.num_kv_heads);
    GatherOut g{};
    for (int i = 0; i < n; i++) {
        if (!buffers[i]) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: NULL buffer %d", i);
        g.p[i] = buffers[i];
    }
    if (signals) {
        if (rank < 0 || rank >= n)
            return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: rank %d outside %d buffers", rank, n);
        if (timeout_us <= 0)
            return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: timeout must be > 0 (got %lld us)",
                             (long long)timeout_us);
        for (int i = 0; i < n; i++) {
            if (!signals[i])
                return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_set_gather: NULL signal array %d", i);
            g.sig[i] = signals[i];
        }
        g.rank = rank;
        g.state = signals[rank] + kMaxGather;  // {CTA counter, epoch} beside this rank's signals
        g.status = k->dev_status;
        g.timeout_ns = (uint64_t)timeout_us * 1000u;
    }
    g.n = n;
    g.col0 = q_head_offset;
    g.cols = q_heads_total;
    k->gather = g;
    return SA_OK;
}

int sa_kv_cache_get_config(const sa_kv_cache *cache, sa_kv_cache_config *config) {
    if (!cache || !config) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_get_config: NULL argument");
    *config = reinterpret_cast<const kv_cache_impl *>(cache)->cfg;
    return SA_OK;
}

// CompressedKVCache::memory_bytes (kv_compression.rs:928-957) of the `position` rows written so
// far, per sequence of the batch and summed over it: per (layer, head, row) a K and a V
// QuantizedBlock (code bytes + 4*4 + 8 + 1, :166-168), with QJL two QJLResidual (8*ceil(D/64)
// + 4 + 8, :352-354); with low-rank K one LowRankK per (layer, head) once a row exists
// ((rows*rank + rank*D)*4 + 8*4, :442-444, rank 1).  `device_bytes` is the allocation.
int sa_kv_cache_memory_bytes(const sa_kv_cache *cache, uint64_t *reference_bytes, uint64_t *device_bytes) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_memory_bytes: NULL cache");
    const kv_cache_impl *k = reinterpret_cast<const kv_cache_impl *>(cache);
    const uint64_t rows = (uint64_t)k->position, D = (uint64_t)k->cfg.head_dim;
    uint64_t per_row = 2 * ((uint64_t)k->code_bytes + 4 * 4 + 8 + 1);
    if (k->cfg.qjl_residual) per_row += 2 * (8 * ((D + 63) / 64) + 4 + 8);
    uint64_t per_head = rows * per_row;
    if (k->cfg.lowrank_k > 0 && rows > 0) per_head += (rows * 1 + 1 * D) * 4 + 8 * 4;
    const uint64_t heads = (uint64_t)k->cfg.num_layers * (uint64_t)k->cfg.kv_head_count * (uint64_t)k->cfg.batch;
    if (reference_bytes) *reference_bytes = heads * per_head;
    if (device_bytes) *device_bytes = (uint64_t)k->base_bytes;
    return SA_OK;
}

// The layer's power-iteration scratch of the low-rank K state (nullptr when off).
static float *lr_scratch_of(const kv_cache_impl *k, int32_t layer) {
    return k->lr_scratch ? k->lr_scratch + (size_t)layer * k->layer_lr_us_floats : nullptr;
}

int sa_kv_cache_layer_view(const sa_kv_cache *cache, int32_t layer, sa_kv_layer_view *v) {
    if (!cache || !v) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_layer_view: NULL argument");
    const kv_cache_impl *k = reinterpret_cast<const kv_cache_impl *>(cache);
    if (layer < 0 || layer >= k->cfg.num_layers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_view:layer_idx %d", layer);
    v->k_codes = k->k_codes + (size_t)layer * k->layer_codes_bytes;
    v->v_codes = k->v_codes + (size_t)layer * k->layer_codes_bytes;
    v->k_meta = k->k_meta + (size_t)layer * k->layer_meta_floats;
    v->v_meta = k->v_meta + (size_t)layer * k->layer_meta_floats;
    v->signs = k->signs + (size_t)layer * k->cfg.kv_head_count * k->cfg.head_dim;
    v->batch = k->cfg.batch;
    v->kv_heads = k->cfg.kv_head_count;
    v->head_dim = k->cfg.head_dim;
    v->bits = k->cfg.bits;
    v->code_bytes = k->code_bytes;
    v->capacity = k->capacity;
    v->wht_scale = k->wht_scale;
    const bool lr = k->lr_vt != nullptr;
    v->lr_vt = lr ? k->lr_vt + (size_t)layer * k->layer_lr_vt_floats : nullptr;
    v->lr_us = lr ? k->lr_us + (size_t)layer * k->layer_lr_us_floats : nullptr;
    v->lr_kmeta = lr ? k->lr_kmeta + (size_t)layer * 2 * k->layer_lr_us_floats : nullptr;
    v->lr_vtr = lr ? k->lr_vtr + (size_t)layer * k->layer_lr_vt_floats : nullptr;
    const bool qjl = k->k_qjl_bits != nullptr;
    v->k_qjl_bits = qjl ? k->k_qjl_bits + (size_t)layer * k->layer_qjl_bytes : nullptr;
    v->v_qjl_bits = qjl ? k->v_qjl_bits + (size_t)layer * k->layer_qjl_bytes : nullptr;
    v->k_qjl_mag = qjl ? k->k_qjl_mag + (size_t)layer * k->layer_qjl_floats : nullptr;
    v->v_qjl_mag = qjl ? k->v_qjl_mag + (size_t)layer * k->layer_qjl_floats : nullptr;
    return SA_OK;
}

static bool dtype_ok(int32_t dt) {
    return dt == SA_DTYPE_FLOAT || dt == SA_DTYPE_FLOAT16 || dt == SA_DTYPE_BFLOAT16;
}

// Shared validation of the RoPE inputs (validate_rope_caches and
// check_rope_position, ops/microsoft.rs:71-131): rows must cover every
// position touched.
static int check_rope(const char *op, int do_rotary, const float *cos_cache, const float *sin_cache,
                      int32_t cache_rows, int64_t last_pos) {
    if (!do_rotary) return SA_OK;
    if (!cos_cache) return set_error(SA_ERR_SHAPE_MISMATCH, "%s: do_rotary=1 but cos_cache is missing", op);
    if (!sin_cache) return set_error(SA_ERR_SHAPE_MISMATCH, "%s: do_rotary=1 but sin_cache is missing", op);
    if (last_pos >= cache_rows)
        return set_error(SA_ERR_SHAPE_MISMATCH, "%s: position %lld out of cache range %d", op,
                         (long long)last_pos, cache_rows);
    return SA_OK;
}

int sa_kv_append(sa_kv_cache *cache, int32_t layer, const void *key, const void *value, int32_t dtype,
                 int32_t batch, int32_t seq_len, const float *cos_cache, const float *sin_cache,
                 int32_t cache_rows, int32_t do_rotary, int32_t rotary_interleaved, sa_stream_t stream) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_append: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    if (layer < 0 || layer >= k->cfg.num_layers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "kv_cache_append:layer_idx %d", layer);
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "kv_append: dtype %d not supported", dtype);
    if (batch != k->cfg.batch)
        return set_error(SA_ERR_SHAPE_MISMATCH, "kv_append: batch %d != cache batch %d", batch, k->cfg.batch);
    if (seq_len < 0) return set_error(SA_ERR_SHAPE_MISMATCH, "kv_append: negative seq_len");
    if (seq_len == 0) return SA_OK;
    if (!key || !value) return set_error(SA_ERR_INVALID_ARGUMENT, "kv_append: NULL key/value");
    if (k->position + seq_len > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "kv_cache_append:position_overflow (%lld + %d > %d)",
                         (long long)k->position, seq_len, k->cfg.max_seq_len);
    int rc = check_rope("kv_append", do_rotary, cos_cache, sin_cache, cache_rows, k->position + seq_len - 1);
    if (rc != SA_OK) return rc;
    sa_kv_layer_view v;
    sa_kv_cache_layer_view(cache, layer, &v);
    AppendArgs a;
    a.key = key;
    a.value = value;
    a.dtype = dtype;
    a.batch = batch;
    a.seq_len = seq_len;
    a.heads = v.kv_heads;
    a.head_dim = v.head_dim;
    a.bits = v.bits;
    a.code_bytes = v.code_bytes;
    a.capacity = v.capacity;
    a.pos0 = k->position;
    a.k_codes = v.k_codes;
    a.v_codes = v.v_codes;
    a.k_meta = v.k_meta;
    a.v_meta = v.v_meta;
    a.k_qjl_bits = v.k_qjl_bits;
    a.v_qjl_bits = v.v_qjl_bits;
    a.k_qjl_mag = v.k_qjl_mag;
    a.v_qjl_mag = v.v_qjl_mag;
    a.lr_vt = v.lr_vt;
    a.lr_us = v.lr_us;
    a.lr_scratch = lr_scratch_of(k, layer);
    a.lr_kmeta = v.lr_kmeta;
    a.lr_vtr = v.lr_vtr;
    a.signs = v.signs;
    a.wht_scale = v.wht_scale;
    a.cos_cache = cos_cache;
    a.sin_cache = sin_cache;
    a.cache_rows = cache_rows;
    a.do_rotary = do_rotary ? 1 : 0;
    a.interleaved = rotary_interleaved ? 1 : 0;
    int rc2 = launch_kv_append(a, static_cast<cudaStream_t>(stream));
    if (rc2 != SA_OK || !a.lr_us) return rc2;
    return launch_lowrank_append(a, static_cast<cudaStream_t>(stream));
}

// Attention of `seq_len` query tokens over the cache.  When `key`/`value`
// are given, the tokens are appended first (the operator); the tensor-core
// decode path fuses that append into its prep kernel.
static int attend_impl(kv_cache_impl *k, int32_t layer, const void *query, void *attn_out, int32_t dtype,
                       int32_t batch, int32_t seq_len, int64_t num_heads, int32_t has_scale, float scale,
                       const float *cos_cache, const float *sin_cache, int32_t cache_rows, int32_t do_rotary,
                       int32_t rotary_interleaved, cudaStream_t stream, const void *key = nullptr,
                       const void *value = nullptr) {
    if (layer < 0 || layer >= k->cfg.num_layers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend: layer_idx %d", layer);
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "gqa_attend: dtype %d not supported", dtype);
    if (batch != k->cfg.batch)
        return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend: batch %d != cache batch %d", batch, k->cfg.batch);
    if (num_heads != k->cfg.num_heads)
        return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend: num_heads %lld != cache num_heads %d",
                         (long long)num_heads, k->cfg.num_heads);
    if (seq_len < 0) return set_error(SA_ERR_SHAPE_MISMATCH, "gqa_attend: negative seq_len");
    if (seq_len == 0) return SA_OK;
    if (!query || !attn_out) return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend: NULL query/attn_out");
    if (k->position + seq_len > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "gqa_attend: queries past max_seq_len");
    int rc = check_rope("gqa_attend", do_rotary, cos_cache, sin_cache, cache_rows, k->position + seq_len - 1);
    if (rc != SA_OK) return rc;
    sa_kv_layer_view v;
    sa_kv_cache_layer_view(reinterpret_cast<sa_kv_cache *>(k), layer, &v);
    AttendArgs a{};
    a.query = query;
    a.out = attn_out;
    a.dtype = dtype;
    a.batch = batch;
    a.seq_len = seq_len;
    a.heads = v.kv_heads;
    a.group = k->group;
    a.head_dim = v.head_dim;
    a.bits = v.bits;
    a.code_bytes = v.code_bytes;
    a.capacity = v.capacity;
    a.pos0 = k->position;
    a.k_codes = v.k_codes;
    a.v_codes = v.v_codes;
    a.k_meta = v.k_meta;
    a.v_meta = v.v_meta;
    a.signs = v.signs;
    a.wht_scale = v.wht_scale;
    // GroupQueryAttention scale (ops/microsoft.rs:1160): attribute, else 1/sqrt_f32(D).
    a.scale = has_scale ? scale : 1.0f / host_sqrt_f32((float)v.head_dim);
    a.cos_cache = cos_cache;
    a.sin_cache = sin_cache;
    a.cache_rows = cache_rows;
    a.do_rotary = do_rotary ? 1 : 0;
    a.interleaved = rotary_interleaved ? 1 : 0;
    a.workspace = k->workspace;
    a.workspace_floats = k->workspace_floats;
    a.sm_count = k->sm_count;
    a.qprep = k->qprep;
    a.dev_status = k->dev_status;
    a.gather = k->gather;
    AppendArgs ap;
    if (key) {
        ap.key = key;
        ap.value = value;
        ap.dtype = dtype;
        ap.batch = batch;
        ap.seq_len = seq_len;
        ap.heads = v.kv_heads;
        ap.head_dim = v.head_dim;
        ap.bits = v.bits;
        ap.code_bytes = v.code_bytes;
        ap.capacity = v.capacity;
        ap.pos0 = k->position;
        ap.k_codes = v.k_codes;
        ap.v_codes = v.v_codes;
        ap.k_meta = v.k_meta;
        ap.v_meta = v.v_meta;
        ap.k_qjl_bits = v.k_qjl_bits;
        ap.v_qjl_bits = v.v_qjl_bits;
        ap.k_qjl_mag = v.k_qjl_mag;
        ap.v_qjl_mag = v.v_qjl_mag;
        ap.lr_vt = v.lr_vt;
        ap.lr_us = v.lr_us;
        ap.lr_scratch = lr_scratch_of(k, layer);
        ap.lr_kmeta = v.lr_kmeta;
        ap.lr_vtr = v.lr_vtr;
        ap.signs = v.signs;
        ap.wht_scale = v.wht_scale;
        ap.cos_cache = cos_cache;
        ap.sin_cache = sin_cache;
        ap.cache_rows = cache_rows;
        ap.do_rotary = a.do_rotary;
        ap.interleaved = a.interleaved;
    }
    if (v.lr_vtr) {
        // low-rank K: keys are lr_us[t] * lr_vt (read_k, kv_compression.rs:870-882); the state of
        // the new tokens first, then the usual kernels on {0, U*S[t]} metadata
        if (key) {
            rc = launch_lowrank_append(ap, stream);
            if (rc != SA_OK) return rc;
        }
        a.k_meta = v.lr_kmeta;
        a.lr_vtr = v.lr_vtr;
    }
    if (decode_fast_eligible(a)) return launch_gqa_decode_fast(a, key ? &ap : nullptr, stream);
    if (key) {
        rc = launch_kv_append(ap, stream);
        if (rc != SA_OK) return rc;
    }
    if (prefill_eligible(a)) return launch_gqa_prefill_umma(a, stream);  // tcgen05 prefill chunk
    // the generic kernels write attn_out; a head-sharded output is copied out after
    AttendArgs ga = a;
    ga.gather.n = 0;
    rc = launch_gqa_attend_generic(ga, stream);
    if (rc != SA_OK || a.gather.n == 0) return rc;
    return launch_gather_scatter(a, stream);
}

int sa_gqa_attend(sa_kv_cache *cache, int32_t layer, const void *query, void *attn_out, int32_t dtype,
                  int32_t batch, int32_t seq_len, int64_t num_heads, int32_t has_scale, float scale,
                  const float *cos_cache, const float *sin_cache, int32_t cache_rows, int32_t do_rotary,
                  int32_t rotary_interleaved, sa_stream_t stream) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "gqa_attend: NULL cache");
    return attend_impl(reinterpret_cast<kv_cache_impl *>(cache), layer, query, attn_out, dtype, batch, seq_len,
                       num_heads, has_scale, scale, cos_cache, sin_cache, cache_rows, do_rotary,
                       rotary_interleaved, static_cast<cudaStream_t>(stream));
}

int sa_group_query_attention(sa_kv_cache *cache, int32_t layer, const void *query, const void *key,
                             const void *value, void *attn_out, int32_t dtype, int32_t batch, int32_t seq_len,
                             int64_t num_heads, int64_t kv_num_heads, int32_t has_scale, float scale,
                             int64_t local_window_size, int32_t do_rotary, int32_t rotary_interleaved,
                             const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                             sa_stream_t stream) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "GroupQueryAttention: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    // op_group_query_attention / gqa_validate order (ops/microsoft.rs:1089-1094, 941-952).
    if (local_window_size != -1)
        return set_error(SA_ERR_INVALID_ATTRIBUTE,
                         "GroupQueryAttention: local_window_size != -1 not supported in this tier");
    if (!query) return set_error(SA_ERR_SHAPE_MISMATCH, "GroupQueryAttention: missing query");
    if (!key) return set_error(SA_ERR_SHAPE_MISMATCH, "GroupQueryAttention: missing key");
    if (!value) return set_error(SA_ERR_SHAPE_MISMATCH, "GroupQueryAttention: missing value");
    if (num_heads <= 0 || kv_num_heads <= 0)
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "GroupQueryAttention: num_heads and kv_num_heads must be > 0");
    if (num_heads % kv_num_heads != 0)
        return set_error(SA_ERR_INVALID_ATTRIBUTE,
                         "GroupQueryAttention: num_heads must be a multiple of kv_num_heads");
    if (kv_num_heads != k->cfg.num_kv_heads || num_heads != k->cfg.num_heads)
        return set_error(SA_ERR_SHAPE_MISMATCH,
                         "GroupQueryAttention: heads (%lld, %lld) do not match the cache (%d, %d)",
                         (long long)num_heads, (long long)kv_num_heads, k->cfg.num_heads, k->cfg.num_kv_heads);
    if (do_rotary && (!cos_cache || !sin_cache))
        return set_error(SA_ERR_SHAPE_MISMATCH, "GroupQueryAttention: do_rotary=1 but %s is missing",
                         !cos_cache ? "cos_cache" : "sin_cache");
    if (batch != k->cfg.batch || seq_len < 0)
        return set_error(SA_ERR_SHAPE_MISMATCH, "GroupQueryAttention: batch/seq_len mismatch");
    if (k->position + seq_len > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "kv_cache_append:position_overflow");
    int rc = check_rope("GroupQueryAttention", do_rotary, cos_cache, sin_cache, cache_rows,
                        k->position + seq_len - 1);
    if (rc != SA_OK) return rc;
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "GroupQueryAttention: dtype %d not supported", dtype);
    if (layer < 0 || layer >= k->cfg.num_layers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "GroupQueryAttention: layer_idx %d", layer);
    if (seq_len == 0) return SA_OK;
    return attend_impl(k, layer, query, attn_out, dtype, batch, seq_len, num_heads, has_scale, scale, cos_cache,
                       sin_cache, cache_rows, do_rotary, rotary_interleaved, static_cast<cudaStream_t>(stream), key,
                       value);
}

int64_t sa_matmul_nbits_packed_bytes(int64_t n, int64_t k, int32_t bits, int32_t block_size, int32_t dtype) {
    if (bits != 4 || !matmul_nbits_packable(dtype, n, k, block_size)) return 0;
    return (int64_t)matmul_nbits_packed_bytes(n, k);
}

int sa_matmul_nbits_prepack(const uint8_t *b, const void *scales, void *packed, int32_t dtype, int64_t n, int64_t k,
                            int32_t bits, int32_t block_size, sa_stream_t stream) {
    if (bits != 4) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits prepack: bits=%d not supported (4 only)", bits);
    if (!matmul_nbits_packable(dtype, n, k, block_size))
        return set_error(SA_ERR_UNSUPPORTED,
                         "MatMulNBits prepack: needs fp16/bf16, block 32, N %% 32 == 0, K %% 1024 == 0 "
                         "(got dtype %d, block %d, N %lld, K %lld)",
                         dtype, block_size, (long long)n, (long long)k);
    if (!b || !scales || !packed) return set_error(SA_ERR_INVALID_ARGUMENT, "MatMulNBits prepack: NULL pointer");
    if ((reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(packed)) & 15)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits prepack: B and packed must be 16-byte aligned");
    return launch_matmul_nbits_prepack(b, scales, packed, dtype, n, k, static_cast<cudaStream_t>(stream));
}

int sa_matmul_nbits_packed(const void *a, const void *packed, const void *bias, void *y, int32_t dtype, int64_t m,
                           int64_t n, int64_t k, int32_t bits, int32_t block_size, sa_stream_t stream) {
    if (bits != 4) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits packed: bits=%d not supported (4 only)", bits);
    if (!matmul_nbits_packable(dtype, n, k, block_size))
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits packed: no packed path for this dtype/shape/block");
    if (m < 0 || m > 8)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits packed: m=%lld rows (1..8 supported)", (long long)m);
    if (m == 0) return SA_OK;
    if (!a || !packed || !y) return set_error(SA_ERR_INVALID_ARGUMENT, "MatMulNBits packed: NULL input/output");
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(packed)) & 15)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits packed: A and packed must be 16-byte aligned");
    return launch_matmul_nbits_packed(a, packed, bias, y, dtype, m, n, k, static_cast<cudaStream_t>(stream));
}

int sa_matmul_nbits(const void *a, const uint8_t *b, const void *scales, const uint8_t *zero_points,
                    const void *bias, void *y, int32_t dtype, int64_t m, int64_t n, int64_t k, int32_t bits,
                    int32_t block_size, sa_stream_t stream) {
    if (bits != 4) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: bits=%d not supported (4 only)", bits);
    if (block_size < 16 || !is_pow2(block_size))
        return set_error(SA_ERR_INVALID_ATTRIBUTE, "MatMulNBits: block_size must be a power of two >= 16");
    if (m < 0 || n <= 0 || k <= 0) return set_error(SA_ERR_SHAPE_MISMATCH, "MatMulNBits: bad shape");
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: dtype %d not supported", dtype);
    if (m == 0) return SA_OK;
    if (!a || !b || !scales || !y) return set_error(SA_ERR_INVALID_ARGUMENT, "MatMulNBits: NULL input/output");
    if (k % block_size != 0)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: K=%lld not a multiple of block_size", (long long)k);
    return launch_matmul_nbits(a, b, scales, zero_points, bias, y, dtype, m, n, k, block_size,
                               static_cast<cudaStream_t>(stream));
}

int sa_qkv_project_append(sa_kv_cache *cache, int32_t layer, const void *x, const uint8_t *w_codes,
                          const void *w_scales, int32_t dtype, int32_t batch, int64_t hidden,
                          const float *cos_cache, const float *sin_cache, int32_t cache_rows,
                          int32_t do_rotary, int32_t rotary_interleaved, void *q_out, void *k_out,
                          void *v_out, sa_stream_t stream) {
    if (!cache) return set_error(SA_ERR_INVALID_ARGUMENT, "qkv_project_append: NULL cache");
    kv_cache_impl *k = reinterpret_cast<kv_cache_impl *>(cache);
    if (layer < 0 || layer >= k->cfg.num_layers)
        return set_error(SA_ERR_INVALID_ARGUMENT, "qkv_project_append: layer_idx %d", layer);
    if (dtype != SA_DTYPE_FLOAT16 && dtype != SA_DTYPE_BFLOAT16)
        return set_error(SA_ERR_UNSUPPORTED, "qkv_project_append: dtype %d (fp16/bf16 only)", dtype);
    if (batch != k->cfg.batch)
        return set_error(SA_ERR_SHAPE_MISMATCH, "qkv_project_append: batch %d != cache batch %d", batch,
                         k->cfg.batch);
    if (hidden <= 0 || hidden % 32 != 0)
        return set_error(SA_ERR_SHAPE_MISMATCH, "qkv_project_append: hidden %lld not a multiple of 32",
                         (long long)hidden);
    if (!x || !w_codes || !w_scales || !q_out || !k_out || !v_out)
        return set_error(SA_ERR_INVALID_ARGUMENT, "qkv_project_append: NULL input/output");
    if (k->position + 1 > k->cfg.max_seq_len)
        return set_error(SA_ERR_CAPACITY, "qkv_project_append: position_overflow (%lld + 1 > %d)",
                         (long long)k->position, k->cfg.max_seq_len);
    int rc = check_rope("qkv_project_append", do_rotary, cos_cache, sin_cache, cache_rows, k->position);
    if (rc != SA_OK) return rc;
    sa_kv_layer_view v;
    sa_kv_cache_layer_view(cache, layer, &v);
    QkvArgs a{};
    AppendArgs &ap = a.ap;
    ap.key = k_out;
    ap.value = v_out;
    ap.dtype = dtype;
    ap.batch = batch;
    ap.seq_len = 1;
    ap.heads = v.kv_heads;
    ap.head_dim = v.head_dim;
    ap.bits = v.bits;
    ap.code_bytes = v.code_bytes;
    ap.capacity = v.capacity;
    ap.pos0 = k->position;
    ap.k_codes = v.k_codes;
    ap.v_codes = v.v_codes;
    ap.k_meta = v.k_meta;
    ap.v_meta = v.v_meta;
    ap.k_qjl_bits = v.k_qjl_bits;
    ap.v_qjl_bits = v.v_qjl_bits;
    ap.k_qjl_mag = v.k_qjl_mag;
    ap.v_qjl_mag = v.v_qjl_mag;
    ap.lr_vt = v.lr_vt;
    ap.lr_us = v.lr_us;
    ap.lr_scratch = lr_scratch_of(k, layer);
    ap.lr_kmeta = v.lr_kmeta;
    ap.lr_vtr = v.lr_vtr;
    ap.signs = v.signs;
    ap.wht_scale = v.wht_scale;
    ap.cos_cache = cos_cache;
    ap.sin_cache = sin_cache;
    ap.cache_rows = cache_rows;
    ap.do_rotary = do_rotary ? 1 : 0;
    ap.interleaved = rotary_interleaved ? 1 : 0;
    a.q_out = q_out;
    a.q_heads = v.kv_heads * k->group;
    const int64_t D = v.head_dim, qc = (int64_t)a.q_heads * D, kc = (int64_t)v.kv_heads * D;
    const int64_t n = qc + 2 * kc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((D == 64 || D == 128) && qc % 128 == 0 && kc % 128 == 0 &&
        matmul_nbits_umma_eligible(x, w_codes, w_scales, nullptr, dtype, batch, n, hidden, 32)) {
        rc = launch_qkv_umma_fused(x, w_codes, w_scales, a, n, hidden, st);
        if (rc != SA_OK || !ap.lr_us) return rc;
        return launch_lowrank_append(ap, st);  // k_out holds the projection before RoPE
    }
    // the three projections (row ranges of the packed weights), then the epilogue launch
    const int64_t row_codes = hidden / 2, row_scales = (hidden / 32) * 2;
    const uint8_t *sc = static_cast<const uint8_t *>(w_scales);
    rc = launch_matmul_nbits(x, w_codes, sc, nullptr, nullptr, q_out, dtype, batch, qc, hidden, 32, st);
    if (rc == SA_OK)
        rc = launch_matmul_nbits(x, w_codes + qc * row_codes, sc + qc * row_scales, nullptr, nullptr, k_out, dtype,
                                 batch, kc, hidden, 32, st);
    if (rc == SA_OK)
        rc = launch_matmul_nbits(x, w_codes + (qc + kc) * row_codes, sc + (qc + kc) * row_scales, nullptr, nullptr,
                                 v_out, dtype, batch, kc, hidden, 32, st);
    if (rc != SA_OK) return rc;
    rc = launch_qkv_finish(a, st);
    if (rc != SA_OK || !ap.lr_us) return rc;
    return launch_lowrank_append(ap, st);
}

int sa_rms_norm(const void *x, const void *skip, const void *bias, const void *weight, void *y, void *pre,
                int32_t dtype, int64_t rows, int64_t cols, float epsilon, sa_stream_t stream) {
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "rms_norm: dtype %d not supported", dtype);
    if (rows < 0 || cols <= 0 || cols > (1 << 30) || rows > 0x7fffffff)
        return set_error(SA_ERR_SHAPE_MISMATCH, "RMSNormalization: normalized region is empty or too large");
    if (rows == 0) return SA_OK;
    if (!x || !weight || !y) return set_error(SA_ERR_INVALID_ARGUMENT, "rms_norm: NULL input/output");
    if (!(epsilon >= 0.0f)) return set_error(SA_ERR_INVALID_ATTRIBUTE, "rms_norm: epsilon must be >= 0");
    return launch_rms_norm(x, skip, bias, weight, y, pre, dtype, rows, cols, epsilon,
                           static_cast<cudaStream_t>(stream));
}

int sa_silu_mul(const void *gate, const void *up, int64_t ld_in, void *y, int32_t dtype, int64_t rows,
                int64_t cols, sa_stream_t stream) {
    if (!dtype_ok(dtype)) return set_error(SA_ERR_UNSUPPORTED, "silu_mul: dtype %d not supported", dtype);
    if (rows < 0 || cols <= 0 || ld_in < cols || cols > (1 << 30))
        return set_error(SA_ERR_SHAPE_MISMATCH, "silu_mul: bad shape (rows %lld, cols %lld, ld_in %lld)",
                         (long long)rows, (long long)cols, (long long)ld_in);
    if (rows == 0) return SA_OK;
    if (!gate || !up || !y) return set_error(SA_ERR_INVALID_ARGUMENT, "silu_mul: NULL input/output");
    return launch_silu_mul(gate, up, ld_in, y, dtype, rows, cols, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

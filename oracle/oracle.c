/*
 * CPU oracle for the smallaios_b200 decode hot path (TEST INFRASTRUCTURE
 * ONLY -- see oracle.h).  Plain-C restatement of SmallAIOS onnx-rt:
 *   onnx-rt/src/kv_compression.rs   PolarQuant / QJL primitives
 *   onnx-rt/src/ops/microsoft.rs    RoPE, SDPA, GroupQueryAttention
 *   onnx-rt/src/operators.rs        expf_approx, sqrt_approx
 *   onnx-rt/src/gemm.rs             gemm_f32 tile order
 * Compiled with -O2 -ffp-contract=off: every a*b+c below is a separately
 * rounded multiply and add, exactly like the Rust source.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Rust `f as i32`: truncate toward zero, saturate, NaN -> 0. */
static int32_t sat_f32_to_i32(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

/* Rust `f as u32`: truncate toward zero, saturate to [0, u32::MAX], NaN -> 0. */
static uint32_t sat_f32_to_u32(float x) {
    if (x != x) return 0;
    if (x <= 0.0f) return 0;
    if (x >= 4294967296.0f) return UINT32_MAX;
    return (uint32_t)x;
}

static float f32_from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* operators.rs:3311-3320 */
float orc_sqrt_approx(float x) {
    if (x <= 0.0f) return 0.0f;
    float s = x;
    for (int i = 0; i < 10; i++) s = 0.5f * (s + x / s);
    return s;
}

/* ops/microsoft.rs:54-62 */
float orc_sqrt_f32(float x) {
    if (x <= 0.0f) return 0.0f;
    float g = x;
    for (int i = 0; i < 16; i++) g = 0.5f * (g + x / g);
    return g;
}

/* operators.rs:1311-1357 (constants 1311-1323). */
float orc_expf_approx(float x) {
    const float clamp_max = 88.7f, clamp_min = -88.7f;
    const float c2 = 0.5f;
    const float c3 = 1.0f / 6.0f;
    const float c4 = 1.0f / 24.0f;
    const float log2_e = 1.44269504088896340735992468100189214f;
    const float ln_2 = 0.693147180559945309417232121458176568f;
    /* f32::clamp keeps NaN. */
    if (x < clamp_min) x = clamp_min;
    if (x > clamp_max) x = clamp_max;
    float t = x * log2_e;
    int32_t k = (t >= 0.0f) ? sat_f32_to_i32(t + 0.5f) : sat_f32_to_i32(t - 0.5f);
    if ((int64_t)k + 127 < 0) return 0.0f;
    float f = x - (float)k * ln_2;
    float f2 = f * f;
    float p = 1.0f + f + f2 * c2 + f2 * f * c3 + f2 * f2 * c4;
    uint32_t bits = ((uint32_t)(k + 127)) << 23;
    return p * f32_from_bits(bits);
}

/* kv_compression.rs:27-37 */
float orc_round_f32(float x) {
    float tr = (float)sat_f32_to_i32(x);
    float frac = x - tr;
    if (frac >= 0.5f) return tr + 1.0f;
    if (frac <= -0.5f) return tr - 1.0f;
    return tr;
}

/* kv_compression.rs:58-67 */
uint64_t orc_xorshift64_next(uint64_t *state) {
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

/* kv_compression.rs:776-779: seed.wrapping_mul(0x9E37..).wrapping_add(layer*nh+head) */
uint64_t orc_head_seed(uint64_t seed, int layer, int num_kv_heads, int head) {
    return seed * 0x9E3779B97F4A7C15ULL + (uint64_t)((uint64_t)layer * (uint64_t)num_kv_heads + (uint64_t)head);
}

static int is_pow2(int n) { return n > 0 && (n & (n - 1)) == 0; }

/* PolarQuantizer::new (kv_compression.rs:197-213) + Xorshift64::new (:48-56). */
int orc_polar_signs(uint64_t seed, int dim, int8_t *signs) {
    if (!is_pow2(dim)) return ORC_INVALID_ATTRIBUTE;
    uint64_t st = seed == 0 ? 0x5EEDDEADBEEFCAFEULL : seed;
    for (int i = 0; i < dim; i++) signs[i] = (orc_xorshift64_next(&st) & 1) == 0 ? 1 : -1;
    return ORC_OK;
}

/* wht_butterfly_normalize (kv_compression.rs:81-107) */
static void wht_butterfly_normalize(float *x, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int i = 0; i < n; i += 2 * h) {
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
        }
    }
    float scale = 1.0f / orc_sqrt_approx((float)n);
    for (int i = 0; i < n; i++) x[i] *= scale;
}

/* apply_signs (kv_compression.rs:113-118) */
static void apply_signs(float *x, int n, const int8_t *signs) {
    for (int i = 0; i < n; i++) x[i] *= (float)signs[i];
}

void orc_wht_with_signs(float *x, int n, const int8_t *signs) {
    apply_signs(x, n, signs);
    wht_butterfly_normalize(x, n);
}

void orc_inverse_wht_with_signs(float *x, int n, const int8_t *signs) {
    wht_butterfly_normalize(x, n);
    apply_signs(x, n, signs);
}

/* pack_bits (kv_compression.rs:294-312): LSB-first contiguous bit stream. */
void orc_pack_bits(const uint32_t *values, int count, int bits, uint8_t *out) {
    int nbytes = (count * bits + 7) / 8;
    memset(out, 0, (size_t)nbytes);
    size_t bit_pos = 0;
    for (int i = 0; i < count; i++) {
        for (int b = 0; b < bits; b++) {
            if ((values[i] >> b) & 1u) out[bit_pos / 8] |= (uint8_t)(1u << (bit_pos % 8));
            bit_pos++;
        }
    }
}

/* unpack_bits (kv_compression.rs:315-333) */
void orc_unpack_bits(const uint8_t *data, int nbytes, int count, int bits, uint32_t *out) {
    size_t bit_pos = 0;
    for (int i = 0; i < count; i++) {
        uint32_t v = 0;
        for (int b = 0; b < bits; b++) {
            size_t byte_idx = bit_pos / 8, bit_idx = bit_pos % 8;
            if ((int)byte_idx < nbytes && ((data[byte_idx] >> bit_idx) & 1u)) v |= 1u << b;
            bit_pos++;
        }
        out[i] = v;
    }
}

static int valid_bits(int bits) { return bits == 3 || bits == 4 || bits == 8; }

/* PolarQuantizer::encode (kv_compression.rs:216-267) */
int orc_polar_encode(const float *in, int dim, int bits, const int8_t *signs,
                     uint8_t *codes, float *scale_out, float *zp_out,
                     float *min_out, float *max_out) {
    if (!is_pow2(dim)) return ORC_INVALID_ATTRIBUTE;
    if (!valid_bits(bits)) return ORC_INVALID_ATTRIBUTE;
    float rot_buf[1024];
    uint32_t q_buf[1024];
    float *rot = dim <= 1024 ? rot_buf : (float *)malloc(sizeof(float) * (size_t)dim);
    uint32_t *q = dim <= 1024 ? q_buf : (uint32_t *)malloc(sizeof(uint32_t) * (size_t)dim);
    memcpy(rot, in, sizeof(float) * (size_t)dim);
    orc_wht_with_signs(rot, dim, signs);
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < dim; i++) {
        float v = rot[i];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    uint32_t levels = (1u << bits) - 1u;
    float range = mx - mn;
    float scale = range > 0.0f ? range / (float)levels : 1.0f;
    float zp = mn;
    for (int i = 0; i < dim; i++) {
        uint32_t qi = scale > 0.0f ? sat_f32_to_u32(orc_round_f32((rot[i] - zp) / scale)) : 0u;
        q[i] = qi < levels ? qi : levels;
    }
    orc_pack_bits(q, dim, bits, codes);
    if (scale_out) *scale_out = scale;
    if (zp_out) *zp_out = zp;
    if (min_out) *min_out = mn;
    if (max_out) *max_out = mx;
    if (rot != rot_buf) free(rot);
    if (q != q_buf) free(q);
    return ORC_OK;
}

/* PolarQuantizer::decode (kv_compression.rs:270-286) */
int orc_polar_decode(const uint8_t *codes, float scale, float zp, int dim, int bits,
                     const int8_t *signs, float *out) {
    if (!is_pow2(dim)) return ORC_INVALID_ATTRIBUTE;
    if (!valid_bits(bits)) return ORC_INVALID_ATTRIBUTE;
    uint32_t q_buf[1024];
    uint32_t *q = dim <= 1024 ? q_buf : (uint32_t *)malloc(sizeof(uint32_t) * (size_t)dim);
    orc_unpack_bits(codes, (dim * bits + 7) / 8, dim, bits, q);
    for (int i = 0; i < dim; i++) out[i] = (float)q[i] * scale + zp;
    orc_inverse_wht_with_signs(out, dim, signs);
    if (q != q_buf) free(q);
    return ORC_OK;
}

/* PolarQuantizer::encode of n independent vectors sharing one sign vector,
 * split over nthreads threads (each vector is encoded exactly as
 * orc_polar_encode does; the threads only change which core runs it). */
typedef struct {
    const float *x;
    const int8_t *signs;
    uint8_t *codes;
    float *meta;
    size_t begin, end;
    int dim, bits, rc;
} encode_job;

static void *encode_worker(void *arg) {
    encode_job *j = (encode_job *)arg;
    size_t cb = ((size_t)j->dim * j->bits + 7) / 8;
    for (size_t i = j->begin; i < j->end && j->rc == ORC_OK; i++)
        j->rc = orc_polar_encode(j->x + i * j->dim, j->dim, j->bits, j->signs, j->codes + i * cb,
                                 j->meta + 2 * i, j->meta + 2 * i + 1, NULL, NULL);
    return NULL;
}

int orc_polar_encode_batch(const float *x, size_t n, int dim, int bits, const int8_t *signs,
                           uint8_t *codes, float *meta, int nthreads) {
    if (!is_pow2(dim) || !valid_bits(bits)) return ORC_INVALID_ATTRIBUTE;
    if (nthreads < 1) nthreads = 1;
    if ((size_t)nthreads > n) nthreads = n > 0 ? (int)n : 1;
    encode_job *jobs = (encode_job *)calloc((size_t)nthreads, sizeof(encode_job));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    int rc = ORC_OK;
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = (encode_job){x, signs, codes, meta, n * i / nthreads, n * (i + 1) / nthreads, dim, bits, ORC_OK};
        if (nthreads > 1) pthread_create(&th[i], NULL, encode_worker, &jobs[i]);
        else encode_worker(&jobs[i]);
    }
    for (int i = 0; i < nthreads; i++) {
        if (nthreads > 1) pthread_join(th[i], NULL);
        if (jobs[i].rc != ORC_OK) rc = jobs[i].rc;
    }
    free(jobs);
    free(th);
    return rc;
}

/* QJLResidualEncoder::encode (kv_compression.rs:365-395) */
void orc_qjl_encode(const float *original, const float *approx, int dim,
                    uint64_t *sign_bits, float *c_magnitude) {
    int words = (dim + 63) / 64;
    for (int w = 0; w < words; w++) sign_bits[w] = 0;
    float msum = 0.0f;
    for (int i = 0; i < dim; i++) {
        float r = original[i] - approx[i];
        msum += fabsf(r);
        if (r >= 0.0f) sign_bits[i / 64] |= 1ULL << (i % 64);
    }
    *c_magnitude = dim > 0 ? msum / (float)dim : 0.0f;
}

/* QJLResidualEncoder::correction (kv_compression.rs:401-417) */
float orc_qjl_correction(const uint64_t *a_bits, float a_c, const uint64_t *b_bits, float b_c, int dim) {
    if (dim == 0) return 0.0f;
    uint32_t xor_popcount = 0;
    for (int w = 0; w < (dim + 63) / 64; w++) xor_popcount += (uint32_t)__builtin_popcountll(a_bits[w] ^ b_bits[w]);
    float sign_inner = (float)dim - 2.0f * (float)xor_popcount;
    return a_c * b_c * sign_inner / (float)dim;
}

/* ---- Low-rank K (LowRankKeyDecomposer, kv_compression.rs:451-690) ------ */

/* norm_vec (:674-681) */
static float lr_norm_vec(const float *v, size_t n) {
    float s = 0.0f;
    for (size_t i = 0; i < n; i++) s += v[i] * v[i];
    return orc_sqrt_approx(s);
}

/* normalize_vec (:683-690) */
static void lr_normalize_vec(float *v, size_t n) {
    float nn = lr_norm_vec(v, n);
    if (nn > 1e-30f)
        for (size_t i = 0; i < n; i++) v[i] /= nn;
}

/* power_iteration_svd (:583-671): u_s [m][rank], vt [rank][n], zero where the loop stops early */
static void lr_power_iteration_svd(const float *matrix, size_t m, size_t n, size_t rank, float *u_s, float *vt) {
    memset(u_s, 0, sizeof(float) * m * rank);
    memset(vt, 0, sizeof(float) * rank * n);
    float *deflated = (float *)malloc(sizeof(float) * (m * n > 0 ? m * n : 1));
    float *v = (float *)malloc(sizeof(float) * (n > 0 ? n : 1));
    float *u = (float *)malloc(sizeof(float) * (m > 0 ? m : 1));
    memcpy(deflated, matrix, sizeof(float) * m * n);
    for (size_t r = 0; r < rank; r++) {
        for (size_t j = 0; j < n; j++) v[j] = ((j + r) % 2 == 0) ? 1.0f : -1.0f;
        lr_normalize_vec(v, n);
        for (int it = 0; it < 10; it++) {
            for (size_t i = 0; i < m; i++) {
                float dot = 0.0f;
                for (size_t j = 0; j < n; j++) dot += deflated[i * n + j] * v[j];
                u[i] = dot;
            }
            for (size_t j = 0; j < n; j++) v[j] = 0.0f;
            for (size_t i = 0; i < m; i++)
                for (size_t j = 0; j < n; j++) v[j] += deflated[i * n + j] * u[i];
            lr_normalize_vec(v, n);
        }
        for (size_t i = 0; i < m; i++) {
            float dot = 0.0f;
            for (size_t j = 0; j < n; j++) dot += deflated[i * n + j] * v[j];
            u[i] = dot;
        }
        float sigma = lr_norm_vec(u, m);
        if (sigma < 1e-12f) break;
        for (size_t i = 0; i < m; i++) u[i] /= sigma;
        for (size_t i = 0; i < m; i++) u_s[i * rank + r] = u[i] * sigma;
        for (size_t j = 0; j < n; j++) vt[r * n + j] = v[j];
        for (size_t i = 0; i < m; i++)
            for (size_t j = 0; j < n; j++) deflated[i * n + j] -= sigma * u[i] * v[j];
    }
    free(deflated);
    free(v);
    free(u);
}

/* LowRankKeyDecomposer::new (:460-465) + decompose (:470-499).  u_s holds rows * min(rank, rows, cols),
 * vt min(rank, rows, cols) * cols; returns that actual rank. */
int orc_lowrank_decompose(const float *k, int rows, int cols, int rank, float *u_s, float *vt) {
    if (rank == 0) rank = 1;
    if (rows == 0 || cols == 0) return rank;
    int actual = rank < rows ? rank : rows;
    if (cols < actual) actual = cols;
    lr_power_iteration_svd(k, (size_t)rows, (size_t)cols, (size_t)actual, u_s, vt);
    return actual;
}

/* LowRankKeyDecomposer::reconstruct (:502-526) */
void orc_lowrank_reconstruct(const float *u_s, const float *vt, int rows, int cols, int rank, float *out) {
    for (size_t i = 0; i < (size_t)rows * (size_t)cols; i++) out[i] = 0.0f;
    if (rows == 0 || cols == 0 || rank == 0) return;
    for (int i = 0; i < rows; i++)
        for (int j = 0; j < cols; j++) {
            float sum = 0.0f;
            for (int r = 0; r < rank; r++) sum += u_s[(size_t)i * rank + r] * vt[(size_t)r * cols + j];
            out[(size_t)i * cols + j] = sum;
        }
}

/* LowRankKeyDecomposer::update (:529-562) + reorthogonalize (:564-579) on a state whose u_s has room
 * for rows + 1 rows.  *rows, *write_counter and *rank are updated in place. */
void orc_lowrank_update(float *u_s, float *vt, int *rows, int cols, int *rank, int *write_counter,
                        const float *new_row) {
    int rk = *rank;
    if (rk == 0 || cols == 0) {
        *rows += 1;
        return;
    }
    for (int r = 0; r < rk; r++) {
        float dot = 0.0f;
        for (int c = 0; c < cols; c++) dot += new_row[c] * vt[(size_t)r * cols + c];
        u_s[(size_t)(*rows) * rk + r] = dot;
    }
    *rows += 1;
    *write_counter += 1;
    if (*write_counter % 512 == 0 && *rows > rk) {
        int m = *rows;
        float *rec = (float *)malloc(sizeof(float) * (size_t)m * cols);
        orc_lowrank_reconstruct(u_s, vt, m, cols, rk, rec);
        int nr = rk < m ? rk : m;
        if (cols < nr) nr = cols;
        lr_power_iteration_svd(rec, (size_t)m, (size_t)cols, (size_t)nr, u_s, vt);
        free(rec);
        *rank = nr;
        *write_counter = 0;
    }
}

/* CompressedKVCache::write_kv's low-rank branch (:842-853) replayed over rows 0..rows-1 of one
 * (layer, head): the first row is decomposed, every later row updates.  u_s holds rows * rank_cfg
 * floats, vt rank_cfg * cols; returns the final rank. */
int orc_lowrank_replay(const float *k_rows, int rows, int cols, int rank_cfg, float *u_s, float *vt) {
    if (rows <= 0) return 0;
    int rank = orc_lowrank_decompose(k_rows, 1, cols, rank_cfg, u_s, vt);
    int n = 1, counter = 0;
    for (int i = 1; i < rows; i++) orc_lowrank_update(u_s, vt, &n, cols, &rank, &counter, k_rows + (size_t)i * cols);
    return rank;
}

/* ---- RoPE: validate_rope_caches (:71-110) + apply_rope_in_place (:177-231)
 * + rotate_rope_block (:137-160) ---------------------------------------- */
int orc_apply_rope(float *x, int b, int h, int sq, int d,
                   const float *cos_cache, const float *sin_cache,
                   int cache_rows, int cache_cols,
                   const int64_t *positions, int n_positions,
                   int interleaved, int rotary_dim) {
    if (n_positions != b * sq && n_positions != sq) return ORC_SHAPE_MISMATCH;
    if (rotary_dim == 0 || rotary_dim > d) return ORC_INVALID_ATTRIBUTE;
    if (rotary_dim % 2 != 0) return ORC_INVALID_ATTRIBUTE;
    int half = rotary_dim / 2;
    if (cache_cols != half) return ORC_SHAPE_MISMATCH;
    size_t head_stride = (size_t)sq * d, batch_stride = (size_t)h * head_stride;
    for (int bi = 0; bi < b; bi++)
        for (int hi = 0; hi < h; hi++)
            for (int qi = 0; qi < sq; qi++) {
                int64_t pos = n_positions == sq ? positions[qi] : positions[(size_t)bi * sq + qi];
                if (pos < 0 || pos >= cache_rows) return ORC_SHAPE_MISMATCH;
                float *base = x + bi * batch_stride + hi * head_stride + (size_t)qi * d;
                for (int pair = 0; pair < half; pair++) {
                    float c = cos_cache[(size_t)pos * cache_cols + pair];
                    float s = sin_cache[(size_t)pos * cache_cols + pair];
                    int i0 = interleaved ? 2 * pair : pair;
                    int i1 = interleaved ? 2 * pair + 1 : pair + half;
                    float x0 = base[i0], x1 = base[i1];
                    base[i0] = c * x0 - s * x1;
                    base[i1] = s * x0 + c * x1;
                }
            }
    return ORC_OK;
}

/* ---- SDPA (ops/microsoft.rs:241-438) ---------------------------------- */
static void sdpa_row(float *out, const float *qrow, const float *kbase, const float *vbase,
                     int sk, int d, int max_k, float scale, float *scores) {
    /* sdpa_scores_row (:241-264) */
    for (int ki = 0; ki < sk; ki++) {
        if (ki >= max_k) {
            scores[ki] = -INFINITY;
            continue;
        }
        const float *kr = kbase + (size_t)ki * d;
        float acc = 0.0f;
        for (int j = 0; j < d; j++) acc += qrow[j] * kr[j];
        scores[ki] = acc * scale;
    }
    /* sdpa_softmax (:270-299) */
    float mx = -INFINITY;
    for (int ki = 0; ki < sk; ki++)
        if (scores[ki] > mx) mx = scores[ki];
    int ok = isfinite(mx);
    float denom = 0.0f;
    if (ok) {
        for (int ki = 0; ki < sk; ki++) {
            float e = isfinite(scores[ki]) ? orc_expf_approx(scores[ki] - mx) : 0.0f;
            denom += e;
            scores[ki] = e;
        }
        if (denom == 0.0f) ok = 0;
    }
    if (!ok) { /* sdpa_write_zero_row (:322-326) */
        for (int j = 0; j < d; j++) out[j] = 0.0f;
        return;
    }
    float inv = 1.0f / denom;
    for (int ki = 0; ki < sk; ki++) scores[ki] *= inv;
    /* sdpa_write_weighted_v (:302-319) */
    for (int j = 0; j < d; j++) {
        float acc = 0.0f;
        for (int ki = 0; ki < sk; ki++) acc += scores[ki] * vbase[(size_t)ki * d + j];
        out[j] = acc;
    }
}

int orc_sdpa(const float *q, const float *k, const float *v, float *out,
             int batch, int hq, int hk, int sq, int sk, int d,
             int past_sk, float scale, int causal) {
    if (hq == 0 || hk == 0 || d == 0) return ORC_SHAPE_MISMATCH;
    if (hq % hk != 0) return ORC_SHAPE_MISMATCH;
    int group = hq / hk;
    size_t out_len = (size_t)batch * hq * sq * d;
    for (size_t i = 0; i < out_len; i++) out[i] = 0.0f;
    if (sk == 0) return ORC_OK;
    float *scores = (float *)malloc(sizeof(float) * (size_t)sk);
    for (int bi = 0; bi < batch; bi++)
        for (int qh = 0; qh < hq; qh++) {
            int kh = qh / group;
            const float *qb = q + ((size_t)bi * hq + qh) * sq * d;
            const float *kb = k + ((size_t)bi * hk + kh) * sk * d;
            const float *vb = v + ((size_t)bi * hk + kh) * sk * d;
            float *ob = out + ((size_t)bi * hq + qh) * sq * d;
            for (int qi = 0; qi < sq; qi++) {
                int max_k = causal ? (past_sk + qi + 1 < sk ? past_sk + qi + 1 : sk) : sk;
                sdpa_row(ob + (size_t)qi * d, qb + (size_t)qi * d, kb, vb, sk, d, max_k, scale, scores);
            }
        }
    free(scores);
    return ORC_OK;
}

/* reshape_to_bhsd (:660-677): (B, Sq, H*D) -> (B, H, Sq, D) */
static void reshape_to_bhsd(const float *src, float *dst, int b, int sq, int h, int d) {
    for (int bi = 0; bi < b; bi++)
        for (int si = 0; si < sq; si++)
            for (int hi = 0; hi < h; hi++)
                for (int j = 0; j < d; j++)
                    dst[(((size_t)bi * h + hi) * sq + si) * d + j] = src[(((size_t)bi * sq + si) * h + hi) * d + j];
}

/* reshape_from_bhsd (:682-704) */
static void reshape_from_bhsd(const float *src, float *dst, int b, int h, int sq, int d) {
    for (int bi = 0; bi < b; bi++)
        for (int hi = 0; hi < h; hi++)
            for (int si = 0; si < sq; si++)
                for (int j = 0; j < d; j++)
                    dst[(((size_t)bi * sq + si) * h + hi) * d + j] = src[(((size_t)bi * h + hi) * sq + si) * d + j];
}

/* kv_copy_block (:737-758) */
static void kv_copy_block(float *dst, const float *src, int b, int h, int src_sk, int total_sk,
                          int d, int dst_start) {
    for (int bi = 0; bi < b; bi++)
        for (int hi = 0; hi < h; hi++)
            for (int si = 0; si < src_sk; si++)
                memcpy(dst + (((size_t)bi * h + hi) * total_sk + dst_start + si) * d,
                       src + (((size_t)bi * h + hi) * src_sk + si) * d, sizeof(float) * (size_t)d);
}

/* op_group_query_attention (:1082-1196) with gqa_validate (:933-985),
 * gqa_apply_rotary (:1004-1050) and kv_concat (:762-794). */
int orc_group_query_attention(const float *query, const float *key, const float *value,
                              const float *past_key, const float *past_value,
                              int b, int sq, int q_hidden, int kv_hidden, int past_sk,
                              const float *cos_cache, const float *sin_cache,
                              int cache_rows, int cache_cols,
                              int64_t num_heads_i, int64_t kv_num_heads_i,
                              int has_scale, float scale_attr,
                              int64_t local_window_size, int do_rotary, int rotary_interleaved,
                              float *attn_out, float *present_k, float *present_v) {
    if (local_window_size != -1) return ORC_INVALID_ATTRIBUTE;
    if (!query || !key || !value) return ORC_SHAPE_MISMATCH;
    if (num_heads_i <= 0 || kv_num_heads_i <= 0) return ORC_INVALID_ATTRIBUTE;
    if (num_heads_i % kv_num_heads_i != 0) return ORC_INVALID_ATTRIBUTE;
    int nh = (int)num_heads_i, kvh = (int)kv_num_heads_i;
    if (q_hidden % nh != 0) return ORC_SHAPE_MISMATCH;
    if (kv_hidden % kvh != 0) return ORC_SHAPE_MISMATCH;
    int d = q_hidden / nh;
    if (kv_hidden / kvh != d) return ORC_SHAPE_MISMATCH;
    if ((past_key == NULL) != (past_value == NULL) && past_sk > 0) return ORC_SHAPE_MISMATCH;

    size_t qn = (size_t)b * nh * sq * d, kn = (size_t)b * kvh * sq * d;
    float *qb = (float *)malloc(sizeof(float) * qn);
    float *kb = (float *)malloc(sizeof(float) * kn);
    float *vb = (float *)malloc(sizeof(float) * kn);
    reshape_to_bhsd(query, qb, b, sq, nh, d);
    reshape_to_bhsd(key, kb, b, sq, kvh, d);
    reshape_to_bhsd(value, vb, b, sq, kvh, d);
    int rc = ORC_OK;
    if (do_rotary) {
        if (!cos_cache || !sin_cache) { rc = ORC_SHAPE_MISMATCH; goto done; }
        int64_t *pos = (int64_t *)malloc(sizeof(int64_t) * (size_t)(sq > 0 ? sq : 1));
        for (int i = 0; i < sq; i++) pos[i] = past_sk + i;
        rc = orc_apply_rope(qb, b, nh, sq, d, cos_cache, sin_cache, cache_rows, cache_cols, pos, sq,
                            rotary_interleaved, d);
        if (rc == ORC_OK)
            rc = orc_apply_rope(kb, b, kvh, sq, d, cos_cache, sin_cache, cache_rows, cache_cols, pos, sq,
                                rotary_interleaved, d);
        free(pos);
        if (rc != ORC_OK) goto done;
    }
    {
        int total = past_sk + sq;
        if (past_sk > 0) {
            kv_copy_block(present_k, past_key, b, kvh, past_sk, total, d, 0);
            kv_copy_block(present_v, past_value, b, kvh, past_sk, total, d, 0);
        }
        kv_copy_block(present_k, kb, b, kvh, sq, total, d, past_sk);
        kv_copy_block(present_v, vb, b, kvh, sq, total, d, past_sk);
        float scale = has_scale ? scale_attr : 1.0f / orc_sqrt_f32((float)d);
        float *ob = (float *)malloc(sizeof(float) * qn);
        rc = orc_sdpa(qb, present_k, present_v, ob, b, nh, kvh, sq, total, d, past_sk, scale, 1);
        if (rc == ORC_OK) reshape_from_bhsd(ob, attn_out, b, nh, sq, d);
        free(ob);
    }
done:
    free(qb);
    free(kb);
    free(vb);
    return rc;
}

/* ---- compressed composite ---------------------------------------------- */
typedef struct {
    const float *q;
    const uint8_t *k_codes, *v_codes;
    const float *k_meta, *v_meta;
    const int8_t *signs;
    int batch, hq, hk, sq, t, d, bits;
    float scale;
    float *out;
    int unit_begin, unit_end, stride;
    int first;
} cgqa_job;

static void cgqa_unit(const cgqa_job *j, int unit, float *kdec, float *vdec, float *scores) {
    int bi = unit / j->hk, kh = unit % j->hk, d = j->d, t = j->t;
    int cb = (d * j->bits + 7) / 8;
    int group = j->hq / j->hk;
    size_t base = ((size_t)bi * j->hk + kh) * t;
    const int8_t *sg = j->signs + (size_t)kh * d;
    /* CompressedKVCache::read_k / read_v (:862-899): decode every token. */
    for (int ti = 0; ti < t; ti++) {
        const float *km = j->k_meta + (base + ti) * 2, *vm = j->v_meta + (base + ti) * 2;
        orc_polar_decode(j->k_codes + (base + ti) * cb, km[0], km[1], d, j->bits, sg, kdec + (size_t)ti * d);
        orc_polar_decode(j->v_codes + (base + ti) * cb, vm[0], vm[1], d, j->bits, sg, vdec + (size_t)ti * d);
    }
    int past = t - j->sq;
    for (int g = 0; g < group; g++) {
        int qh = kh * group + g;
        for (int qi = 0; qi < j->sq; qi++) {
            const float *qrow = j->q + (((size_t)bi * j->hq + qh) * j->sq + qi) * d;
            float *orow = j->out + (((size_t)bi * j->sq + qi) * j->hq + qh) * d;
            int max_k = past + qi + 1 < t ? past + qi + 1 : t;
            sdpa_row(orow, qrow, kdec, vdec, t, d, max_k, j->scale, scores);
        }
    }
}

static void *cgqa_worker(void *arg) {
    const cgqa_job *j = (const cgqa_job *)arg;
    float *kdec = (float *)malloc(sizeof(float) * (size_t)j->t * j->d);
    float *vdec = (float *)malloc(sizeof(float) * (size_t)j->t * j->d);
    float *scores = (float *)malloc(sizeof(float) * (size_t)(j->t > 0 ? j->t : 1));
    for (int u = j->unit_begin + j->first; u < j->unit_end; u += j->stride) cgqa_unit(j, u, kdec, vdec, scores);
    free(kdec);
    free(vdec);
    free(scores);
    return NULL;
}

int orc_compressed_gqa(const float *q, const uint8_t *k_codes, const float *k_meta,
                       const uint8_t *v_codes, const float *v_meta,
                       const int8_t *signs, int batch, int hq, int hk, int sq, int t,
                       int d, int bits, float scale, float *out, int nthreads,
                       int unit_begin, int unit_end) {
    if (hk <= 0 || hq % hk != 0 || !is_pow2(d) || !valid_bits(bits)) return ORC_SHAPE_MISMATCH;
    if (sq > t) return ORC_SHAPE_MISMATCH;
    int units = batch * hk;
    if (unit_end < 0 || unit_end > units) unit_end = units;
    if (unit_begin < 0) unit_begin = 0;
    if (t == 0) {
        memset(out, 0, sizeof(float) * (size_t)batch * sq * hq * d);
        return ORC_OK;
    }
    if (nthreads < 1) nthreads = 1;
    cgqa_job base = {q, k_codes, v_codes, k_meta, v_meta, signs, batch, hq, hk, sq, t, d, bits,
                     scale, out, unit_begin, unit_end, nthreads, 0};
    if (nthreads == 1) {
        cgqa_worker(&base);
        return ORC_OK;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    cgqa_job *jobs = (cgqa_job *)malloc(sizeof(cgqa_job) * (size_t)nthreads);
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = base;
        jobs[i].first = i;
        pthread_create(&th[i], NULL, cgqa_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return ORC_OK;
}

/* ---- gemm_f32 (gemm.rs:34-63, gemm_tile :121-156, micro-kernels :163-243) */
static void micro_kernel_generic(int k_stride, int n_stride, const float *a, const float *b, float *c,
                                 int i0, int j0, int k0, int mr, int nr, int kb) {
    for (int di = 0; di < mr; di++)
        for (int dj = 0; dj < nr; dj++) {
            float sum = 0.0f;
            for (int dk = 0; dk < kb; dk++)
                sum += a[(size_t)(i0 + di) * k_stride + (k0 + dk)] * b[(size_t)(k0 + dk) * n_stride + (j0 + dj)];
            c[(size_t)(i0 + di) * n_stride + (j0 + dj)] += sum;
        }
}

static void micro_kernel_8x8(int k_stride, int n_stride, const float *a, const float *b, float *c,
                             int i0, int j0, int k0, int kb) {
    float acc[8][8];
    memset(acc, 0, sizeof(acc));
    for (int dk = 0; dk < kb; dk++) {
        size_t a_base = (size_t)i0 * k_stride + (k0 + dk);
        size_t b_base = (size_t)(k0 + dk) * n_stride + j0;
        float av[8];
        for (int r = 0; r < 8; r++) av[r] = a[a_base + (size_t)r * k_stride];
        for (int dj = 0; dj < 8; dj++) {
            float bv = b[b_base + dj];
            for (int r = 0; r < 8; r++) acc[r][dj] += av[r] * bv;
        }
    }
    for (int r = 0; r < 8; r++)
        for (int dj = 0; dj < 8; dj++) c[(size_t)(i0 + r) * n_stride + j0 + dj] += acc[r][dj];
}

void orc_gemm_f32(int m, int n, int k, const float *a, const float *b, float *c) {
    const int T = 64;
    for (size_t i = 0; i < (size_t)m * n; i++) c[i] = 0.0f;
    for (int ii = 0; ii < m; ii += T) {
        int mb = T < m - ii ? T : m - ii;
        for (int jj = 0; jj < n; jj += T) {
            int nb = T < n - jj ? T : n - jj;
            for (int kk = 0; kk < k; kk += T) {
                int kb = T < k - kk ? T : k - kk;
                for (int i = 0; i < mb; i += 8) {
                    int mr = 8 < mb - i ? 8 : mb - i;
                    for (int j = 0; j < nb; j += 8) {
                        int nr = 8 < nb - j ? 8 : nb - j;
                        if (mr == 8 && nr == 8)
                            micro_kernel_8x8(k, n, a, b, c, ii + i, jj + j, kk, kb);
                        else
                            micro_kernel_generic(k, n, a, b, c, ii + i, jj + j, kk, mr, nr, kb);
                    }
                }
            }
        }
    }
}

/* MatMulNBits: Y(M,N) = A(M,K) * W^T with W[n][k] = (code - zp) * scale[n][k/block].
 * ORT com.microsoft.MatMulNBits contract (not in the reference); the
 * contraction is gemm_f32 above. */
int orc_matmul_nbits(const float *a, const uint8_t *b_codes, const float *scales,
                     const uint8_t *zero_points, float *y, int m, int n, int k,
                     int bits, int block_size) {
    if (bits != 4) return ORC_UNSUPPORTED;
    if (block_size < 16 || !is_pow2(block_size)) return ORC_INVALID_ATTRIBUTE;
    int nblk = (k + block_size - 1) / block_size;
    int blob = block_size * bits / 8;
    int zp_row = (nblk * bits + 7) / 8;
    float *wt = (float *)malloc(sizeof(float) * (size_t)k * n);
    for (int nn = 0; nn < n; nn++)
        for (int kk = 0; kk < k; kk++) {
            int blk = kk / block_size, in_blk = kk % block_size;
            uint8_t byte = b_codes[((size_t)nn * nblk + blk) * blob + in_blk / 2];
            uint32_t code = (in_blk & 1) ? (byte >> 4) : (byte & 15u);
            uint32_t zp = 8u;
            if (zero_points) {
                uint8_t zb = zero_points[(size_t)nn * zp_row + blk / 2];
                zp = (blk & 1) ? (zb >> 4) : (zb & 15u);
            }
            float s = scales[(size_t)nn * nblk + blk];
            wt[(size_t)kk * n + nn] = ((float)code - (float)zp) * s;
        }
    orc_gemm_f32(m, n, k, a, wt, y);
    free(wt);
    return ORC_OK;
}

/* ---- decoder-layer glue ----------------------------------------------------
 * sqrt of op_rms_normalization: libm_sqrt (ops/generative.rs:96-106), 16
 * Newton steps from x, 0 for x <= 0. */
static float libm_sqrt_newton(float x) {
    if (x <= 0.0f) return 0.0f;
    float guess = x;
    for (int i = 0; i < 16; i++) guess = 0.5f * (guess + x / guess);
    return guess;
}

/* SkipSimplifiedLayerNormalization (ops/microsoft.rs:491-540) over rows of
 * `cols`: pre = x + skip (+ bias), y = rms_norm(pre) * w with
 * op_rms_normalization (ops/generative.rs:517-580): ss accumulated in index
 * order, rms_inv = 1 / libm_sqrt(ss / n + eps), y = v * rms_inv * w.  With
 * skip == NULL it is SimplifiedLayerNormalization without its bias. */
void orc_rms_norm(const float *x, const float *skip, const float *bias, const float *w, float *y, float *pre,
                  int rows, int cols, float eps) {
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * cols;
        float *pr = pre + (size_t)r * cols;
        float ss = 0.0f;
        for (int i = 0; i < cols; i++) {
            float v = xr[i];
            if (skip) v = v + skip[(size_t)r * cols + i];
            if (bias) v = v + bias[i];
            pr[i] = v;
            ss += v * v;
        }
        float rms_inv = 1.0f / libm_sqrt_newton(ss / (float)cols + eps);
        for (int i = 0; i < cols; i++) y[(size_t)r * cols + i] = pr[i] * rms_inv * w[i];
    }
}

/* SwiGLU: Swish (ops/activations.rs:37-39, x / (1 + expf_approx(-x))) of the
 * gate times up (the Mul of GraphBuilder::swiglu, graph_builder.rs:366-369). */
void orc_silu_mul(const float *gate, const float *up, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = gate[i] / (1.0f + orc_expf_approx(-gate[i])) * up[i];
}

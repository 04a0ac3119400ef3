// Internal (non-ABI) structures shared by the sa_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sa_b200.h"

namespace sa {

constexpr int kCapacityAlign = 64;   // token capacity is padded to this
constexpr int kVGroup = 4;           // V codes are byte-interleaved by 4 tokens ...
constexpr int kVBlock = 16;          // ... and 16-byte chunks of 4 such groups interleave in 16-token blocks

// Byte offset, within one (row, head)'s V codes, of byte j of token t
// (cb = code bytes per token, a multiple of 4): 16-token blocks of 16*cb
// bytes; inside a block, 16-byte chunk c of token group g (4 tokens) sits at
// c*64 + g*16, and a group's bytes are ordered k = 4*j + t%4.
__host__ __device__ __forceinline__ int64_t v_byte_offset(int64_t t, int j, int cb) {
    const int k = 4 * j + (int)(t & 3);
    return (t >> 4) * (int64_t)(16 * cb) + (k >> 4) * 64 + ((t >> 2) & 3) * 16 + (k & 15);
}
constexpr int kMaxSplits = 64;       // split-K partitions per (row, kv head)
constexpr int kMaxGather = 8;        // ranks of one node in the head-sharded mode

// Head-sharded output: the attention output of this rank's query heads goes
// to every buffer p[0..n) (this GPU's and its peers', mapped into this
// process) at columns [col0, col0 + heads*group) of a [B][S][cols*D] tensor.
// With signal arrays (sig[0] != nullptr) the writing kernel also completes
// the gather on the device (sa_gather.cuh): sig[r] is rank r's array of
// kMaxGather + 2 words, mapped here (one epoch per peer, then this rank's
// CTA counter and epoch), and this rank is buffer `rank`.
struct GatherOut {
    void *p[kMaxGather];
    int n;     // 0: plain attn_out
    int col0;  // first global query head of this rank
    int cols;  // query heads in total
    uint32_t *sig[kMaxGather];  // nullptr: the caller synchronises the ranks itself
    int rank;
    uint32_t *state;      // sig[rank] + kMaxGather: {CTA counter, epoch}
    int *status;          // this cache's device status word
    uint64_t timeout_ns;  // bound of the wait for the peers' epochs
};

struct kv_cache_impl {
    sa_kv_cache_config cfg;
    int device;
    int sm_count;
    int capacity;      // padded token capacity
    int code_bytes;    // head_dim * bits / 8
    int group;         // num_heads / num_kv_heads
    float wht_scale;   // 1 / sqrt_approx(head_dim)
    int64_t position;  // committed tokens
    // one device allocation carved into the arrays below
    void *base;
    size_t base_bytes;
    uint8_t *k_codes;  // [L][B][H][T][CB]
    uint8_t *v_codes;  // [L][B][H][T/4][CB][4]
    float *k_meta;     // [L][B][H][T][2]
    float *v_meta;     // [L][B][H][T][2]
    float *signs;      // [L][H][D]  +-1.0f
    float *workspace;  // split-K partials
    size_t workspace_floats;
    uint32_t *qprep;   // [B*H] x decode_qprep_words(group): q-digit words, then score constants
    int *dev_status;   // one int: device-side status bits
    GatherOut gather;  // head-sharded output buffers (n = 0: off)
    size_t layer_codes_bytes;  // B*H*T*CB
    size_t layer_meta_floats;  // B*H*T*2
    uint8_t *k_qjl_bits;       // [L][B][H][T][D/8], nullptr unless cfg.qjl_residual
    uint8_t *v_qjl_bits;
    float *k_qjl_mag;          // [L][B][H][T]
    float *v_qjl_mag;
    size_t layer_qjl_bytes;    // B*H*T*D/8
    size_t layer_qjl_floats;   // B*H*T
    float *lr_vt;              // [L][B][H][D], nullptr unless cfg.lowrank_k
    float *lr_us;              // [L][B][H][T]
    float *lr_scratch;         // [L][B][H][T]: the power iteration's u vector
    float *lr_kmeta;           // [L][B][H][T][2]: {0, U*S[t]}, the K metadata attention reads
    float *lr_vtr;             // [L][B][H][D]: V^T rotated like q' (signs, WHT, 1/sqrt(n))
    size_t layer_lr_vt_floats; // B*H*D
    size_t layer_lr_us_floats; // B*H*T
};

// Parameters of one append launch (K and V of `batch * seq_len` tokens).
struct AppendArgs {
    const void *key;
    const void *value;
    int dtype;
    int batch, seq_len, heads, head_dim, bits, code_bytes, capacity;
    int64_t pos0;
    uint8_t *k_codes, *v_codes;
    float *k_meta, *v_meta;
    const float *signs;
    float wht_scale;
    const float *cos_cache, *sin_cache;
    int cache_rows, do_rotary, interleaved;
    // QJL residuals of the appended vectors (all nullptr: not stored)
    uint8_t *k_qjl_bits, *v_qjl_bits;
    float *k_qjl_mag, *v_qjl_mag;
    // low-rank K state (all nullptr: off)
    float *lr_vt, *lr_us, *lr_scratch, *lr_kmeta, *lr_vtr;
};

// Parameters of the fused QKV projection's epilogue (one token per row):
// `ap` appends k_out / v_out (key / value, seq_len 1) at the cache position.
struct QkvArgs {
    AppendArgs ap;
    void *q_out;  // [batch][q_heads * head_dim], RoPE applied in place
    int q_heads;
};

// Parameters of one attention launch.
struct AttendArgs {
    const void *query;
    void *out;
    int dtype;
    int batch, seq_len, heads, group, head_dim, bits, code_bytes, capacity;
    int64_t pos0;  // tokens cached before query token 0
    const uint8_t *k_codes, *v_codes;
    const float *k_meta, *v_meta;
    const float *signs;
    float wht_scale;
    float scale;  // attention scale
    const float *cos_cache, *sin_cache;
    int cache_rows, do_rotary, interleaved;
    float *workspace;
    size_t workspace_floats;
    int sm_count;
    uint32_t *qprep;  // decode prep area: per (row, head) q-digit fragments + constants
    int *dev_status;  // device-side status word (bounded waits that gave up)
    GatherOut gather;  // head-sharded output (n = 0: write `out`)
    // low-rank K: V^T rotated like q' (nullptr: off).  With it, k_meta holds {0, U*S[t]} and the
    // zero-point term's sum(q') becomes q'.lr_vtr, so scores are U*S[t] * (q . V^T).
    const float *lr_vtr;
};

int launch_kv_append(const AppendArgs &a, cudaStream_t stream);
int launch_lowrank_append(const AppendArgs &a, cudaStream_t stream);
int launch_gqa_attend(const AttendArgs &a, cudaStream_t stream);
int launch_gather_scatter(const AttendArgs &a, cudaStream_t stream);
bool decode_fast_eligible(const AttendArgs &a);
size_t decode_workspace_floats(int sm_count, int64_t units, int head_dim, int group);
size_t decode_qprep_words(int group);
size_t decode8_workspace_floats(int sm_count, int64_t units, int head_dim);
size_t decode8_qprep_words();
int launch_gqa_decode8(const AttendArgs &a, const AppendArgs *append, cudaStream_t stream);
int launch_gqa_decode_fast(const AttendArgs &a, const AppendArgs *append, cudaStream_t stream);
bool prefill_eligible(const AttendArgs &a);
int launch_gqa_prefill_umma(const AttendArgs &a, cudaStream_t stream);
int launch_matmul_nbits(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp,
                        const void *bias, void *y, int dtype, int64_t m, int64_t n, int64_t k,
                        int block_size, cudaStream_t stream);
int launch_qkv_finish(const QkvArgs &a, cudaStream_t stream);
int launch_rms_norm(const void *x, const void *skip, const void *bias, const void *w, void *y, void *pre, int dtype,
                    int64_t rows, int64_t cols, float eps, cudaStream_t stream);
int launch_silu_mul(const void *gate, const void *up, int64_t ld_in, void *y, int dtype, int64_t rows, int64_t cols,
                    cudaStream_t stream);
int launch_qkv_umma_fused(const void *x, const uint8_t *w_codes, const void *w_scales, const QkvArgs &a,
                          int64_t n, int64_t k, cudaStream_t stream);
bool matmul_nbits_umma_eligible(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, int dtype,
                                int64_t m, int64_t n, int64_t k, int block_size);
int launch_matmul_nbits_umma(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y,
                             int dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream);
bool matmul_nbits_packable(int dtype, int64_t n, int64_t k, int block_size);
size_t matmul_nbits_packed_bytes(int64_t n, int64_t k);
int launch_matmul_nbits_prepack(const uint8_t *b, const void *scales, void *packed, int dtype, int64_t n, int64_t k,
                                cudaStream_t stream);
int launch_matmul_nbits_packed(const void *a, const void *packed, const void *bias, void *y, int dtype, int64_t m,
                               int64_t n, int64_t k, cudaStream_t stream);

void count_launch(int n = 1);
float host_sqrt_approx(float x);
float host_sqrt_f32(float x);

}  // namespace sa

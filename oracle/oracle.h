/*
 * CPU oracle for the smallaios_b200 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the
 * SmallAIOS onnx-rt Rust CPU path (the reference cannot be compiled in this
 * image: it is Rust and no rustc is installed).  Only tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline / --impl reference legs
 * of bench.py may load it, and only as the checker or the timed CPU
 * baseline.  The product library (libsa_b200.so) never links or calls it.
 *
 * Every function names the reference file:line it follows.  Build flags
 * are -O2 -ffp-contract=off (no FMA contraction, no fast-math) so that
 * every float operation rounds exactly as the Rust code does.
 */
#ifndef SA_ORACLE_H
#define SA_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes mirroring OpError variants used on this path
 * (onnx-rt/src/operators.rs OpError). */
#define ORC_OK 0
#define ORC_INVALID_ATTRIBUTE 1
#define ORC_SHAPE_MISMATCH 2
#define ORC_UNSUPPORTED 3

/* ---- scalar helpers ---------------------------------------------------- */
float orc_sqrt_approx(float x);     /* operators.rs:3311-3320 */
float orc_sqrt_f32(float x);        /* ops/microsoft.rs:54-62 */
float orc_expf_approx(float x);     /* operators.rs:1328-1357 */
float orc_round_f32(float x);       /* kv_compression.rs:27-37 */

/* ---- PolarQuant primitives (kv_compression.rs) ------------------------- */
uint64_t orc_xorshift64_next(uint64_t *state);                     /* :58-67 */
uint64_t orc_head_seed(uint64_t seed, int layer, int num_kv_heads, int head); /* :776-779 */
int orc_polar_signs(uint64_t seed, int dim, int8_t *signs);        /* :197-213 */
void orc_wht_with_signs(float *x, int n, const int8_t *signs);     /* :119-123 */
void orc_inverse_wht_with_signs(float *x, int n, const int8_t *signs); /* :134-139 */
void orc_pack_bits(const uint32_t *values, int count, int bits, uint8_t *out); /* :294-312 */
void orc_unpack_bits(const uint8_t *data, int nbytes, int count, int bits, uint32_t *out); /* :315-333 */
/* PolarQuantizer::encode (:216-267).  codes gets ceil(dim*bits/8) bytes. */
int orc_polar_encode(const float *in, int dim, int bits, const int8_t *signs,
                     uint8_t *codes, float *scale, float *zero_point,
                     float *min_val, float *max_val);
/* orc_polar_encode of n vectors x[n][dim] with one sign vector, split over
 * nthreads threads; codes[n][ceil(dim*bits/8)], meta[n][2] = {scale, zp}. */
int orc_polar_encode_batch(const float *x, size_t n, int dim, int bits, const int8_t *signs,
                           uint8_t *codes, float *meta, int nthreads);
/* PolarQuantizer::decode (:270-286). */
int orc_polar_decode(const uint8_t *codes, float scale, float zero_point,
                     int dim, int bits, const int8_t *signs, float *out);
/* QJLResidualEncoder::encode (:365-395).  sign_bits gets ceil(dim/64) words. */
void orc_qjl_encode(const float *original, const float *approx, int dim,
                    uint64_t *sign_bits, float *c_magnitude);
float orc_qjl_correction(const uint64_t *a_bits, float a_c, const uint64_t *b_bits, float b_c, int dim);
int orc_lowrank_decompose(const float *k, int rows, int cols, int rank, float *u_s, float *vt);
void orc_lowrank_reconstruct(const float *u_s, const float *vt, int rows, int cols, int rank, float *out);
void orc_lowrank_update(float *u_s, float *vt, int *rows, int cols, int *rank, int *write_counter,
                        const float *new_row);
int orc_lowrank_replay(const float *k_rows, int rows, int cols, int rank_cfg, float *u_s, float *vt);

/* ---- attention (ops/microsoft.rs) -------------------------------------- */
/* apply_rope_in_place (:177-231) over a (B, H, Sq, D) f32 tensor.
 * positions has Sq or B*Sq entries.  cos/sin are (rows, rotary_dim/2). */
int orc_apply_rope(float *x, int b, int h, int sq, int d,
                   const float *cos_cache, const float *sin_cache,
                   int cache_rows, int cache_cols,
                   const int64_t *positions, int n_positions,
                   int interleaved, int rotary_dim);
/* scaled_dot_product_attention (:380-438).  q (B,Hq,Sq,D), k/v (B,Hk,Sk,D). */
int orc_sdpa(const float *q, const float *k, const float *v, float *out,
             int batch, int hq, int hk, int sq, int sk, int d,
             int past_sk, float scale, int causal);
/* op_group_query_attention (:1082-1196).  past_sk may be 0 (no past).
 * present_k / present_v get (B, Hk, past_sk+Sq, D).  cos/sin may be NULL.
 * has_scale selects the `scale` attribute; otherwise 1/sqrt_f32(D). */
int orc_group_query_attention(const float *query, const float *key, const float *value,
                              const float *past_key, const float *past_value,
                              int batch, int sq, int q_hidden, int kv_hidden, int past_sk,
                              const float *cos_cache, const float *sin_cache,
                              int cache_rows, int cache_cols,
                              int64_t num_heads, int64_t kv_num_heads,
                              int has_scale, float scale_attr,
                              int64_t local_window_size, int do_rotary, int rotary_interleaved,
                              float *attn_out, float *present_k, float *present_v);

/* ---- compressed-cache composite (our composition; the reference never
 * wires kv_compression.rs into GQA) --------------------------------------
 * k_codes/v_codes: (B, Hk, T, code_bytes) in pack_bits order; k_meta/v_meta:
 * (B, Hk, T, 2) = {scale, zero_point}.  signs: (Hk, D) per-head sign vectors.
 * q: (B, Hq, Sq, D) already rotated by RoPE.  Decodes every token with
 * PolarQuantizer::decode (CompressedKVCache::read_k/read_v, :862-899), then
 * runs scaled_dot_product_attention with causal mask and past_sk = T - Sq.
 * out: (B, Sq, Hq*D).  nthreads > 1 splits (b, kv_head) units over pthreads
 * (used only for the timed CPU baseline). */
int orc_compressed_gqa(const float *q, const uint8_t *k_codes, const float *k_meta,
                       const uint8_t *v_codes, const float *v_meta,
                       const int8_t *signs, int batch, int hq, int hk, int sq, int t,
                       int d, int bits, float scale, float *out, int nthreads,
                       int unit_begin, int unit_end);

/* ---- MatMulNBits (parity unpinned: ORT com.microsoft.MatMulNBits contract
 * on top of gemm.rs) ------------------------------------------------------ */
/* gemm_f32 (gemm.rs:34-63, tile 64, micro-kernels 8x8 / generic). */
void orc_gemm_f32(int m, int n, int k, const float *a, const float *b, float *c);
/* Dequantize (q - zp) * scale in f32 into W^T (K, N) and run gemm_f32.
 * b_codes: (N, K/block, block*bits/8) uint8, low nibble first; scales (N, K/block)
 * as f32 (fp16 widened by the caller); zero_points: NULL (=> 2^(bits-1)) or
 * packed uint8 (N, ceil(K/block*bits/8)). */
int orc_matmul_nbits(const float *a, const uint8_t *b_codes, const float *scales,
                     const uint8_t *zero_points, float *y, int m, int n, int k,
                     int bits, int block_size);

#ifdef __cplusplus
}
#endif
#endif

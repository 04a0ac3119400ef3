// The epilogue of the fused QKV projection (decode step, one token per row):
// the projection has been rounded to the activation type and stored as
// q_out [B][Hq*D], k_out / v_out [B][Hkv*D]; one warp then finishes one head
// vector of one row:
//   query head : RoPE in place (rotate_rope_block order, ops/microsoft.rs:137-160);
//   key head   : quantize-on-append of RoPE(k) (the append encoder);
//   value head : quantize-on-append of v.
// Heads are numbered in the packed projection's order: Hq query heads, then
// Hkv key heads, then Hkv value heads.
#pragma once

#include "sa_append.cuh"

namespace sa {

template <typename T, int EPL>
__device__ __forceinline__ void qkv_finish_vector(const QkvArgs &a, int m, int hh, int lane, uint8_t *s_codes) {
    const int d = a.ap.head_dim;
    if (hh < a.q_heads) {
        if (!a.ap.do_rotary) return;
        T *src = static_cast<T *>(a.q_out) + ((int64_t)m * a.q_heads + hh) * d;
        const bool active = lane * EPL < d;  // head_dim 16 uses half the lanes
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            x[r] = active ? rope_element(src, ld_f32(src + e), e, d, a.ap.pos0, a.ap.cos_cache, a.ap.sin_cache,
                                         a.ap.interleaved)
                          : 0.0f;
        }
        __syncwarp();  // every lane has read its partners
        if (active) {
#pragma unroll
            for (int r = 0; r < EPL; r++) st_from_f32(src + lane * EPL + r, x[r]);
        }
        return;
    }
    const int kv = hh - a.q_heads;
    if (kv < a.ap.heads) encode_append_vector<T, EPL>(a.ap, m, 0, kv, 0, lane, s_codes);
    else encode_append_vector<T, EPL>(a.ap, m, 0, kv - a.ap.heads, 1, lane, s_codes);
}

}  // namespace sa

// Quantize-on-append of one vector: RoPE (K only) + PolarQuant encode + bit
// packing by one warp.  Bit-exact with PolarQuantizer::encode
// (kv_compression.rs:216-267) on the f32 value of the input: every float
// operation is an explicitly rounded intrinsic in the reference's order, so
// nvcc cannot contract or reassociate it.  Shared by the append kernel and
// the decode prep kernel.
#pragma once

#include <type_traits>

#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

// Signed-integer key with the order of the (non-NaN) float x: non-negative floats keep their
// bits, negative ones flip the magnitude bits.
__device__ __forceinline__ int order_key(float x) {
    const int i = __float_as_int(x);
    return i >= 0 ? i : (i ^ 0x7fffffff);
}

// RoPE of element e of a vector at `pos` (rotate_rope_block,
// ops/microsoft.rs:137-160): y0 = c*x0 - s*x1, y1 = s*x0 + c*x1, each product
// rounded before the add.  `x` is element e, `src` the whole input vector.
template <typename T>
__device__ __forceinline__ float rope_element(const T *src, float x, int e, int d, int64_t pos, const float *cos_cache,
                                              const float *sin_cache, int interleaved) {
    const int half = d / 2;
    int pair, partner;
    bool first;
    if (interleaved) {
        pair = e >> 1;
        first = (e & 1) == 0;
        partner = first ? e + 1 : e - 1;
    } else {
        first = e < half;
        pair = first ? e : e - half;
        partner = first ? e + half : e - half;
    }
    const float c = cos_cache[pos * half + pair], sn = sin_cache[pos * half + pair];
    const float xo = ld_f32(src + partner);
    return first ? __fsub_rn(__fmul_rn(c, x), __fmul_rn(sn, xo)) : __fadd_rn(__fmul_rn(sn, xo), __fmul_rn(c, x));
}

// The EPL consecutive elements at p as f32: one vector load when p is aligned to their size.
template <typename T, int EPL>
__device__ __forceinline__ void load_elems(const T *p, float (&x)[EPL]) {
    constexpr int kBytes = EPL * (int)sizeof(T);
    if constexpr (kBytes == 16 || kBytes == 8 || kBytes == 4) {
        if ((reinterpret_cast<uintptr_t>(p) & (kBytes - 1)) == 0) {
            using V = typename std::conditional<kBytes == 16, uint4,
                                                typename std::conditional<kBytes == 8, uint2, uint32_t>::type>::type;
            union {
                V v;
                T t[EPL];
            } u;
            u.v = *reinterpret_cast<const V *>(p);
#pragma unroll
            for (int r = 0; r < EPL; r++) x[r] = DT<T>::to_f32(u.t[r]);
            return;
        }
    }
#pragma unroll
    for (int r = 0; r < EPL; r++) x[r] = ld_f32(p + r);
}

// RoPE of the EPL consecutive elements lane * EPL .. of a d-element vector held by a warp
// (rotate_rope_block, ops/microsoft.rs:137-160: y0 = c*x0 - s*x1, y1 = s*x0 + c*x1, each
// product rounded before the add).  The partner of element e is e ^ 1 (interleaved) or e +- d/2,
// held by lane ^ (d / 2 / EPL) at the same slot, so it comes by a shuffle instead of a reload.
// All 32 lanes must call it; lanes past d hold zeros and are left alone.
template <int EPL>
__device__ __forceinline__ void rope_lane(float (&x)[EPL], int lane, int d, int64_t pos, const float *cos_cache,
                                          const float *sin_cache, int interleaved) {
    float xp[EPL];
    if (interleaved) {
        if constexpr (EPL >= 2) {
#pragma unroll
            for (int r = 0; r < EPL; r++) xp[r] = x[r ^ 1];
        } else {
            xp[0] = __shfl_xor_sync(0xffffffffu, x[0], 1);
        }
    } else {
        const int m = d / 2 / EPL;
#pragma unroll
        for (int r = 0; r < EPL; r++) xp[r] = __shfl_xor_sync(0xffffffffu, x[r], m);
    }
    if (lane * EPL < d) {
        const int half = d / 2;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            const bool first = interleaved ? (e & 1) == 0 : e < half;
            const int pair = interleaved ? e >> 1 : (first ? e : e - half);
            const float c = cos_cache[pos * half + pair], sn = sin_cache[pos * half + pair];
            x[r] = first ? __fsub_rn(__fmul_rn(c, x[r]), __fmul_rn(sn, xp[r]))
                         : __fadd_rn(__fmul_rn(sn, xp[r]), __fmul_rn(c, x[r]));
        }
    }
}

// PolarQuantizer::encode (kv_compression.rs:216-267) of NV vectors a warp holds, EPL elements
// per lane each (x, rotated in place): apply_signs, butterfly and 1/sqrt_approx(n) (:81-123), the
// first-occurrence min / max, scale = range / levels and codes round_f32((v - zp) / scale).  sg
// holds this lane's signs (1 on inactive lanes), shared by the NV vectors.  The vectors are
// independent: each step is issued for all of them before the next, so their shuffle and
// reduction latencies overlap.  All 32 lanes must call it.
template <int EPL, int NV = 1>
__device__ __forceinline__ void polar_encode_warp(float (&x)[NV][EPL], const float (&sg)[EPL], bool active, int lane,
                                                  int d, float wht_scale, uint32_t levels,
                                                  uint32_t (&qc)[NV][EPL], float (&scale)[NV], float (&zp)[NV]) {
#pragma unroll
    for (int v = 0; v < NV; v++)
#pragma unroll
        for (int r = 0; r < EPL; r++) x[v][r] = __fmul_rn(x[v][r], sg[r]);
    // the butterfly (warp_wht_butterfly) of the NV vectors, stage by stage
#pragma unroll
    for (int hs = 1; hs < EPL; hs <<= 1)
#pragma unroll
        for (int v = 0; v < NV; v++)
#pragma unroll
            for (int r = 0; r < EPL; r++)
                if ((r & hs) == 0) {
                    const float p0 = x[v][r], p1 = x[v][r + hs];
                    x[v][r] = __fadd_rn(p0, p1);
                    x[v][r + hs] = __fsub_rn(p0, p1);
                }
    for (int lm = 1; lm < d / EPL; lm <<= 1) {
        float other[NV][EPL];
#pragma unroll
        for (int v = 0; v < NV; v++)
#pragma unroll
            for (int r = 0; r < EPL; r++) other[v][r] = __shfl_xor_sync(0xffffffffu, x[v][r], lm);
#pragma unroll
        for (int v = 0; v < NV; v++)
#pragma unroll
            for (int r = 0; r < EPL; r++)
                x[v][r] = (lane & lm) ? __fsub_rn(other[v][r], x[v][r]) : __fadd_rn(x[v][r], other[v][r]);
    }
#pragma unroll
    for (int v = 0; v < NV; v++)
#pragma unroll
        for (int r = 0; r < EPL; r++) x[v][r] = __fmul_rn(x[v][r], wht_scale);

    // min / max with strict comparisons in index order: the first occurrence
    // wins, as in the sequential loop of encode (this matters for +-0).
    float mn[NV], mx[NV];
    int imn[NV], imx[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) {
        mn[v] = INFINITY;
        mx[v] = -INFINITY;
        imn[v] = imx[v] = 0x7fffffff;
        if (active) {
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                const int e = lane * EPL + r;
                if (x[v][r] < mn[v]) {
                    mn[v] = x[v][r];
                    imn[v] = e;
                }
                if (x[v][r] > mx[v]) {
                    mx[v] = x[v][r];
                    imx[v] = e;
                }
            }
        }
    }
    // Across the warp: the extreme value by an integer reduction over an order-preserving key
    // (-0 and +0 share the key of +0, since they compare equal), then the lowest element index
    // among the lanes holding that value, and that element's own bits.
    int kmn[NV], kmx[NV], wmn[NV], wmx[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) {
        kmn[v] = __reduce_min_sync(0xffffffffu, order_key(mn[v] + 0.0f));
        kmx[v] = __reduce_max_sync(0xffffffffu, order_key(mx[v] + 0.0f));
    }
#pragma unroll
    for (int v = 0; v < NV; v++) {
        wmn[v] = __reduce_min_sync(0xffffffffu, order_key(mn[v] + 0.0f) == kmn[v] ? imn[v] : 0x7fffffff);
        wmx[v] = __reduce_min_sync(0xffffffffu, order_key(mx[v] + 0.0f) == kmx[v] ? imx[v] : 0x7fffffff);
    }
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const unsigned lmn = __ballot_sync(0xffffffffu, order_key(mn[v] + 0.0f) == kmn[v] && imn[v] == wmn[v]);
        const unsigned lmx = __ballot_sync(0xffffffffu, order_key(mx[v] + 0.0f) == kmx[v] && imx[v] == wmx[v]);
        mn[v] = __shfl_sync(0xffffffffu, mn[v], __ffs(lmn) - 1);
        mx[v] = __shfl_sync(0xffffffffu, mx[v], __ffs(lmx) - 1);
    }

#pragma unroll
    for (int v = 0; v < NV; v++) {
        const float range = __fsub_rn(mx[v], mn[v]);
        const float sc = range > 0.0f ? __fdiv_rn(range, (float)levels) : 1.0f;
        scale[v] = sc;
        zp[v] = mn[v];
        // (x - zp) / scale with x - zp in [0, levels * scale]: by Markstein's correction from one
        // reciprocal when scale is in [2^-90, 2^100] (warp-uniform), else by division; both give
        // the correctly rounded quotient.
        const bool fast = sc >= 0x1p-90f && sc <= 0x1p100f;
        const float rcp = fast ? __frcp_rn(sc) : 1.0f;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            uint32_t q = 0u;
            if (active && sc > 0.0f) {
                const float num = __fsub_rn(x[v][r], mn[v]);
                q = __float2uint_rz(rust_round_f32(fast ? div_rn_markstein(num, sc, rcp) : __fdiv_rn(num, sc)));
            }
            qc[v][r] = q < levels ? q : levels;
        }
    }
}

// Encode and store vector (b, s, h, which) of an append (which: 0 = K, 1 = V).
// All 32 lanes of the warp must call it; s_codes holds >= head_dim bytes.
template <typename T, int EPL>
__device__ __forceinline__ void encode_append_vector(const AppendArgs &a, int b, int s, int h, int which, int lane,
                                                     uint8_t *s_codes) {
    const int d = a.head_dim;
    const int64_t pos = a.pos0 + s;
    const bool active = lane * EPL < d;
    const T *src = static_cast<const T *>(which ? a.value : a.key) + (((int64_t)b * a.seq_len + s) * a.heads + h) * d;
    float x[EPL];
    if (active) {
        load_elems<T, EPL>(src + lane * EPL, x);
    } else {
#pragma unroll
        for (int r = 0; r < EPL; r++) x[r] = 0.0f;
    }
    if (which == 0 && a.do_rotary)  // warp-uniform
        rope_lane<EPL>(x, lane, d, pos, a.cos_cache, a.sin_cache, a.interleaved);

    float x0[EPL];  // the vector as written (after RoPE): the QJL residual is taken against it
#pragma unroll
    for (int r = 0; r < EPL; r++) x0[r] = x[r];

    const float *sgp = a.signs + (int64_t)h * d;
    float sg[EPL];
#pragma unroll
    for (int r = 0; r < EPL; r++) sg[r] = active ? sgp[lane * EPL + r] : 1.0f;
    const uint32_t levels = (1u << a.bits) - 1u;
    uint32_t qc[EPL];  // the codes of this lane's elements
    float scale, zp;
    {
        float xv[1][EPL];
        uint32_t qv[1][EPL];
        float sv[1], zv[1];
#pragma unroll
        for (int r = 0; r < EPL; r++) xv[0][r] = x[r];
        polar_encode_warp<EPL, 1>(xv, sg, active, lane, d, a.wht_scale, levels, qv, sv, zv);
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            x[r] = xv[0][r];
            qc[r] = qv[0][r];
        }
        scale = sv[0];
        zp = zv[0];
    }

    // pack_bits (kv_compression.rs:294-312): LSB-first contiguous bit stream.
    const int cb = a.code_bytes;
    const int64_t row = ((int64_t)b * a.heads + h);
    uint8_t *kdst = a.k_codes + (row * a.capacity + pos) * cb;
    uint8_t *vdst = a.v_codes + row * a.capacity * cb;
    if (a.bits == 8 || (a.bits == 4 && EPL >= 2)) {
        // 8 bits: byte e is element e; 4 bits: byte i is elements 2i (low nibble) and 2i + 1 --
        // this lane's elements make whole bytes lane*NB .. lane*NB + NB - 1 (NB = EPL*bits/8)
        uint64_t word = 0;
        int nb;
        if (a.bits == 8) {
#pragma unroll
            for (int r = 0; r < EPL; r++) word |= (uint64_t)qc[r] << (8 * r);
            nb = EPL;
        } else {
#pragma unroll
            for (int r = 0; r + 1 < EPL; r += 2) word |= (uint64_t)(qc[r] | (qc[r + 1] << 4)) << (4 * r);
            nb = EPL / 2;
        }
        if (active) {
            if (which == 0) {
                uint8_t *dst = kdst + lane * nb;  // cb = 32 * nb: aligned to nb bytes
                if (nb == 8) *reinterpret_cast<uint64_t *>(dst) = word;
                else if (nb == 4) *reinterpret_cast<uint32_t *>(dst) = (uint32_t)word;
                else if (nb == 2) *reinterpret_cast<uint16_t *>(dst) = (uint16_t)word;
                else *dst = (uint8_t)word;
            } else {
                for (int i = 0; i < nb; i++) vdst[v_byte_offset(pos, lane * nb + i, cb)] = (uint8_t)(word >> (8 * i));
            }
        }
    } else {
        // 3 bits, or 4 bits with one element per lane: the bit stream through shared memory
        if (active)
#pragma unroll
            for (int r = 0; r < EPL; r++) s_codes[lane * EPL + r] = (uint8_t)qc[r];
        __syncwarp();
        for (int j = lane; j < cb; j += 32) {
            uint32_t byte = 0;
#pragma unroll
            for (int bit = 0; bit < 8; bit++) {
                const int g = 8 * j + bit;
                const int e = g / a.bits, eb = g % a.bits;
                if (e < d) byte |= ((uint32_t)(s_codes[e] >> eb) & 1u) << bit;
            }
            if (which == 0) kdst[j] = (uint8_t)byte;
            else vdst[v_byte_offset(pos, j, cb)] = (uint8_t)byte;
        }
    }
    if (lane == 0) {
        float *meta = (which == 0 ? a.k_meta : a.v_meta) + (row * a.capacity + pos) * 2;
        meta[0] = scale;
        meta[1] = zp;
    }

    // QJL residual (CompressedKVCache::write_kv, kv_compression.rs:826-840): the input minus
    // PolarQuantizer::decode of its own codes (:270-286: q * scale + zp, butterfly, * 1/sqrt_approx(n),
    // * sign), then QJLResidualEncoder::encode (:365-395): sign bits and sum|r| / n, the sum taken
    // sequentially in element order.
    uint8_t *qbits = which == 0 ? a.k_qjl_bits : a.v_qjl_bits;
    if (qbits != nullptr) {
        float y[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++)
            y[r] = active ? __fadd_rn(__fmul_rn((float)qc[r], scale), zp) : 0.0f;
        warp_wht_butterfly<EPL>(y, lane, d);
        uint32_t pos_bits[EPL];  // bit l: element l * EPL + r of the residual is >= 0
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const float sgn = sg[r];
            y[r] = __fsub_rn(x0[r], __fmul_rn(__fmul_rn(y[r], a.wht_scale), sgn));
            pos_bits[r] = __ballot_sync(0xffffffffu, active && y[r] >= 0.0f);
        }
        const int64_t vec = row * a.capacity + pos;
        if (lane < d / 8) {
            // byte `lane` holds elements 8 * lane + i, i = 0..7; EPL divides 8
            uint32_t byte = 0;
#pragma unroll
            for (int i = 0; i < 8; i++)
                byte |= ((pos_bits[i % EPL] >> (8 * lane / EPL + i / EPL)) & 1u) << i;
            qbits[vec * (d / 8) + lane] = (uint8_t)byte;
        }
        float msum = 0.0f;
        for (int l = 0; l < d / EPL; l++) {
            if (lane == l) {
#pragma unroll
                for (int r = 0; r < EPL; r++) msum = __fadd_rn(msum, fabsf(y[r]));
            }
            msum = __shfl_sync(0xffffffffu, msum, l);
        }
        if (lane == 0) (which == 0 ? a.k_qjl_mag : a.v_qjl_mag)[vec] = __fdiv_rn(msum, (float)d);
    }
    __syncwarp();
}

}  // namespace sa

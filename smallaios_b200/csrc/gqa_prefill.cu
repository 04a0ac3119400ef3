// GroupQueryAttention of a prefill chunk (many query tokens per sequence) over
// the PolarQuant cache, on tensor cores (mma.m16n8k16, fp16 operands, f32
// accumulation), flash-attention style in the rotated domain:
//
//   q . k_hat = q' . (c*scale + zp),   sum_t p_t v_hat_t = S.H.(sum_t p_t (c_t*scale_t + zp_t))/sqrt(n)
//
// with q' = H.S.RoPE(q)/sqrt(n) (the identity the decode kernels use;
// PolarQuantizer::decode, kv_compression.rs:270-286).  One CTA (8 warps)
// takes 128 query rows -- 128/G positions times the G query heads of one KV
// head -- and walks the causal range of the cache in tiles of 64 tokens:
//   - the K tile is dequantized to fp16 k' = c*scale + zp into shared memory
//     (row per token), the V tile likewise but transposed (row per dimension);
//   - S = Q'.K'^T (16 rows x 64 tokens per warp), the causal mask, an online
//     softmax in base 2 (the attention scale and log2 e are folded into q');
//   - O' += P.V' with P re-used from the score accumulators as the A operand.
// At the end O'/L is rotated back (one warp butterfly per row) and stored.
// Causal semantics as scaled_dot_product_attention with past_sk = T - S
// (ops/microsoft.rs:380-438): query i attends tokens [0, pos0 + i].
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kPfWarps = 8;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfTok = 64;              // tokens per KV tile

template <int D>
struct PfGeo {
    static constexpr int QS = D + 8;           // fp16 per Q' / K' row (bank offset)
    static constexpr int VS = kPfTok + 8;      // fp16 per V'^T row
    static constexpr int Q_BYTES = kPfRows * QS * 2;
    static constexpr int K_BYTES = kPfTok * QS * 2;
    static constexpr int V_BYTES = D * VS * 2;
    static constexpr int META_BYTES = 2 * kPfTok * 8;
    static constexpr int O_BYTES = kPfRows * D * 4;  // f32 staging of O' (reuses Q/K/V)
    static constexpr int MAIN = Q_BYTES + K_BYTES + V_BYTES + META_BYTES;
    static constexpr int SMEM = MAIN > O_BYTES ? MAIN : O_BYTES;
    static constexpr int NKS = D / 16;  // k-steps of Q'.K'^T
    static constexpr int NTO = D / 8;   // n-tiles of O'
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// grid = (ceil(seq_len * G / 128), kv heads, batch), 256 threads.
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(32 * kPfWarps, 2) prefill_attend_kernel(AttendArgs a) {
    using GG = PfGeo<D>;
    constexpr int EPL = D / 32;
    constexpr int CB = D * BITS / 8;
    extern __shared__ __align__(16) unsigned char smem[];
    __half *qs = reinterpret_cast<__half *>(smem);
    __half *ks = reinterpret_cast<__half *>(smem + GG::Q_BYTES);
    __half *vt = reinterpret_cast<__half *>(smem + GG::Q_BYTES + GG::K_BYTES);
    float2 *kms = reinterpret_cast<float2 *>(smem + GG::Q_BYTES + GG::K_BYTES + GG::V_BYTES);
    float2 *vms = kms + kPfTok;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int G = a.group, h = blockIdx.y, b = blockIdx.z;
    const int r0 = blockIdx.x * kPfRows;  // first query row (row = position * G + head)
    const int nrows = a.seq_len * G;
    const int64_t unit = (int64_t)b * a.heads + h;
    const float *sg = a.signs + (int64_t)h * D;

    // ---- q' of this warp's 16 rows: RoPE, signs, WHT, * scale * log2 e / sqrt(n), to fp16 ----
    const float qmul = a.wht_scale * a.scale * 1.4426950408889634f;
    for (int i = 0; i < 16; i++) {
        const int row = warp * 16 + i, gr = r0 + row;
        float x[EPL];
        if (gr < nrows) {
            const int s = gr / G, hd = gr % G;
            const T *src = static_cast<const T *>(a.query) +
                           (((int64_t)b * a.seq_len + s) * (a.heads * G) + h * G + hd) * D;
            const int64_t pos = a.pos0 + s;
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                const int e = lane * EPL + r;
                x[r] = ld_f32(src + e);
                if (a.do_rotary) {
                    const int half = D / 2;
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
                    const float c = a.cos_cache[pos * half + pair], sn = a.sin_cache[pos * half + pair];
                    const float xo = ld_f32(src + partner);
                    x[r] = first ? __fsub_rn(__fmul_rn(c, x[r]), __fmul_rn(sn, xo))
                                 : __fadd_rn(__fmul_rn(sn, xo), __fmul_rn(c, x[r]));
                }
                x[r] *= sg[e];
            }
        } else {
#pragma unroll
            for (int r = 0; r < EPL; r++) x[r] = 0.0f;
        }
        warp_wht_butterfly<EPL>(x, lane, D);
#pragma unroll
        for (int r = 0; r < EPL; r++) qs[row * GG::QS + lane * EPL + r] = __float2half_rn(x[r] * qmul);
    }

    // this lane's two rows g and g + 8: their positions (a padding row takes the last position)
    int pos_r[2];
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        int gr = r0 + warp * 16 + g + 8 * hf;
        if (gr >= nrows) gr = nrows - 1;
        pos_r[hf] = (int)a.pos0 + gr / G;
    }
    const int last_row = min(r0 + kPfRows, nrows) - 1;
    const int pos_last = (int)a.pos0 + last_row / G;  // the CTA's largest position
    const int ntiles = pos_last / kPfTok + 1;

    float oacc[GG::NTO][4];
#pragma unroll
    for (int n = 0; n < GG::NTO; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.0f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};

    const uint8_t *kc = a.k_codes + unit * a.capacity * (int64_t)CB;
    const uint8_t *vc = a.v_codes + unit * a.capacity * (int64_t)CB;
    const float2 *kmeta = reinterpret_cast<const float2 *>(a.k_meta) + unit * a.capacity;
    const float2 *vmeta = reinterpret_cast<const float2 *>(a.v_meta) + unit * a.capacity;

    for (int kt = 0; kt < ntiles; kt++) {
        const int t0 = kt * kPfTok;
        __syncthreads();  // the previous tile's K'/V' are no longer read (and q' is complete)
        if (tid < kPfTok) kms[tid] = kmeta[t0 + tid];
        else if (tid < 2 * kPfTok) vms[tid - kPfTok] = vmeta[t0 + tid - kPfTok];
        __syncthreads();
        // K tile: token rows of CB code bytes, 16 bytes per uint4
        for (int u = tid; u < kPfTok * CB / 16; u += 32 * kPfWarps) {
            const int tok = u / (CB / 16), ch = u % (CB / 16);
            const uint4 w = *reinterpret_cast<const uint4 *>(kc + (int64_t)(t0 + tok) * CB + 16 * ch);
            const float2 m = kms[tok];
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
            __half *dst = ks + tok * GG::QS;
            if constexpr (BITS == 8) {
#pragma unroll
                for (int q = 0; q < 4; q++)
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {
                        const float c0 = (float)((wv[q] >> (8 * e)) & 0xffu), c1 = (float)((wv[q] >> (8 * e + 8)) & 0xffu);
                        *reinterpret_cast<uint32_t *>(dst + 16 * ch + 4 * q + e) =
                            pack_h2(fmaf(c0, m.x, m.y), fmaf(c1, m.x, m.y));
                    }
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++)
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const float c0 = (float)((wv[q] >> (4 * e)) & 0xfu), c1 = (float)((wv[q] >> (4 * e + 4)) & 0xfu);
                        *reinterpret_cast<uint32_t *>(dst + 32 * ch + 8 * q + e) =
                            pack_h2(fmaf(c0, m.x, m.y), fmaf(c1, m.x, m.y));
                    }
            }
        }
        // V tile: four 16-token blocks of 16*CB contiguous bytes; a uint4 is chunk c of token
        // group gq of a block: bytes k = 4j + (token & 3) for j = 4c .. 4c+3
        const uint8_t *vtile = vc + (int64_t)(t0 / 16) * 16 * CB;
        for (int u = tid; u < kPfTok * CB / 16; u += 32 * kPfWarps) {
            const int blk = u / CB, rem = u % CB, c = rem / 4, gq = rem % 4;
            const uint4 w = *reinterpret_cast<const uint4 *>(vtile + (int64_t)blk * 16 * CB + 64 * c + 16 * gq);
            const int tok0 = blk * 16 + 4 * gq;  // tokens tok0 .. tok0 + 3 of the tile
            const float2 m0 = vms[tok0], m1 = vms[tok0 + 1], m2 = vms[tok0 + 2], m3 = vms[tok0 + 3];
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};  // word jj: byte j = 4c + jj, tokens 0..3
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t x = wv[jj];
                if constexpr (BITS == 8) {
                    const int dim = 4 * c + jj;
                    const float c0 = (float)(x & 0xffu), c1 = (float)((x >> 8) & 0xffu);
                    const float c2 = (float)((x >> 16) & 0xffu), c3 = (float)(x >> 24);
                    uint2 o;
                    o.x = pack_h2(fmaf(c0, m0.x, m0.y), fmaf(c1, m1.x, m1.y));
                    o.y = pack_h2(fmaf(c2, m2.x, m2.y), fmaf(c3, m3.x, m3.y));
                    *reinterpret_cast<uint2 *>(vt + dim * GG::VS + tok0) = o;
                } else {
#pragma unroll
                    for (int hi = 0; hi < 2; hi++) {
                        const int dim = 2 * (4 * c + jj) + hi;
                        const int sh = 4 * hi;
                        const float c0 = (float)((x >> sh) & 0xfu), c1 = (float)((x >> (8 + sh)) & 0xfu);
                        const float c2 = (float)((x >> (16 + sh)) & 0xfu), c3 = (float)((x >> (24 + sh)) & 0xfu);
                        uint2 o;
                        o.x = pack_h2(fmaf(c0, m0.x, m0.y), fmaf(c1, m1.x, m1.y));
                        o.y = pack_h2(fmaf(c2, m2.x, m2.y), fmaf(c3, m3.x, m3.y));
                        *reinterpret_cast<uint2 *>(vt + dim * GG::VS + tok0) = o;
                    }
                }
            }
        }
        __syncthreads();

        // ---- S = Q'.K'^T: rows warp*16 + (g, g+8), tokens 8j + (2t, 2t+1) ----
        float sacc[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
        const __half *qrow = qs + (warp * 16 + g) * GG::QS;
#pragma unroll
        for (int kk = 0; kk < GG::NKS; kk++) {
            const int c0 = 16 * kk + 2 * t;
            const uint32_t a0 = *reinterpret_cast<const uint32_t *>(qrow + c0);
            const uint32_t a1 = *reinterpret_cast<const uint32_t *>(qrow + 8 * GG::QS + c0);
            const uint32_t a2 = *reinterpret_cast<const uint32_t *>(qrow + c0 + 8);
            const uint32_t a3 = *reinterpret_cast<const uint32_t *>(qrow + 8 * GG::QS + c0 + 8);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const __half *krow = ks + (8 * j + g) * GG::QS + c0;
                mma_f16(sacc[j], a0, a1, a2, a3, *reinterpret_cast<const uint32_t *>(krow),
                        *reinterpret_cast<const uint32_t *>(krow + 8));
            }
        }
        // ---- causal mask, online softmax (base 2) ----
        float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int hf = e >> 1, tok = t0 + 8 * j + 2 * t + (e & 1);
                if (tok > pos_r[hf]) sacc[j][e] = -INFINITY;
                mx[hf] = fmaxf(mx[hf], sacc[j][e]);
            }
        float fac[2], rs[2] = {0.0f, 0.0f};
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 1));
            mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 2));
            fac[hf] = exp2f(m_r[hf] - mx[hf]);  // 0 on the first tile (m = -inf)
            m_r[hf] = mx[hf];
        }
        uint32_t pa[8][2];  // P as fp16 pairs: [n-tile][row g / row g+8]
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float p0 = exp2f(sacc[j][0] - mx[0]), p1 = exp2f(sacc[j][1] - mx[0]);
            const float p2 = exp2f(sacc[j][2] - mx[1]), p3 = exp2f(sacc[j][3] - mx[1]);
            rs[0] += p0 + p1;
            rs[1] += p2 + p3;
            pa[j][0] = pack_h2(p0, p1);
            pa[j][1] = pack_h2(p2, p3);
        }
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            rs[hf] += __shfl_xor_sync(0xffffffffu, rs[hf], 1);
            rs[hf] += __shfl_xor_sync(0xffffffffu, rs[hf], 2);
            l_r[hf] = fmaf(l_r[hf], fac[hf], rs[hf]);
        }
#pragma unroll
        for (int n = 0; n < GG::NTO; n++) {
            oacc[n][0] *= fac[0];
            oacc[n][1] *= fac[0];
            oacc[n][2] *= fac[1];
            oacc[n][3] *= fac[1];
        }
        // ---- O' += P.V' ----
#pragma unroll
        for (int kk = 0; kk < kPfTok / 16; kk++) {
            const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
            for (int n = 0; n < GG::NTO; n++) {
                const __half *vrow = vt + (8 * n + g) * GG::VS + 16 * kk + 2 * t;
                mma_f16(oacc[n], a0, a1, a2, a3, *reinterpret_cast<const uint32_t *>(vrow),
                        *reinterpret_cast<const uint32_t *>(vrow + 8));
            }
        }
    }

    // ---- O'/L to shared memory, then rotate back and store, one row per warp pass ----
    __syncthreads();  // the tiles are no longer read
    float *os = reinterpret_cast<float *>(smem) + warp * 16 * D;
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        const float inv = l_r[hf] > 0.0f ? 1.0f / l_r[hf] : 0.0f;
#pragma unroll
        for (int n = 0; n < GG::NTO; n++) {
            os[(g + 8 * hf) * D + 8 * n + 2 * t] = oacc[n][2 * hf] * inv;
            os[(g + 8 * hf) * D + 8 * n + 2 * t + 1] = oacc[n][2 * hf + 1] * inv;
        }
    }
    __syncwarp();
    for (int i = 0; i < 16; i++) {
        const int gr = r0 + warp * 16 + i;
        if (gr >= nrows) break;
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) x[r] = os[i * D + lane * EPL + r];
        warp_wht_butterfly<EPL>(x, lane, D);
        const int s = gr / G, hd = gr % G;
        T *dst = static_cast<T *>(a.out) + (((int64_t)b * a.seq_len + s) * (a.heads * G) + h * G + hd) * D;
#pragma unroll
        for (int r = 0; r < EPL; r++)
            st_from_f32(dst + lane * EPL + r, x[r] * a.wht_scale * sg[lane * EPL + r]);
    }
}

template <typename T, int BITS, int D>
int launch_shape(const AttendArgs &a, cudaStream_t stream) {
    using GG = PfGeo<D>;
    auto kern = prefill_attend_kernel<T, BITS, D>;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GG::SMEM);
        if (e != cudaSuccess) return check_cuda(e, "gqa prefill smem attribute");
        if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
    }
    const int rows = a.seq_len * a.group;
    const dim3 grid((unsigned)((rows + kPfRows - 1) / kPfRows), (unsigned)a.heads, (unsigned)a.batch);
    kern<<<grid, 32 * kPfWarps, GG::SMEM, stream>>>(a);
    count_launch();
    return check_cuda(cudaGetLastError(), "gqa prefill launch");
}

template <typename T>
int launch_dtype(const AttendArgs &a, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch_shape<T, 4, 128>(a, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch_shape<T, 8, 128>(a, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch_shape<T, 4, 64>(a, stream);
    return launch_shape<T, 8, 64>(a, stream);
}

}  // namespace

// Tensor-core prefill: chunks of 16 or more query tokens, 4/8-bit codes,
// head_dim 64/128, group 1..8, output to attn_out (no head-sharded gather).
bool prefill_eligible(const AttendArgs &a) {
    if (a.seq_len < 16 || a.group < 1 || a.group > 8 || a.gather.n != 0) return false;
    if ((a.bits != 4 && a.bits != 8) || (a.head_dim != 64 && a.head_dim != 128)) return false;
    if (a.capacity % kPfTok != 0) return false;
    return (int64_t)a.seq_len * a.group <= ((int64_t)1 << 30) && a.pos0 + a.seq_len <= ((int64_t)1 << 30);
}

int launch_gqa_prefill(const AttendArgs &a, cudaStream_t stream) {
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_dtype<float>(a, stream);
        case SA_DTYPE_FLOAT16: return launch_dtype<__half>(a, stream);
        default: return launch_dtype<__nv_bfloat16>(a, stream);
    }
}

}  // namespace sa

// GroupQueryAttention of a prefill chunk (many query tokens per sequence) over
// the PolarQuant cache, on tensor cores (mma.m16n8k16, fp16 operands, f32
// accumulation), flash-attention style in the rotated domain, with the codes
// themselves as the K and V operands (small integers are exact in fp16):
//
//   q . k_hat = scale_t * (q' . c_t) + zp_t * sum(q')
//   sum_t p_t v_hat_t = S.H.(sum_t (p_t scale_t) c_t + (sum_t p_t zp_t) 1)/sqrt(n)
//
// with q' = H.S.RoPE(q)/sqrt(n) (the identity the decode kernels use;
// PolarQuantizer::decode, kv_compression.rs:270-286).  q' and p_t scale_t are
// each split into two fp16 halves (hi + lo), so every product is exact to
// about 2^-22 of its value and the rest of the arithmetic is f32.  One CTA
// (8 warps) takes 128 query rows -- 128/G positions times the G query heads of
// one KV head -- and walks the causal range of the cache in tiles of 64 tokens:
//   - the K codes of a tile go to shared memory as fp16 integers (row per
//     token), the V codes likewise but transposed (row per dimension);
//   - S = (Q'hi + Q'lo).C^T (16 rows x 64 tokens per warp), then scale and
//     zero point per token in f32, the causal mask, an online softmax in base 2
//     (the attention scale and log2 e are folded into q');
//   - O' += U.C with u_t = 2^(s_t - R) scale_t <= 1 (R >= the running max plus
//     log2 of the largest V scale seen, the decode kernels' reference), and the
//     zero-point sum kept per row in f32.
// At the end O' = (O'_u 2^(R - m) + Z)/L is rotated back (one warp butterfly
// per row) and stored.  Causal semantics as scaled_dot_product_attention with
// past_sk = T - S (ops/microsoft.rs:380-438): query i attends tokens
// [0, pos0 + i].
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kPfWarps = 8;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfTok = 64;              // tokens per KV tile
constexpr int kPfSub = 32;              // tokens per softmax step within a tile

template <int D>
struct PfGeo {
    static constexpr int QS = D + 8;       // fp16 per Q' / code row (bank offset)
    static constexpr int VS = kPfTok + 8;  // fp16 per transposed V code row
    static constexpr int Q_BYTES = kPfRows * QS * 2;  // one of the two q' planes
    static constexpr int K_BYTES = kPfTok * QS * 2;
    static constexpr int V_BYTES = D * VS * 2;
    static constexpr int META_BYTES = kPfTok * 16;  // {k scale, k zp, v scale, v zp} per token
    static constexpr int QSUM_BYTES = kPfRows * 4;
    static constexpr int K_OFF = 2 * Q_BYTES;
    static constexpr int V_OFF = K_OFF + K_BYTES;
    static constexpr int META_OFF = V_OFF + V_BYTES;
    static constexpr int QSUM_OFF = META_OFF + META_BYTES;
    static constexpr int OS = D + 8;                  // f32 per staged O' row (rows g, g+8 on distinct banks)
    static constexpr int O_BYTES = kPfRows * OS * 4;  // f32 staging of O' (reuses the q' planes)
    static constexpr int SMEM = QSUM_OFF + QSUM_BYTES;
    static_assert(O_BYTES <= K_OFF, "O' staging overlaps the code tiles");
    static constexpr int NKS = D / 16;  // k-steps of Q'.C^T
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

// (lo, hi) -> fp16 pairs h = rn(x) and l = rn(x - h), so that h + l = x to about 2^-22 |x|
__device__ __forceinline__ void split_h2(float lo, float hi, uint32_t &h, uint32_t &l) {
    const __half2 hh = __floats2half2_rn(lo, hi);
    const float2 back = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(lo - back.x, hi - back.y);
    h = *reinterpret_cast<const uint32_t *>(&hh);
    l = *reinterpret_cast<const uint32_t *>(&ll);
}

// bytes b0, b1 of x (selected by sel) -> fp16 pair (b0, b1): 0x64XX is the fp16 1024 + XX
__device__ __forceinline__ uint32_t bytes_to_h2(uint32_t x, uint32_t sel) {
    const uint32_t biased = __byte_perm(x, 0x64646464u, sel);
    const __half2 v = __hsub2(*reinterpret_cast<const __half2 *>(&biased), __float2half2_rn(1024.0f));
    return *reinterpret_cast<const uint32_t *>(&v);
}

// grid = ceil(seq_len * G / 128) * kv heads * batch blocks (1-D), 256 threads.
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(32 * kPfWarps, 2) prefill_attend_kernel(AttendArgs a) {
    using GG = PfGeo<D>;
    constexpr int EPL = D / 32;
    constexpr int CB = D * BITS / 8;
    extern __shared__ __align__(16) unsigned char smem[];
    __half *qhs = reinterpret_cast<__half *>(smem);
    __half *qls = reinterpret_cast<__half *>(smem + GG::Q_BYTES);
    __half *ks = reinterpret_cast<__half *>(smem + GG::K_OFF);
    __half *vt = reinterpret_cast<__half *>(smem + GG::V_OFF);
    float4 *meta = reinterpret_cast<float4 *>(smem + GG::META_OFF);
    float *qsum = reinterpret_cast<float *>(smem + GG::QSUM_OFF);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    // one block per (row block, KV head, batch row), row blocks slowest and in reverse: the last
    // row blocks walk the most tiles, so they take the lowest block indices and start first
    const int units = a.heads * a.batch;
    const int rblocks = (int)(gridDim.x / (unsigned)units);
    const int h = (int)(blockIdx.x % (unsigned)a.heads), b = (int)(blockIdx.x / (unsigned)a.heads) % a.batch;
    const int G = a.group;
    const int r0 = (rblocks - 1 - (int)(blockIdx.x / (unsigned)units)) * kPfRows;  // row = position * G + head
    const int nrows = a.seq_len * G;
    const int64_t unit = (int64_t)b * a.heads + h;
    const float *sg = a.signs + (int64_t)h * D;

    // ---- q' of this warp's 16 rows: RoPE, signs, WHT, * scale * log2 e / sqrt(n), as hi + lo fp16 ----
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
        float sum = 0.0f;
#pragma unroll
        for (int r = 0; r < EPL; r += 2) {
            const float x0 = x[r] * qmul, x1 = x[r + 1] * qmul;
            sum += x0 + x1;
            uint32_t hi, lo;
            split_h2(x0, x1, hi, lo);
            *reinterpret_cast<uint32_t *>(qhs + row * GG::QS + lane * EPL + r) = hi;
            *reinterpret_cast<uint32_t *>(qls + row * GG::QS + lane * EPL + r) = lo;
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
        if (lane == 0) qsum[row] = sum;
    }
    __syncwarp();

    // this lane's two rows g and g + 8: positions (a padding row takes the last position) and sum(q')
    int pos_r[2];
    float qs_r[2];
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        int gr = r0 + warp * 16 + g + 8 * hf;
        qs_r[hf] = qsum[warp * 16 + g + 8 * hf];
        if (gr >= nrows) gr = nrows - 1;
        pos_r[hf] = (int)a.pos0 + gr / G;
    }
    const int last_row = min(r0 + kPfRows, nrows) - 1;
    const int pos_last = (int)a.pos0 + last_row / G;  // the CTA's largest position
    const int ntiles = pos_last / kPfTok + 1;
    const int pos_wmax = (int)a.pos0 + (min(r0 + warp * 16 + 15, nrows - 1)) / G;  // this warp's largest position

    float oacc[GG::NTO][4];
#pragma unroll
    for (int n = 0; n < GG::NTO; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.0f;
    // running max m, the V reference R, and this lane's partial sums of p and p * zp (per row)
    float m_r[2] = {-INFINITY, -INFINITY}, R_r[2] = {-INFINITY, -INFINITY};
    float l_r[2] = {0.0f, 0.0f}, z_r[2] = {0.0f, 0.0f};

    const uint8_t *kc = a.k_codes + unit * a.capacity * (int64_t)CB;
    const uint8_t *vc = a.v_codes + unit * a.capacity * (int64_t)CB;
    const float2 *kmeta = reinterpret_cast<const float2 *>(a.k_meta) + unit * a.capacity;
    const float2 *vmeta = reinterpret_cast<const float2 *>(a.v_meta) + unit * a.capacity;

    for (int kt = 0; kt < ntiles; kt++) {
        const int t0 = kt * kPfTok;
        __syncthreads();  // the previous tile is no longer read (and q' is complete)
        if (tid < kPfTok) {
            // tokens past every row's position are masked; zero their (possibly unwritten) metadata
            float4 m4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (t0 + tid <= pos_last) {
                const float2 km = kmeta[t0 + tid], vm = vmeta[t0 + tid];
                m4 = make_float4(km.x, km.y, vm.x, vm.y);
            }
            meta[tid] = m4;
        }
        // K tile: token rows of CB code bytes, 16 bytes per uint4
        for (int u = tid; u < kPfTok * CB / 16; u += 32 * kPfWarps) {
            const int tok = u / (CB / 16), ch = u % (CB / 16);
            const uint4 w = *reinterpret_cast<const uint4 *>(kc + (int64_t)(t0 + tok) * CB + 16 * ch);
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
            __half *dst = ks + tok * GG::QS;
            if constexpr (BITS == 8) {
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    uint2 o;
                    o.x = bytes_to_h2(wv[q], 0x4140u);
                    o.y = bytes_to_h2(wv[q], 0x4342u);
                    *reinterpret_cast<uint2 *>(dst + 16 * ch + 4 * q) = o;
                }
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    // byte i holds dimensions 2i (low nibble) and 2i + 1 (high nibble)
                    const uint32_t lo = wv[q] & 0x0f0f0f0fu, hi = (wv[q] >> 4) & 0x0f0f0f0fu;
                    const uint32_t d03 = __byte_perm(lo, hi, 0x5140u), d47 = __byte_perm(lo, hi, 0x7362u);
                    uint4 o;
                    o.x = bytes_to_h2(d03, 0x4140u);
                    o.y = bytes_to_h2(d03, 0x4342u);
                    o.z = bytes_to_h2(d47, 0x4140u);
                    o.w = bytes_to_h2(d47, 0x4342u);
                    *reinterpret_cast<uint4 *>(dst + 32 * ch + 8 * q) = o;
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
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};  // word jj: byte j = 4c + jj, tokens 0..3
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t x = wv[jj];
                if constexpr (BITS == 8) {
                    const int dim = 4 * c + jj;
                    uint2 o;
                    o.x = bytes_to_h2(x, 0x4140u);
                    o.y = bytes_to_h2(x, 0x4342u);
                    *reinterpret_cast<uint2 *>(vt + dim * GG::VS + tok0) = o;
                } else {
#pragma unroll
                    for (int hi = 0; hi < 2; hi++) {
                        const int dim = 2 * (4 * c + jj) + hi;
                        const uint32_t nib = (x >> (4 * hi)) & 0x0f0f0f0fu;
                        uint2 o;
                        o.x = bytes_to_h2(nib, 0x4140u);
                        o.y = bytes_to_h2(nib, 0x4342u);
                        *reinterpret_cast<uint2 *>(vt + dim * GG::VS + tok0) = o;
                    }
                }
            }
        }
        __syncthreads();

        // the tile's largest V scale (metadata of masked tokens is zero)
        float vmax = fmaxf(meta[lane].z, meta[lane + 32].z);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, m));
        const float lvmax = __log2f(fmaxf(vmax, 1.17549435e-38f));

        // two halves of 32 tokens (fewer live score registers); a half past every row of this
        // warp is skipped
#pragma unroll 1
        for (int th = 0; th < kPfTok; th += kPfSub) {
            if (t0 + th > pos_wmax) break;
            // ---- S = (Q'hi + Q'lo).C^T: rows warp*16 + (g, g+8), tokens th + 8j + (2t, 2t+1) ----
            float sacc[kPfSub / 8][4];
#pragma unroll
            for (int j = 0; j < kPfSub / 8; j++) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
            const __half *qh = qhs + (warp * 16 + g) * GG::QS;
            const __half *ql = qls + (warp * 16 + g) * GG::QS;
#pragma unroll
            for (int kk = 0; kk < GG::NKS; kk++) {
                const int c0 = 16 * kk + 2 * t;
                const uint32_t a0 = *reinterpret_cast<const uint32_t *>(qh + c0);
                const uint32_t a1 = *reinterpret_cast<const uint32_t *>(qh + 8 * GG::QS + c0);
                const uint32_t a2 = *reinterpret_cast<const uint32_t *>(qh + c0 + 8);
                const uint32_t a3 = *reinterpret_cast<const uint32_t *>(qh + 8 * GG::QS + c0 + 8);
                const uint32_t e0 = *reinterpret_cast<const uint32_t *>(ql + c0);
                const uint32_t e1 = *reinterpret_cast<const uint32_t *>(ql + 8 * GG::QS + c0);
                const uint32_t e2 = *reinterpret_cast<const uint32_t *>(ql + c0 + 8);
                const uint32_t e3 = *reinterpret_cast<const uint32_t *>(ql + 8 * GG::QS + c0 + 8);
                uint32_t bk[kPfSub / 8][2];
#pragma unroll
                for (int j = 0; j < kPfSub / 8; j++) {
                    const __half *krow = ks + (th + 8 * j + g) * GG::QS + c0;
                    bk[j][0] = *reinterpret_cast<const uint32_t *>(krow);
                    bk[j][1] = *reinterpret_cast<const uint32_t *>(krow + 8);
                }
                // all hi products, then all lo products: no MMA waits on the one before it
#pragma unroll
                for (int j = 0; j < kPfSub / 8; j++) mma_f16(sacc[j], a0, a1, a2, a3, bk[j][0], bk[j][1]);
#pragma unroll
                for (int j = 0; j < kPfSub / 8; j++) mma_f16(sacc[j], e0, e1, e2, e3, bk[j][0], bk[j][1]);
            }
            // ---- scale / zero point per token, causal mask, running max ----
            float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
            for (int j = 0; j < kPfSub / 8; j++)
#pragma unroll
                for (int ee = 0; ee < 2; ee++) {
                    const int tok = th + 8 * j + 2 * t + ee;
                    const float2 km = *reinterpret_cast<const float2 *>(&meta[tok]);
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        float s = fmaf(sacc[j][2 * hf + ee], km.x, km.y * qs_r[hf]);
                        if (t0 + tok > pos_r[hf]) s = -INFINITY;
                        sacc[j][2 * hf + ee] = s;
                        mx[hf] = fmaxf(mx[hf], s);
                    }
                }
            float kr[2];
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 1));
                mx[hf] = fmaxf(mx[hf], __shfl_xor_sync(0xffffffffu, mx[hf], 2));
                const float fac = exp2f(m_r[hf] - mx[hf]);  // 0 on the first half-tile (m = -inf)
                l_r[hf] *= fac;
                z_r[hf] *= fac;
                m_r[hf] = mx[hf];
                const float rn = fmaxf(R_r[hf], mx[hf] + lvmax);
                const float ofac = exp2f(R_r[hf] - rn);
                R_r[hf] = rn;
                kr[hf] = exp2f(mx[hf] - rn);  // p * vscale * kr <= 1
#pragma unroll
                for (int n = 0; n < GG::NTO; n++) {
                    oacc[n][2 * hf] *= ofac;
                    oacc[n][2 * hf + 1] *= ofac;
                }
            }
            // ---- P, U = P * vscale * kr as hi + lo fp16, O'_u += U.C ----
#pragma unroll
            for (int kk = 0; kk < kPfSub / 16; kk++) {
                uint32_t ah[4], al[4];  // A fragments: (row g, j = 2kk), (row g+8, 2kk), (g, 2kk+1), (g+8, 2kk+1)
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    const int j = 2 * kk + jj;
                    const float2 m0 = *reinterpret_cast<const float2 *>(&meta[th + 8 * j + 2 * t].z);
                    const float2 m1 = *reinterpret_cast<const float2 *>(&meta[th + 8 * j + 2 * t + 1].z);
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        const float p0 = exp2f(sacc[j][2 * hf] - m_r[hf]);
                        const float p1 = exp2f(sacc[j][2 * hf + 1] - m_r[hf]);
                        l_r[hf] += p0 + p1;
                        z_r[hf] = fmaf(p0, m0.y, fmaf(p1, m1.y, z_r[hf]));
                        split_h2(p0 * m0.x * kr[hf], p1 * m1.x * kr[hf], ah[2 * jj + hf], al[2 * jj + hf]);
                    }
                }
                // groups of 4 n-tiles: hi products, then lo products
#pragma unroll
                for (int n0 = 0; n0 < GG::NTO; n0 += 4) {
                    uint32_t bv[4][2];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const __half *vrow = vt + (8 * (n0 + i) + g) * GG::VS + th + 16 * kk + 2 * t;
                        bv[i][0] = *reinterpret_cast<const uint32_t *>(vrow);
                        bv[i][1] = *reinterpret_cast<const uint32_t *>(vrow + 8);
                    }
#pragma unroll
                    for (int i = 0; i < 4; i++) mma_f16(oacc[n0 + i], ah[0], ah[1], ah[2], ah[3], bv[i][0], bv[i][1]);
#pragma unroll
                    for (int i = 0; i < 4; i++) mma_f16(oacc[n0 + i], al[0], al[1], al[2], al[3], bv[i][0], bv[i][1]);
                }
            }
        }
    }

    // ---- O' = (O'_u 2^(R - m) + Z)/L to shared memory, then rotate back and store ----
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
#pragma unroll
        for (int m = 1; m <= 2; m <<= 1) {
            l_r[hf] += __shfl_xor_sync(0xffffffffu, l_r[hf], m);
            z_r[hf] += __shfl_xor_sync(0xffffffffu, z_r[hf], m);
        }
    }
    __syncthreads();  // the tiles and q' planes are no longer read
    float *os = reinterpret_cast<float *>(smem) + warp * 16 * GG::OS;
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        const float inv = l_r[hf] > 0.0f ? 1.0f / l_r[hf] : 0.0f;
        const float cu = exp2f(R_r[hf] - m_r[hf]) * inv, cz = z_r[hf] * inv;
#pragma unroll
        for (int n = 0; n < GG::NTO; n++) {
            *reinterpret_cast<float2 *>(&os[(g + 8 * hf) * GG::OS + 8 * n + 2 * t]) =
                make_float2(fmaf(oacc[n][2 * hf], cu, cz), fmaf(oacc[n][2 * hf + 1], cu, cz));
        }
    }
    __syncwarp();
    for (int i = 0; i < 16; i++) {
        const int gr = r0 + warp * 16 + i;
        if (gr >= nrows) break;
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) x[r] = os[i * GG::OS + lane * EPL + r];
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
    const int64_t nblocks = (int64_t)((rows + kPfRows - 1) / kPfRows) * a.heads * a.batch;
    if (nblocks > 0x7fffffff) return set_error(SA_ERR_UNSUPPORTED, "gqa prefill: %lld blocks", (long long)nblocks);
    const dim3 grid((unsigned)nblocks);
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

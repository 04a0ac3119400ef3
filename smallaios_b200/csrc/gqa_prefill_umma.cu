// GroupQueryAttention of a prefill chunk (16 or more query tokens per
// sequence) on the 5th-generation tensor cores (tcgen05), flash-attention
// style in the rotated domain, with the codes themselves as the K and V
// operands (integers below 256 are exact in fp16):
//
//   q . k_hat = scale_t * (q' . c_t) + zp_t * sum(q')
//   sum_t p_t v_hat_t = S.H.(sum_t u_t c_t * 2^(R-m) + (sum_t p_t zp_t) 1)/sqrt(n)
//
// with q' = H.S.RoPE(q)/sqrt(n) (PolarQuantizer::decode, kv_compression.rs:
// 270-286, read backwards) and u_t = p_t * scale_t * 2^(m-R).  q' and u are
// each split into two fp16 halves (hi + lo), so the products are exact to
// about 2^-22 and everything else is f32.
//
// One CTA of 8 warps takes 128 query rows -- 128/G positions times the G query
// heads of one KV head -- as the MMA's M = 128 (one TMEM lane per row), and
// walks the causal range of the cache in tiles of 64 tokens:
//   warps 4-7  stage the tiles: K and V codes as fp16 into shared memory in the
//              128-byte-swizzle K-major layout the MMA reads (K once S(kt-1)
//              has read the previous one, V once PV(kt-1) has), and the tile's
//              {k scale, k zp, v scale, v zp}; the next tile's codes are loaded
//              into registers while the softmax runs;
//   warp 4     one elected lane issues, once the softmax of tile kt-1 has
//              written U, O += (Uhi + Ulo).C_V of kt-1 (A from TMEM, N = D) and
//              then S = (Q'hi + Q'lo).C_K^T of kt (A and B from shared memory,
//              D = f32 in TMEM, N = 64);
//   warps 0-3  one thread per row: tcgen05.ld of its 64 scores, per-token
//              scale / zero point, causal mask, online softmax in base 2, U
//              into TMEM (tcgen05.st).  The V reference R (u <= 2^8) moves
//              only when the row's maximum outgrows it by 8 octaves; then the
//              thread rescales its row of O in TMEM.
// At the end O' = (O 2^(R-m) + Z)/L goes through shared memory, one warp
// butterfly per row rotates it back, and it is stored.  Causal semantics as
// scaled_dot_product_attention with past_sk = T - S (ops/microsoft.rs:380-438).
//
// Every mbarrier wait is bounded (2 s); a wait that gives up sets the abort
// flag and bit 0 of the cache's status word, every role leaves its loop, the
// issued MMAs are waited for (bounded) and TMEM is freed; the output is then
// not written.
#include <type_traits>

#include "sa_common.cuh"
#include "sa_internal.h"
#include "sa_tcgen05.cuh"

namespace sa {

namespace {

constexpr int kPuRows = 128;  // query rows per CTA: UMMA M, TMEM lanes
constexpr int kPuTok = 64;    // tokens per KV tile: UMMA N of S, K of O += U.C
constexpr int kPuWarps = 8;
constexpr int kPuMmaWarp = 4;
constexpr uint32_t kPuTmemCols = 256;
constexpr uint32_t kPuS = 0, kPuUh = 64, kPuUl = 96, kPuO = 128;  // TMEM columns
constexpr float kPuLazy = 8.0f;  // octaves the V reference may lag the row maximum (u <= 2^8)

template <int D>
struct PuGeo {
    static constexpr int KBLK = D / 64;                // 64-element (128-byte) k-blocks per row
    static constexpr int Q_PLANE = kPuRows * D * 2;    // KBLK tiles of [128 rows][128 B]
    static constexpr int K_BLK = kPuTok * 128;         // one k-block of the K tile: [64 tokens][128 B]
    static constexpr int K_TILE = KBLK * K_BLK;
    static constexpr int V_TILE = D * 128;             // [D dims][64 tokens]
    static constexpr int K_OFF = 2 * Q_PLANE;
    static constexpr int V_OFF = K_OFF + K_TILE;
    // per tile buffer: [32 token pairs] {k scale, k scale, k zp, k zp} then [32] {v scale x2, v zp x2}
    static constexpr int META_OFF = V_OFF + V_TILE;
    static constexpr int QSUM_OFF = META_OFF + 2 * kPuTok * 16;
    static constexpr int BAR_OFF = QSUM_OFF + kPuRows * 4 + 16;  // + the tiles' V-scale maxima [2][2]
    static constexpr int SMEM = BAR_OFF + 64 + 1024;   // + slack to align the base to 1024 B
    static_assert(kPuRows * D * 4 <= K_OFF, "O' staging reuses the q' planes");
};

// (lo, hi) -> fp16 pairs h = rn(x) and l = rn(x - h)
__device__ __forceinline__ void split_h2(float lo, float hi, uint32_t &h, uint32_t &l) {
    const __half2 hh = __floats2half2_rn(lo, hi);
    const float2 back = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(lo - back.x, hi - back.y);
    h = *reinterpret_cast<const uint32_t *>(&hh);
    l = *reinterpret_cast<const uint32_t *>(&ll);
}

// bytes of x picked by sel -> fp16 pair of small integers (0x64XX is the fp16 1024 + XX)
__device__ __forceinline__ uint32_t bytes_to_h2(uint32_t x, uint32_t sel) {
    const uint32_t biased = __byte_perm(x, 0x64646464u, sel);
    const __half2 v = __hsub2(*reinterpret_cast<const __half2 *>(&biased), __float2half2_rn(1024.0f));
    return *reinterpret_cast<const uint32_t *>(&v);
}

// 2^x by the MUFU instruction (ex2.approx.ftz: relative error near 2^-22, subnormal results
// flushed to zero -- weights below 2^-126 of the row maximum)
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// Packed f32x2 arithmetic (fma / mul / add .rn.f32x2): each lane rounded exactly as the scalar
// operation, two per instruction.
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
        "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
        "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
        "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Byte offset of 16-byte chunk c (0..7) of row r in a [rows][128 B] 128-byte-swizzle tile.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Barrier of warps 4-7 (named barrier 1, 128 threads) returning the OR of `v` over them.
__device__ __forceinline__ bool bar_or_4to7(bool v) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbarrier.cta.red.or.pred p, 1, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// Instruction descriptor, kind::f16: D f32, A and B fp16 (K-major), M = 128, N.
__host__ __device__ constexpr uint32_t pu_idesc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kPuRows >> 4) << 24);
}

// grid = ceil(seq_len * G / 128) * kv heads * batch blocks (1-D), 256 threads.
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(32 * kPuWarps, 2) prefill_umma_kernel(AttendArgs a) {
    using GG = PuGeo<D>;
    constexpr int EPL = D / 32;
    constexpr int CB = D * BITS / 8;
    extern __shared__ unsigned char pu_raw[];
    // aligned by pointer arithmetic on the shared array (not through an integer), so that the
    // compiler keeps every access below in the shared address space (LDS/STS, not generic LD/ST)
    unsigned char *smem = pu_raw + ((1024 - (smem_u32(pu_raw) & 1023)) & 1023);
    unsigned char *qh = smem, *ql = smem + GG::Q_PLANE;
    unsigned char *kt_s = smem + GG::K_OFF, *vt_s = smem + GG::V_OFF;
    float4 *meta = reinterpret_cast<float4 *>(smem + GG::META_OFF);
    float *qsum = reinterpret_cast<float *>(smem + GG::QSUM_OFF);
    uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + GG::BAR_OFF);
    uint64_t *bar_u = bar_s + 1, *bar_o = bar_s + 2, *bar_fin = bar_s + 3;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar_s + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bar_s + 5);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int units = a.heads * a.batch;
    const int rblocks = (int)(gridDim.x / (unsigned)units);
    const int h = (int)(blockIdx.x % (unsigned)a.heads), b = (int)(blockIdx.x / (unsigned)a.heads) % a.batch;
    const int G = a.group;
    // the last row blocks walk the most tiles: they take the lowest block indices
    const int r0 = (rblocks - 1 - (int)(blockIdx.x / (unsigned)units)) * kPuRows;  // row = position * G + head
    const int nrows = a.seq_len * G;
    const int64_t unit = (int64_t)b * a.heads + h;
    const float *sg = a.signs + (int64_t)h * D;

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_u, 4);
        mbar_init(bar_o, 1);
        mbar_init(bar_fin, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) tmem_alloc(tslot, kPuTmemCols);

    // ---- q' of 16 rows per warp: RoPE, signs, WHT, * scale * log2 e / sqrt(n), as hi + lo fp16 ----
    const float qmul = a.wht_scale * a.scale * 1.4426950408889634f;
    const float *vtr = a.lr_vtr ? a.lr_vtr + unit * D : nullptr;
    constexpr int RB = 4;  // rows whose global loads are in flight together
    for (int i0 = 0; i0 < kPuRows / kPuWarps; i0 += RB) {
        // loads of RB rows: the elements, their rotary partners and the cos / sin entries
        float xv[RB][EPL], xo[RB][EPL], cv[RB][EPL], sv[RB][EPL];
#pragma unroll
        for (int j = 0; j < RB; j++) {
            const int gr = r0 + warp * (kPuRows / kPuWarps) + i0 + j;
            const bool live = gr < nrows;
            const int s = live ? gr / G : 0, hd = live ? gr % G : 0;
            const T *src = static_cast<const T *>(a.query) +
                           (((int64_t)b * a.seq_len + s) * (a.heads * G) + h * G + hd) * D;
            const int64_t pos = a.pos0 + s;
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                const int e = lane * EPL + r;
                xv[j][r] = live ? ld_f32(src + e) : 0.0f;
                cv[j][r] = 1.0f;
                sv[j][r] = 0.0f;
                xo[j][r] = 0.0f;
                if (a.do_rotary && live) {
                    const int half = D / 2;
                    int pair, partner;
                    if (a.interleaved) {
                        pair = e >> 1;
                        partner = (e & 1) == 0 ? e + 1 : e - 1;
                    } else {
                        pair = e < half ? e : e - half;
                        partner = e < half ? e + half : e - half;
                    }
                    cv[j][r] = a.cos_cache[pos * half + pair];
                    sv[j][r] = a.sin_cache[pos * half + pair];
                    xo[j][r] = ld_f32(src + partner);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < RB; j++) {
            const int row = warp * (kPuRows / kPuWarps) + i0 + j;
            float x[EPL];
#pragma unroll
            for (int r = 0; r < EPL; r++) {
                const int e = lane * EPL + r;
                x[r] = xv[j][r];
                if (a.do_rotary) {
                    const bool first = a.interleaved ? (e & 1) == 0 : e < D / 2;
                    x[r] = first ? __fsub_rn(__fmul_rn(cv[j][r], x[r]), __fmul_rn(sv[j][r], xo[j][r]))
                                 : __fadd_rn(__fmul_rn(sv[j][r], xo[j][r]), __fmul_rn(cv[j][r], x[r]));
                }
                x[r] *= sg[e];
            }
            warp_wht_butterfly<EPL>(x, lane, D);
            float sum = 0.0f;
#pragma unroll
            for (int r = 0; r < EPL; r += 2) {
                const int e = lane * EPL + r;
                const float x0 = x[r] * qmul, x1 = x[r + 1] * qmul;
                // sum(q'), or q'.V^T with low-rank K
                sum += vtr ? fmaf(x0, vtr[e], x1 * vtr[e + 1]) : x0 + x1;
                uint32_t hi, lo;
                split_h2(x0, x1, hi, lo);
                const uint32_t off =
                    (uint32_t)((e >> 6) * (kPuRows * 128)) + sw_off(row, (e & 63) >> 3) + (e & 7) * 2;
                *reinterpret_cast<uint32_t *>(qh + off) = hi;
                *reinterpret_cast<uint32_t *>(ql + off) = lo;
            }
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
            if (lane == 0) qsum[row] = sum;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // q' planes -> the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    // this thread's row (warps 0-3): position (a padding row takes the last position) and sum(q')
    const int my_row = tid;  // valid for tid < 128
    int pos_r = 0;
    float qs_r = 0.0f;
    if (warp < 4) {
        int gr = r0 + my_row;
        if (gr >= nrows) gr = nrows - 1;
        pos_r = (int)a.pos0 + gr / G;
        qs_r = qsum[my_row];
    }
    const int last_row = min(r0 + kPuRows, nrows) - 1;
    const int pos_last = (int)a.pos0 + last_row / G;  // the CTA's largest position
    const int ntiles = pos_last / kPuTok + 1;
    const uint32_t tl = tbase + ((uint32_t)(32 * (warp & 3)) << 16);  // this warp's TMEM lane quarter

    const uint8_t *kc = a.k_codes + unit * a.capacity * (int64_t)CB;
    const uint8_t *vc = a.v_codes + unit * a.capacity * (int64_t)CB;
    const float2 *kmeta = reinterpret_cast<const float2 *>(a.k_meta) + unit * a.capacity;
    const float2 *vmeta = reinterpret_cast<const float2 *>(a.v_meta) + unit * a.capacity;
    float *vmax_w = qsum + kPuRows;  // [2 tiles][2]: the tile's largest V scale, per staging warp 4 / 5

    // running max m, the V reference R, sums of p and p * zp (rows of warps 0-3)
    float m_r = -INFINITY, R_r = -INFINITY, l_r = 0.0f, z_r = 0.0f;
    bool aborted = false;
    if (warp >= 4) {
        // ================= staging warps 4-7 (warp 4 also issues the MMAs) =================
        const int st = tid - 128;
        constexpr int NR = CB / 32;  // 16-byte units of K (and of V) per thread per tile
        uint4 rk[NR], rv[NR];
        float2 rkm = make_float2(0.0f, 0.0f), rvm = make_float2(0.0f, 0.0f);
        // raw codes and metadata of tile kt into registers (in flight while the softmax runs)
        auto fetch = [&](int kt) {
            const int t0 = kt * kPuTok;
#pragma unroll
            for (int i = 0; i < NR; i++) {
                const int u = st + 128 * i;
                const int tok = u / (CB / 16), ch = u % (CB / 16);
                rk[i] = *reinterpret_cast<const uint4 *>(kc + (int64_t)(t0 + tok) * CB + 16 * ch);
                const int blk = u / CB, rem = u % CB, c = rem / 4, gq = rem % 4;
                rv[i] = *reinterpret_cast<const uint4 *>(vc + (int64_t)(t0 / 16) * 16 * CB + (int64_t)blk * 16 * CB +
                                                        64 * c + 16 * gq);
            }
            if (st < kPuTok) {
                // tokens past every row's position are masked; their (possibly unwritten) metadata is zeroed
                const bool live = t0 + st <= pos_last;
                rkm = live ? kmeta[t0 + st] : make_float2(0.0f, 0.0f);
                rvm = live ? vmeta[t0 + st] : make_float2(0.0f, 0.0f);
            }
        };
        // registers -> the metadata (buffer mb) and the fp16 K tile (128-byte swizzle) in shared memory
        auto stage_k = [&](int mb) {
            if (st < kPuTok) {
                // token st's metadata in the pair layout the softmax reads two tokens at a time
                float *mt = reinterpret_cast<float *>(meta + mb * kPuTok);
                const int j = st >> 1, sl = st & 1;
                mt[4 * j + sl] = rkm.x;
                mt[4 * j + 2 + sl] = rkm.y;
                mt[4 * kPuTok / 2 + 4 * j + sl] = rvm.x;
                mt[4 * kPuTok / 2 + 4 * j + 2 + sl] = rvm.y;
                float vm = rvm.x;
#pragma unroll
                for (int m = 16; m >= 1; m >>= 1) vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, m));
                if (lane == 0) vmax_w[2 * mb + (st >> 5)] = vm;
            }
#pragma unroll
            for (int i = 0; i < NR; i++) {
                const int u = st + 128 * i;
                const int tok = u / (CB / 16), ch = u % (CB / 16);
                const uint32_t wv[4] = {rk[i].x, rk[i].y, rk[i].z, rk[i].w};
                if constexpr (BITS == 8) {
                    const int e = 16 * ch;  // dims e .. e + 15: two 16-byte chunks of fp16
                    unsigned char *blk = kt_s + (e >> 6) * GG::K_BLK;
                    const int c0 = (e & 63) >> 3;
#pragma unroll
                    for (int hlf = 0; hlf < 2; hlf++) {
                        uint4 o;
                        o.x = bytes_to_h2(wv[2 * hlf], 0x4140u);
                        o.y = bytes_to_h2(wv[2 * hlf], 0x4342u);
                        o.z = bytes_to_h2(wv[2 * hlf + 1], 0x4140u);
                        o.w = bytes_to_h2(wv[2 * hlf + 1], 0x4342u);
                        *reinterpret_cast<uint4 *>(blk + sw_off(tok, c0 + hlf)) = o;
                    }
                } else {
                    const int e = 32 * ch;  // dims e .. e + 31; byte i holds dims 2i (low nibble), 2i + 1
                    unsigned char *blk = kt_s + (e >> 6) * GG::K_BLK;
                    const int c0 = (e & 63) >> 3;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const uint32_t lo = wv[q] & 0x0f0f0f0fu, hi = (wv[q] >> 4) & 0x0f0f0f0fu;
                        const uint32_t d03 = __byte_perm(lo, hi, 0x5140u), d47 = __byte_perm(lo, hi, 0x7362u);
                        uint4 o;
                        o.x = bytes_to_h2(d03, 0x4140u);
                        o.y = bytes_to_h2(d03, 0x4342u);
                        o.z = bytes_to_h2(d47, 0x4140u);
                        o.w = bytes_to_h2(d47, 0x4342u);
                        *reinterpret_cast<uint4 *>(blk + sw_off(tok, c0 + q)) = o;
                    }
                }
            }
        };
        // registers -> the fp16 V tile ([dims][tokens], 128-byte swizzle)
        auto stage_v = [&]() {
#pragma unroll
            for (int i = 0; i < NR; i++) {
                const int u = st + 128 * i;
                // V: chunk c of token group gq of 16-token block blk: byte 4c + jj of tokens tok0 .. tok0 + 3
                const int blkv = u / CB, rem = u % CB, c = rem / 4, gq = rem % 4;
                const int tok0 = blkv * 16 + 4 * gq;
                const uint32_t vv[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w};
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const uint32_t x = vv[jj];
                    if constexpr (BITS == 8) {
                        const int dim = 4 * c + jj;
                        uint2 o;
                        o.x = bytes_to_h2(x, 0x4140u);
                        o.y = bytes_to_h2(x, 0x4342u);
                        *reinterpret_cast<uint2 *>(vt_s + sw_off(dim, tok0 >> 3) + (tok0 & 7) * 2) = o;
                    } else {
#pragma unroll
                        for (int hi = 0; hi < 2; hi++) {
                            const int dim = 2 * (4 * c + jj) + hi;
                            const uint32_t nib = (x >> (4 * hi)) & 0x0f0f0f0fu;
                            uint2 o;
                            o.x = bytes_to_h2(nib, 0x4140u);
                            o.y = bytes_to_h2(nib, 0x4342u);
                            *reinterpret_cast<uint2 *>(vt_s + sw_off(dim, tok0 >> 3) + (tok0 & 7) * 2) = o;
                        }
                    }
                }
            }
        };

        // O += (Uhi + Ulo).C_V of tile kt (the softmax has written U); elected lane of the MMA warp
        auto issue_pv = [&](int kt) {
            constexpr uint32_t ido = pu_idesc(D);
#pragma unroll
            for (int kk = 0; kk < kPuTok / 16; kk++) {
                const uint64_t bd = sw128_kmajor_desc(smem_u32(vt_s) + 32 * kk);
                umma_ts(tbase + kPuO, tbase + kPuUh + 8 * kk, bd, ido, (kt | kk) != 0 ? 1u : 0u);
                umma_ts(tbase + kPuO, tbase + kPuUl + 8 * kk, bd, ido, 1u);
            }
            umma_commit(bar_o);
        };
        // S = (Q'hi + Q'lo).C_K^T of the staged K tile
        auto issue_s = [&]() {
            constexpr uint32_t ids = pu_idesc(kPuTok);
#pragma unroll
            for (int pl = 0; pl < 2; pl++)
#pragma unroll
                for (int kb = 0; kb < GG::KBLK; kb++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t ad = sw128_kmajor_desc(smem_u32((pl ? ql : qh) + kb * (kPuRows * 128)) + 32 * kk);
                        const uint64_t bd = sw128_kmajor_desc(smem_u32(kt_s + kb * GG::K_BLK) + 32 * kk);
                        umma_ss(tbase + kPuS, ad, bd, ids, (pl | kb | kk) != 0 ? 1u : 0u);
                    }
            umma_commit(bar_s);
        };

        fetch(0);
        for (int kt = 0; kt < ntiles; kt++) {
            // K tile and metadata of tile kt: S(kt-1) has read the K tile, and the softmax of
            // tile kt-2 (metadata buffer kt & 1) finished before S(kt-1) was issued
            bool ok = kt == 0 || tc_wait_sleep(bar_s, (uint32_t)((kt - 1) & 1), abort_flag, a.dev_status);
            if (ok) stage_k(kt & 1);
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // staged tiles -> the tensor core
            if (bar_or_4to7(!ok || *abort_flag)) {  // one decision for warps 4-7
                aborted = true;
                break;
            }
            if (warp == kPuMmaWarp) {
                // once the softmax of kt-1 has written U (and read S): PV(kt-1), then S(kt)
                bool uok = kt == 0 || tc_wait_sleep(bar_u, (uint32_t)((kt - 1) & 1), abort_flag, a.dev_status);
                uok = __all_sync(0xffffffffu, uok) && !*abort_flag;
                if (uok) {
                    tc_fence_after();
                    if (elect_one()) {
                        if (kt > 0) issue_pv(kt - 1);
                        issue_s();
                    }
                    __syncwarp();
                }
            }
            // V tile of kt: PV(kt-1) has read the V tile
            ok = kt == 0 || tc_wait_sleep(bar_o, (uint32_t)((kt - 1) & 1), abort_flag, a.dev_status);
            if (ok) stage_v();
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            if (kt + 1 < ntiles) fetch(kt + 1);
        }
        // PV of the last tile, after every staging warp has written its V tile
        if (!bar_or_4to7(aborted || *abort_flag) && warp == kPuMmaWarp) {
            bool uok = tc_wait_sleep(bar_u, (uint32_t)((ntiles - 1) & 1), abort_flag, a.dev_status);
            uok = __all_sync(0xffffffffu, uok) && !*abort_flag;
            if (uok) {
                tc_fence_after();
                if (elect_one()) issue_pv(ntiles - 1);
                __syncwarp();
            }
        }
        // every issued MMA has completed before TMEM is read or freed
        if (warp == kPuMmaWarp) {
            if (elect_one()) umma_commit(bar_fin);
            __syncwarp();
            const uint64_t tw = um_clock_ns();
            while (!um_try(bar_fin, 0) && um_clock_ns() - tw < kTcWaitNs) {
            }
        }
    } else {
        // ================= softmax warps 0-3: one thread per row =================
        for (int kt = 0; kt < ntiles; kt++) {
            const int t0 = kt * kPuTok;
            // S of this tile is complete (and with it every earlier MMA: O and U are free)
            // this tile's metadata, two tokens per float4: {k scale, k zp} pairs, then {v scale, v zp}
            const float4 *kpt = meta + (kt & 1) * kPuTok, *vpt = kpt + kPuTok / 2;
            bool sok = tc_wait_sleep(bar_s, (uint32_t)(kt & 1), abort_flag, a.dev_status);
            sok = __all_sync(0xffffffffu, sok);
            if (!sok) {
                aborted = true;
                break;
            }
            tc_fence_after();
            // tiles that lie wholly at or before every row of the warp need no causal mask
            const bool full = __all_sync(0xffffffffu, t0 + kPuTok - 1 <= pos_r);
            auto softmax_tile = [&](auto masked) {
                constexpr bool MASK = decltype(masked)::value;
                // pass 1: scores (scale / zero point per token, causal mask) and their maximum
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < kPuTok; c += 32) {
                    uint32_t v[32];  // two loads in flight per wait
                    tmem_ld16(tl + kPuS + c, *reinterpret_cast<uint32_t(*)[16]>(v));
                    tmem_ld16(tl + kPuS + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                    tmem_wait_ld();
                    const float2 qq = make_float2(qs_r, qs_r);
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float4 kq = kpt[(c + i) >> 1];
                        // s = acc * kscale + kzp * sum(q'), two tokens per instruction
                        const float2 sp = f2_fma(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                                 make_float2(kq.x, kq.y), f2_mul(make_float2(kq.z, kq.w), qq));
                        mx = fmaxf(mx, (MASK && t0 + c + i > pos_r) ? -INFINITY : sp.x);
                        mx = fmaxf(mx, (MASK && t0 + c + i + 1 > pos_r) ? -INFINITY : sp.y);
                    }
                }
                const float lvmax =
                    __log2f(fmaxf(fmaxf(vmax_w[2 * (kt & 1)], vmax_w[2 * (kt & 1) + 1]), 1.17549435e-38f));
                const float mn = fmaxf(m_r, mx);  // finite: every row sees token 0 in the first tile
                const float fac = exp2f(m_r - mn);
                l_r *= fac;
                z_r *= fac;
                m_r = mn;
                const float cand = mn + lvmax;
                float ofac = 1.0f;
                if (R_r == -INFINITY) {
                    R_r = cand;  // first tile: O is still empty
                } else if (cand > R_r + kPuLazy) {
                    ofac = exp2f(R_r - cand);
                    R_r = cand;
                }
                const float kr = exp2f(mn - R_r);
                if (__any_sync(0xffffffffu, ofac != 1.0f)) {
                    // rescale this warp's rows of O
#pragma unroll 1
                    for (int c = 0; c < D; c += 16) {
                        uint32_t v[16];
                        tmem_ld16(tl + kPuO + c, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * ofac);
                        tmem_st16(tl + kPuO + c, v);
                    }
                }
                // pass 2: p = 2^(s - m), the sums, U = p * vscale * 2^(m-R) as hi + lo fp16 into TMEM
                // (sums of p and p * vzp kept per token parity, added at the end of the tile)
                float2 l2 = make_float2(0.0f, 0.0f), z2 = make_float2(0.0f, 0.0f);
                const float2 qq = make_float2(qs_r, qs_r), nm = make_float2(-mn, -mn), kk = make_float2(kr, kr);
#pragma unroll 1
                for (int c = 0; c < kPuTok; c += 16) {
                    uint32_t v[16];
                    tmem_ld16(tl + kPuS + c, v);
                    tmem_wait_ld();
                    uint32_t uh[8], ul[8];
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const float4 kq = kpt[(c + i) >> 1], vq = vpt[(c + i) >> 1];
                        // s - m = acc * kscale + (kzp * sum(q') - m), two tokens per instruction
                        float2 e = f2_fma(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                          make_float2(kq.x, kq.y), f2_fma(make_float2(kq.z, kq.w), qq, nm));
                        if (MASK) {
                            if (t0 + c + i > pos_r) e.x = -INFINITY;
                            if (t0 + c + i + 1 > pos_r) e.y = -INFINITY;
                        }
                        const float2 p = make_float2(ex2_ftz(e.x), ex2_ftz(e.y));
                        l2 = f2_add(l2, p);
                        z2 = f2_fma(p, make_float2(vq.z, vq.w), z2);
                        const float2 u = f2_mul(p, f2_mul(make_float2(vq.x, vq.y), kk));  // p * (vscale * 2^(m-R))
                        split_h2(u.x, u.y, uh[i / 2], ul[i / 2]);
                    }
                    tmem_st8(tl + kPuUh + c / 2, uh);
                    tmem_st8(tl + kPuUl + c / 2, ul);
                }
                l_r += l2.x + l2.y;
                z_r += z2.x + z2.y;
            };
            if (full) softmax_tile(std::false_type{});
            else softmax_tile(std::true_type{});
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_u);
        }
    }
    if (__syncthreads_or(aborted || *abort_flag)) {
        aborted = true;
    } else {
        tc_fence_after();
    }

    if (!aborted) {
        // ---- O' = (O 2^(R - m) + Z)/L of the row into shared memory (f32, rotated columns) ----
        float *os = reinterpret_cast<float *>(smem);
        if (warp < 4) {
            const float inv = l_r > 0.0f ? 1.0f / l_r : 0.0f;
            const float cu = exp2f(R_r - m_r) * inv, cz = z_r * inv;
#pragma unroll 1
            for (int c = 0; c < D; c += 16) {
                uint32_t v[16];
                tmem_ld16(tl + kPuO + c, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; i++)
                    os[my_row * D + ((c + i + my_row) & (D - 1))] = fmaf(__uint_as_float(v[i]), cu, cz);
            }
        }
        __syncthreads();
        // ---- rotate back and store, one row per warp pass ----
        for (int i = 0; i < kPuRows / kPuWarps; i++) {
            const int row = warp * (kPuRows / kPuWarps) + i, gr = r0 + row;
            if (gr >= nrows) break;
            float x[EPL];
#pragma unroll
            for (int r = 0; r < EPL; r++) x[r] = os[row * D + ((lane * EPL + r + row) & (D - 1))];
            warp_wht_butterfly<EPL>(x, lane, D);
            const int s = gr / G, hd = gr % G;
            T *dst = static_cast<T *>(a.out) + (((int64_t)b * a.seq_len + s) * (a.heads * G) + h * G + hd) * D;
#pragma unroll
            for (int r = 0; r < EPL; r++)
                st_from_f32(dst + lane * EPL + r, x[r] * a.wht_scale * sg[lane * EPL + r]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tbase, kPuTmemCols);
}

template <typename T, int BITS, int D>
int launch_shape(const AttendArgs &a, cudaStream_t stream) {
    using GG = PuGeo<D>;
    auto kern = prefill_umma_kernel<T, BITS, D>;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GG::SMEM);
        if (e != cudaSuccess) return check_cuda(e, "gqa prefill (tcgen05) smem attribute");
        if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
    }
    const int rows = a.seq_len * a.group;
    const int64_t nblocks = (int64_t)((rows + kPuRows - 1) / kPuRows) * a.heads * a.batch;
    if (nblocks > 0x7fffffff)
        return set_error(SA_ERR_UNSUPPORTED, "gqa prefill (tcgen05): %lld blocks", (long long)nblocks);
    kern<<<dim3((unsigned)nblocks), 32 * kPuWarps, GG::SMEM, stream>>>(a);
    count_launch();
    return check_cuda(cudaGetLastError(), "gqa prefill (tcgen05) launch");
}

template <typename T>
int launch_dtype(const AttendArgs &a, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch_shape<T, 4, 128>(a, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch_shape<T, 8, 128>(a, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch_shape<T, 4, 64>(a, stream);
    return launch_shape<T, 8, 64>(a, stream);
}

}  // namespace

// Prefill chunks of 16 or more query tokens, 4/8-bit codes, head_dim 64/128,
// group 1..8, output to attn_out (no head-sharded gather).
bool prefill_eligible(const AttendArgs &a) {
    if (a.seq_len < 16 || a.group < 1 || a.group > 8 || a.gather.n != 0) return false;
    if ((a.bits != 4 && a.bits != 8) || (a.head_dim != 64 && a.head_dim != 128)) return false;
    if (a.capacity % kPuTok != 0) return false;
    return (int64_t)a.seq_len * a.group <= ((int64_t)1 << 30) && a.pos0 + a.seq_len <= ((int64_t)1 << 30);
}

int launch_gqa_prefill_umma(const AttendArgs &a, cudaStream_t stream) {
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_dtype<float>(a, stream);
        case SA_DTYPE_FLOAT16: return launch_dtype<__half>(a, stream);
        default: return launch_dtype<__nv_bfloat16>(a, stream);
    }
}

}  // namespace sa

// Tensor-core decode attention over the PolarQuant cache: one query token per
// sequence, 4/8-bit codes, head_dim 64/128, up to 4 query heads per KV head.
//
// Two launches per step:
//
//  decode_prep_kernel, one CTA per (KV head, batch row):
//    - quantize-on-append of the new token's K and V (same bit-exact encoder
//      as sa_kv_append), when the operator appends;
//    - RoPE + rotation of the G query heads, q' = H.S.q/sqrt(n), written as
//      three signed 8-bit digits of a 24-bit fixed-point number per head:
//      q' ~= sigma * (d0*2^16 + d1*2^8 + d2), |d| <= 127, stored already
//      arranged as each lane's mma B-fragment words.
//
//  decode_persistent_kernel, two CTAs per SM, each looping over work items
//  (batch row, KV head, split of the context).  Warp 8 is the producer: one
//  thread streams every item's K then V chunks (256 tokens each) into a ring
//  of shared-memory slots with 1-D bulk copies (cp.async.bulk + mbarrier, no
//  multicast), running ahead across items as far as free slots allow.
//  Warps 0-7 consume:
//    phase 1 (K): K codes are unpacked to u8 in registers and contracted with
//      the q' digits by mma.m16n8k32 u8 x s8 -> exact int32 dots q'.c; the
//      score s = scale_t*sigma*(q'.c) + zp_t*sum(q') (log2 units) goes to
//      shared memory.
//    phase 2 (V): with the item's reference R = max over max(s, s + log2
//      vscale), every token gets u = 2^(s + log2 vscale - R) in (0, 1] as a
//      24-bit fixed-point number (three unsigned digits) and sum_t u_t * c_t
//      is an exact int32 mma.m16n8k32 u8 x u8 whose B fragments are single
//      32-bit words of the 4-token interleaved V layout.  L = sum u/vscale and
//      Z = sum u*vzp/vscale are float sums.  No rescaling: R is known before
//      phase 2 starts.
//    The last CTA to finish a (row, head) merges its splits (counter per
//    (row, head)), normalises, applies the inverse rotation and stores.
//  Every mbarrier wait is bounded; a wait that gives up sets the cache's
//  device status, the CTA stops writing and drains its own copies.
#include "sa_append.cuh"

namespace sa {

int launch_gqa_combine(const AttendArgs &a, int n_splits, cudaStream_t stream);

namespace {

constexpr int kNW = 8;            // warps per decode CTA
constexpr int kTileW = 12;        // u32 words per row of a warp's P-digit tile
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kQMax = 8355711.0f;   // 127*65536 + 127*256 + 127
constexpr float kUMax = 16777215.0f;  // 2^24 - 1
constexpr uint32_t kWaitLimit = 1u << 22;

// ---- PTX helpers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}


__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// ---- fragment layouts ---------------------------------------------------------
// Dimension carried by logical k (0..31) of K-chunk c for quad q in the QK
// A fragment built from one token's packed codes.
template <int BITS, int D>
__device__ __forceinline__ int k_dim(int c, int q, int k) {
    constexpr int KB = D * BITS / 8;
    constexpr int SEG = KB / 4;
    const int hi = k >> 4, e = k & 3;
    if (BITS == 4) return 2 * (q * SEG + 4 * c + e) + hi;
    return q * SEG + 8 * c + 4 * hi + e;
}

// Dimension carried by column `col` of PV n-tile `nt` (B fragment from the
// 4-token interleaved V words; word index 32*(i/4) + 4*col + i%4).
template <int BITS, int D>
__device__ __forceinline__ int v_dim(int nt, int col) {
    if (BITS == 4) {
        const int i = nt >> 1, hi = nt & 1;
        return 2 * (32 * (i >> 2) + 4 * col + (i & 3)) + hi;
    }
    return 32 * (nt >> 2) + 4 * col + (nt & 3);
}

// Inverse of v_dim: n-tile and column of dimension `dim`.
template <int BITS, int D>
__device__ __forceinline__ void v_inv(int dim, int &nt, int &col) {
    if (BITS == 4) {
        const int w = dim >> 1, hi = dim & 1;
        col = (w >> 2) & 7;
        nt = 2 * (4 * (w >> 5) + (w & 3)) + hi;
    } else {
        col = (dim >> 2) & 7;
        nt = 4 * (dim >> 5) + (dim & 3);
    }
}

template <int BITS, int D>
struct Geo {
    static constexpr int NCH = D / 32;  // QK k-chunks of 32 dimensions
    static constexpr int QW = NCH * 4;  // q-digit words per lane
};

// ---- prep: append the new token + q digits --------------------------------
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(192) decode_prep_kernel(AttendArgs a, AppendArgs ap, int do_append,
                                                          uint32_t *qfrag, float *qscal) {
    using GG = Geo<BITS, D>;
    constexpr int EPL = D / 32;
    __shared__ float s_q[4][D];
    __shared__ float s_sig[4], s_qs[4];
    __shared__ uint8_t s_codes[2][256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.x, b = blockIdx.y;
    const int G = a.group;
    const int q0w = do_append ? 2 : 0;
    const float *sg = a.signs + (int64_t)h * D;
    if (do_append && warp < 2) {
        encode_append_vector<T, EPL>(ap, b, 0, h, warp, lane, s_codes[warp]);
    } else if (warp >= q0w && warp - q0w < G) {
        const int g = warp - q0w;
        const int qheads = a.heads * G;
        const T *src = static_cast<const T *>(a.query) + ((int64_t)b * qheads + h * G + g) * D;
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            const int e = lane * EPL + r;
            x[r] = ld_f32(src + e);
            if (a.do_rotary) x[r] = rope_element(src, x[r], e, D, a.pos0, a.cos_cache, a.sin_cache, a.interleaved);
            x[r] *= sg[e];
        }
        warp_wht_butterfly<EPL>(x, lane, D);
        float sum = 0.0f, mabs = 0.0f;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            x[r] *= a.wht_scale;
            s_q[g][lane * EPL + r] = x[r];
            sum += x[r];
            mabs = fmaxf(mabs, fabsf(x[r]));
        }
        sum = warp_sum(sum);
        mabs = warp_max(mabs);
        if (lane == 0) {
            s_qs[g] = sum;
            s_sig[g] = mabs > 0.0f ? mabs / kQMax : 1.0f;
        }
    }
    __syncthreads();
    if (warp != 0) return;
    // lane (r, q): B fragment words for k-chunk c, n-tile t, half.  n-tile 0
    // column 2j -> (head j, digit 0), 2j+1 -> (head j, digit 1); n-tile 1
    // column 2j -> (head j, digit 2), 2j+1 -> zero.  Column = r.
    const int r = lane >> 2, q = lane & 3;
    const int hh = r >> 1;
    const bool has_head = hh < G;
    const float inv_sigma = has_head ? 1.0f / s_sig[hh] : 0.0f;
    const int64_t bh = (int64_t)b * a.heads + h;
    uint32_t *dst = qfrag + (bh * 32 + lane) * GG::QW;
#pragma unroll
    for (int c = 0; c < GG::NCH; c++) {
#pragma unroll
        for (int half = 0; half < 2; half++) {
            uint32_t w0 = 0, w1 = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int k = 16 * half + 4 * q + e;
                int qi = 0;
                if (has_head) {
                    qi = __float2int_rn(s_q[hh][k_dim<BITS, D>(c, q, k)] * inv_sigma);
                    qi = min(max(qi, -(int)kQMax), (int)kQMax);  // keep the top digit within int8
                }
                const int d2 = (int)(int8_t)(qi & 0xff);
                const int rest = (qi - d2) >> 8;
                const int d1 = (int)(int8_t)(rest & 0xff);
                const int d0 = (rest - d1) >> 8;
                w0 |= ((uint32_t)(((r & 1) ? d1 : d0) & 0xff)) << (8 * e);
                w1 |= ((uint32_t)(((r & 1) ? 0 : d2) & 0xff)) << (8 * e);
            }
            dst[c * 4 + 0 * 2 + half] = w0;  // n-tile 0
            dst[c * 4 + 1 * 2 + half] = w1;  // n-tile 1
        }
    }
    if (lane < 4) {
        const float sl2 = a.scale * kLog2eF;
        qscal[bh * 8 + lane] = lane < G ? s_sig[lane] * sl2 : 0.0f;
        qscal[bh * 8 + 4 + lane] = lane < G ? s_qs[lane] * sl2 : 0.0f;
    }
}

// ---- decode: independent warp streams -------------------------------------------
// Each warp owns a contiguous range of up to kTPW tokens of an item and streams
// it through its own two shared-memory slots (K chunks, then V chunks), so no
// warp ever waits for another inside an item.
constexpr int kTPW = 128;           // tokens per warp per item
constexpr int kScStride = kTPW + 8;  // floats per head row of a warp's score buffer (bank offset)

template <int BITS, int D>
struct WGeo {
    static constexpr int KB = D * BITS / 8;             // code bytes per token
    static constexpr int CT = (KB > 64) ? 32 : 64;       // tokens per chunk
    static constexpr int SLOT = CT * (KB + 16);          // K chunk: codes + K meta + V meta (a V chunk is smaller)
    static constexpr int SEGW = KB / 16;                 // K words per quad per row
    static constexpr int NCH = D / 32;                   // QK k-chunks
    static constexpr int NTV = D / 8;                    // PV n-tiles
    static constexpr int VV = ((BITS == 4) ? NTV / 2 : NTV) / 4;  // 16-byte V loads per 16-token block
    static constexpr int QW = NCH * 4;                   // q-digit words per lane
    static constexpr int SCW = 4 * kScStride;            // floats of a warp's score buffer / merge area
    static constexpr int SMEM = kNW * 2 * SLOT + kNW * SCW * 4 + kNW * 12 * kTileW * 4 + 1024;
    static_assert(4 * D <= SCW, "merge area must fit the score buffer");
};

struct ItemGeo {
    int64_t u;  // b * heads + h
    int b, h, split;
    int64_t s_begin;
    int n_tok;
};

__device__ __forceinline__ ItemGeo item_geo(const AttendArgs &a, int item, int n_splits, int tps) {
    ItemGeo g;
    g.u = item / n_splits;
    g.split = item % n_splits;
    g.b = (int)(g.u / a.heads);
    g.h = (int)(g.u % a.heads);
    g.s_begin = (int64_t)g.split * tps;
    const int64_t total = a.pos0 + 1;
    const int64_t e = g.s_begin + tps < total ? g.s_begin + tps : total;
    g.n_tok = (int)(e - g.s_begin);
    return g;
}

// Tokens of warp `warp` in an item (0 if the item ends before its range).
__device__ __forceinline__ int warp_tokens(int n_tok, int warp, int tpw) {
    const int n = n_tok - warp * tpw;
    return n <= 0 ? 0 : (n < tpw ? n : tpw);
}

// The chunk schedule of one warp over the CTA's items: for every item with a
// non-empty range, its K chunks then its V chunks.  Lane 0 keeps the cursor
// of the next chunk to issue, two chunks ahead of consumption.
template <int BITS, int D>
struct WarpStream {
    using GG = WGeo<BITS, D>;
    int item, c, nk, n;
    int64_t u, t0;

    __device__ __forceinline__ void seek(const AttendArgs &a, int n_items, int n_splits, int tps, int tpw, int warp) {
        for (; item < n_items; item += gridDim.x) {
            const ItemGeo g = item_geo(a, item, n_splits, tps);
            n = warp_tokens(g.n_tok, warp, tpw);
            if (n > 0) {
                u = g.u;
                t0 = g.s_begin + (int64_t)warp * tpw;
                nk = (n + GG::CT - 1) / GG::CT;
                c = 0;
                return;
            }
        }
    }

    __device__ __forceinline__ void issue(const AttendArgs &a, unsigned char *dst, uint64_t *bar) const {
        constexpr int KB = GG::KB, CT = GG::CT;
        const int64_t cap = a.capacity;
        const int cc = c < nk ? c : c - nk;
        const int cnt = n - cc * CT < CT ? n - cc * CT : CT;
        const int mcnt = (cnt + 1) & ~1;  // meta rows rounded to even: 16-byte copies
        const int64_t g0 = t0 + cc * CT;  // multiple of CT (>= 32)
        const uint32_t mb = (uint32_t)(mcnt * 8);
        if (c < nk) {  // K chunk: codes, K meta, V meta
            const uint32_t cb = (uint32_t)(cnt * KB);
            mbar_expect_tx(bar, cb + 2 * mb);
            bulk_g2s(dst, a.k_codes + (u * cap + g0) * KB, cb, bar);
            bulk_g2s(dst + CT * KB, a.k_meta + (u * cap + g0) * 2, mb, bar);
            bulk_g2s(dst + CT * KB + CT * 8, a.v_meta + (u * cap + g0) * 2, mb, bar);
        } else {  // V chunk: whole 16-token blocks of codes, V meta
            const uint32_t vb = (uint32_t)(((cnt + kVBlock - 1) / kVBlock) * KB * kVBlock);
            mbar_expect_tx(bar, vb + mb);
            bulk_g2s(dst, a.v_codes + (u * cap + g0) * KB, vb, bar);
            bulk_g2s(dst + CT * KB, a.v_meta + (u * cap + g0) * 2, mb, bar);
        }
    }

    __device__ __forceinline__ void advance(const AttendArgs &a, int n_items, int n_splits, int tps, int tpw,
                                            int warp) {
        if (++c == 2 * nk) {
            item += gridDim.x;
            seek(a, n_items, n_splits, tps, tpw, warp);
        }
    }
};

template <typename T, int BITS, int D>
__global__ void __launch_bounds__(kNW * 32, 2)
    decode_stream_kernel(AttendArgs a, int n_splits, int tps, int tpw, int n_items, const uint32_t *__restrict__ qfrag,
                         const float *__restrict__ qscal) {
    using GG = WGeo<BITS, D>;
    constexpr int KB = GG::KB, CT = GG::CT;
    constexpr int EPL = D / 32;

    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned char *slots = smem + warp * 2 * GG::SLOT;                              // this warp's 2 slots
    float *scw_all = reinterpret_cast<float *>(smem + kNW * 2 * GG::SLOT);          // [kNW][4][kScStride]
    float *scw = scw_all + warp * GG::SCW;                                          // s' scores, then merge area
    uint32_t *tile = reinterpret_cast<uint32_t *>(scw_all + kNW * GG::SCW) + warp * 12 * kTileW;
    float *rlz = reinterpret_cast<float *>(reinterpret_cast<uint32_t *>(scw_all + kNW * GG::SCW) + kNW * 12 * kTileW);
    int *s_flag = reinterpret_cast<int *>(rlz + kNW * 4 * 3);                       // [1] failure
    uint64_t *bars = reinterpret_cast<uint64_t *>(rlz + 128);                      // [kNW][2]
    uint64_t *mybar = bars + 2 * warp;

    const int G = a.group;
    const int r = lane >> 2, q = lane & 3;
    const int ph = lane >> 3, tq = lane & 7;  // P-digit role: head ph, token quad tq of a 32-token step
    const bool my_head = q < G;

    if (tid == 0) {
        for (int i = 0; i < 2 * kNW; i++) mbar_init(bars + i, 1);
        s_flag[0] = 0;
        s_flag[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();

    WarpStream<BITS, D> ws;
    if (lane == 0) {
        ws.item = blockIdx.x;
        ws.seek(a, n_items, n_splits, tps, tpw, warp);
        for (int k = 0; k < 2 && ws.item < n_items; k++) {
            ws.issue(a, slots + k * GG::SLOT, mybar + k);
            ws.advance(a, n_items, n_splits, tps, tpw, warp);
        }
    }

    int j = 0;  // chunks consumed by this warp
    bool failed = false;
    // wait for chunk j; afterwards lane 0 refills its slot with the chunk two ahead
    auto wait_chunk = [&](int jj) {
        if (!failed && !mbar_wait_bounded(mybar + (jj & 1), (uint32_t)((jj >> 1) & 1))) {
            failed = true;
            atomicOr(a.dev_status, 1);
            s_flag[1] = 1;
        }
    };
    auto release_chunk = [&](int jj) {
        __syncwarp();
        if (lane == 0 && ws.item < n_items) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            ws.issue(a, slots + (jj & 1) * GG::SLOT, mybar + (jj & 1));
            ws.advance(a, n_items, n_splits, tps, tpw, warp);
        }
    };

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const ItemGeo ig = item_geo(a, item, n_splits, tps);
        const int n_w = warp_tokens(ig.n_tok, warp, tpw);
        const int nk = (n_w + CT - 1) / CT;
        float Rp = -INFINITY, Lp = 0.0f, Zp = 0.0f;
        int pacc[GG::NTV][4];
#pragma unroll
        for (int nt = 0; nt < GG::NTV; nt++) pacc[nt][0] = pacc[nt][1] = pacc[nt][2] = pacc[nt][3] = 0;

        if (n_w > 0) {
            uint32_t bq[GG::QW];
            {
                const uint4 *src = reinterpret_cast<const uint4 *>(qfrag + (ig.u * 32 + lane) * GG::QW);
#pragma unroll
                for (int v = 0; v < GG::QW / 4; v++) {
                    const uint4 x = src[v];
                    bq[4 * v] = x.x;
                    bq[4 * v + 1] = x.y;
                    bq[4 * v + 2] = x.z;
                    bq[4 * v + 3] = x.w;
                }
            }
            const float c1 = qscal[ig.u * 8 + q], c2 = qscal[ig.u * 8 + 4 + q];

            // ---------------- phase 1: scores s' = s + log2(vscale) ----------------
            float rmax = -INFINITY;
            for (int cc = 0; cc < nk; cc++, j++) {
                wait_chunk(j);
                const unsigned char *st = slots + (j & 1) * GG::SLOT;
                const float *kms = reinterpret_cast<const float *>(st + CT * KB);
                const float *vms = kms + 2 * CT;
#pragma unroll
                for (int mt = 0; mt < CT / 16; mt++) {
                    uint32_t w[2][GG::SEGW];
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        const unsigned char *p = st + (16 * mt + r + 8 * hf) * KB + q * (KB / 4);
                        if constexpr (GG::SEGW == 2) {
                            const uint2 x = *reinterpret_cast<const uint2 *>(p);
                            w[hf][0] = x.x;
                            w[hf][1] = x.y;
                        } else {
#pragma unroll
                            for (int v = 0; v < GG::SEGW / 4; v++) {
                                const uint4 x = reinterpret_cast<const uint4 *>(p)[v];
                                w[hf][4 * v] = x.x;
                                w[hf][4 * v + 1] = x.y;
                                w[hf][4 * v + 2] = x.z;
                                w[hf][4 * v + 3] = x.w;
                            }
                        }
                    }
                    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
                    for (int k = 0; k < GG::NCH; k++) {
                        uint32_t a0, a1, a2, a3;
                        if constexpr (BITS == 4) {
                            a0 = w[0][k] & 0x0F0F0F0Fu;
                            a1 = w[1][k] & 0x0F0F0F0Fu;
                            a2 = (w[0][k] >> 4) & 0x0F0F0F0Fu;
                            a3 = (w[1][k] >> 4) & 0x0F0F0F0Fu;
                        } else {
                            a0 = w[0][2 * k];
                            a1 = w[1][2 * k];
                            a2 = w[0][2 * k + 1];
                            a3 = w[1][2 * k + 1];
                        }
                        mma_u8s8(acc[0], a0, a1, a2, a3, bq[k * 4 + 0], bq[k * 4 + 1]);
                        mma_u8s8(acc[1], a0, a1, a2, a3, bq[k * 4 + 2], bq[k * 4 + 3]);
                    }
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        const int row = 16 * mt + r + 8 * hf;  // token within the chunk
                        const int tl = cc * CT + row;          // token within the warp's range
                        const float dot = fmaf((float)acc[0][2 * hf], 65536.0f,
                                               (float)(acc[0][2 * hf + 1] * 256 + acc[1][2 * hf]));
                        const float2 km = *reinterpret_cast<const float2 *>(kms + 2 * row);
                        const float s = fmaf(km.x * c1, dot, km.y * c2);
                        const float sp = s + __log2f(vms[2 * row]);
                        if (tl < n_w && my_head) {
                            scw[q * kScStride + tl] = sp;
                            rmax = fmaxf(rmax, fmaxf(s, sp));
                        }
                    }
                }
                release_chunk(j);
            }
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
            Rp = __shfl_sync(0xffffffffu, rmax, ph);  // lane ph holds head ph's max

            // ---------------- phase 2: values ----------------
            for (int cc = 0; cc < nk; cc++, j++) {
                wait_chunk(j);
                const unsigned char *st = slots + (j & 1) * GG::SLOT;
                const float *vms = reinterpret_cast<const float *>(st + CT * KB);
#pragma unroll
                for (int sp = 0; sp < CT / 32; sp++) {
                    const int tc = 32 * sp + 4 * tq;  // this lane's first token within the chunk
                    const int tb = cc * CT + tc;      // ... within the warp's range
                    uint32_t U[4] = {0u, 0u, 0u, 0u};
                    if (ph < G && tb < n_w) {
                        const float4 s4 = *reinterpret_cast<const float4 *>(scw + ph * kScStride + tb);
                        const float4 m01 = *reinterpret_cast<const float4 *>(vms + 2 * tc);
                        const float4 m23 = *reinterpret_cast<const float4 *>(vms + 2 * tc + 4);
                        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
                        const float vs[4] = {m01.x, m01.z, m23.x, m23.z}, vz[4] = {m01.y, m01.w, m23.y, m23.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            if (tb + e < n_w) {
                                const float u = fminf(ex2_approx(sv[e] - Rp), 1.0f);
                                const float iv = __frcp_rn(vs[e]);
                                Lp = fmaf(u, iv, Lp);
                                Zp = fmaf(u, vz[e] * iv, Zp);
                                U[e] = __float2uint_rn(u * kUMax);
                            }
                        }
                    }
                    // digit j of the 4 tokens -> one A-fragment word (row 4j + head, token quad tq)
                    const uint32_t lo0 = __byte_perm(U[0], U[1], 0x0062), hi0 = __byte_perm(U[2], U[3], 0x0062);
                    const uint32_t lo1 = __byte_perm(U[0], U[1], 0x0051), hi1 = __byte_perm(U[2], U[3], 0x0051);
                    const uint32_t lo2 = __byte_perm(U[0], U[1], 0x0040), hi2 = __byte_perm(U[2], U[3], 0x0040);
                    tile[(0 + ph) * kTileW + tq] = __byte_perm(lo0, hi0, 0x5410);
                    tile[(4 + ph) * kTileW + tq] = __byte_perm(lo1, hi1, 0x5410);
                    tile[(8 + ph) * kTileW + tq] = __byte_perm(lo2, hi2, 0x5410);
                    __syncwarp();
                    const uint32_t pa0 = tile[r * kTileW + q], pa2 = tile[r * kTileW + 4 + q];
                    const uint32_t pa1 = r < 4 ? tile[(r + 8) * kTileW + q] : 0u;
                    const uint32_t pa3 = r < 4 ? tile[(r + 8) * kTileW + 4 + q] : 0u;
                    __syncwarp();
                    // V words of token group q of 16-token blocks 2sp (b0) and 2sp+1 (b1)
#pragma unroll
                    for (int v = 0; v < GG::VV; v++) {
                        const unsigned char *vb0 = st + (2 * sp) * (KB * kVBlock) + (8 * v + r) * 64 + 16 * q;
                        const uint4 x0 = *reinterpret_cast<const uint4 *>(vb0);
                        const uint4 x1 = *reinterpret_cast<const uint4 *>(vb0 + KB * kVBlock);
                        const uint32_t y0[4] = {x0.x, x0.y, x0.z, x0.w}, y1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) {
                            const int i = 4 * v + jj;
                            if constexpr (BITS == 4) {
                                // high nibbles used in place (16 * code): n-tile 2i+1 sums 16x, scaled at the end
                                mma_u8u8(pacc[2 * i], pa0, pa1, pa2, pa3, y0[jj] & 0x0F0F0F0Fu, y1[jj] & 0x0F0F0F0Fu);
                                mma_u8u8(pacc[2 * i + 1], pa0, pa1, pa2, pa3, y0[jj] & 0xF0F0F0F0u,
                                         y1[jj] & 0xF0F0F0F0u);
                            } else {
                                mma_u8u8(pacc[i], pa0, pa1, pa2, pa3, y0[jj], y1[jj]);
                            }
                        }
                    }
                }
                release_chunk(j);
            }
        }

        // ---------------- warp partial -> its merge area ----------------
        Lp += __shfl_xor_sync(0xffffffffu, Lp, 1);
        Lp += __shfl_xor_sync(0xffffffffu, Lp, 2);
        Lp += __shfl_xor_sync(0xffffffffu, Lp, 4);
        Zp += __shfl_xor_sync(0xffffffffu, Zp, 1);
        Zp += __shfl_xor_sync(0xffffffffu, Zp, 2);
        Zp += __shfl_xor_sync(0xffffffffu, Zp, 4);
        __syncwarp();  // scw (scores) becomes the merge area
        {
            // rows: r < 4 -> (digit 0, head r) in c0/c1 and (digit 2, head r) in c2/c3;
            // r >= 4 -> (digit 1, head r - 4) in c0/c1.  value = (d0*2^16 + d1*2^8 + d2) / (2^24 - 1).
            // Lanes r < 4 store head r's value of column 2q+cc of n-tile nt at
            // (nt*2 + cc)*16 + lane: 16 consecutive words per store, no bank conflicts.
            const float w_lo = (r < 4) ? 65536.0f / kUMax : 256.0f / kUMax;
            const float w_d2 = 1.0f / kUMax;
#pragma unroll
            for (int nt = 0; nt < GG::NTV; nt++) {
                const float ntw = (BITS == 4 && (nt & 1)) ? 0.0625f : 1.0f;  // high-nibble tiles hold 16 * code
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    float f = (float)pacc[nt][cc] * w_lo;
                    if (r < 4) f = fmaf((float)pacc[nt][2 + cc], w_d2, f);
                    const float mid = __shfl_down_sync(0xffffffffu, f, 16);
                    if (r < 4) scw[(nt * 2 + cc) * 16 + lane] = (f + mid) * ntw;
                }
            }
        }
        if (tq == 0) {
            rlz[(warp * 4 + ph) * 3 + 0] = (n_w > 0 && ph < G) ? Rp : -INFINITY;
            rlz[(warp * 4 + ph) * 3 + 1] = Lp;
            rlz[(warp * 4 + ph) * 3 + 2] = Zp;
        }
        __syncthreads();

        // ---------------- merge the warps: warp g finishes head g ----------------
        // Splits are merged afterwards by attend_combine_kernel.
        const bool fail_now = *reinterpret_cast<volatile int *>(&s_flag[1]) != 0;
        if (warp < G && !fail_now) {
            const int g = warp;
            float M = -INFINITY;
#pragma unroll
            for (int w2 = 0; w2 < kNW; w2++) M = fmaxf(M, rlz[(w2 * 4 + g) * 3]);
            int idx[EPL];
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) {
                int nt, col;
                v_inv<BITS, D>(lane * EPL + rr, nt, col);
                idx[rr] = (nt * 2 + (col & 1)) * 16 + 4 * g + (col >> 1);
            }
            float L = 0.0f, Z = 0.0f, x[EPL];
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) x[rr] = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < kNW; w2++) {
                const float Rw = rlz[(w2 * 4 + g) * 3];
                if (Rw == -INFINITY) continue;
                const float wt = exp2f(Rw - M);
                L = fmaf(wt, rlz[(w2 * 4 + g) * 3 + 1], L);
                Z = fmaf(wt, rlz[(w2 * 4 + g) * 3 + 2], Z);
                const float *mw = scw_all + w2 * GG::SCW;
#pragma unroll
                for (int rr = 0; rr < EPL; rr++) x[rr] = fmaf(wt, mw[idx[rr]], x[rr]);
            }
            if (n_splits == 1) {
                const float *sg = a.signs + (int64_t)ig.h * D;
                const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
                for (int rr = 0; rr < EPL; rr++) x[rr] = L > 0.0f ? (x[rr] + Z) * inv : 0.0f;
                warp_wht_butterfly<EPL>(x, lane, D);
                T *dst = static_cast<T *>(a.out) + ((int64_t)ig.b * a.heads * G + ig.h * G + g) * D;
#pragma unroll
                for (int rr = 0; rr < EPL; rr++)
                    st_from_f32(dst + lane * EPL + rr, x[rr] * a.wht_scale * sg[lane * EPL + rr]);
            } else {
                float *wsp = a.workspace + ((ig.u * n_splits + ig.split) * G + g) * (D + 4);
                if (EPL == 4) {
                    *reinterpret_cast<float4 *>(wsp + lane * 4) = make_float4(x[0], x[1 % EPL], x[2 % EPL], x[3 % EPL]);
                } else {
#pragma unroll
                    for (int rr = 0; rr < EPL; rr++) wsp[lane * EPL + rr] = x[rr];
                }
                if (lane == 0) {
                    wsp[D] = M;
                    wsp[D + 1] = L;
                    wsp[D + 2] = Z;
                }
            }
        }
        __syncthreads();  // merge areas and flags are reused by the next item
    }

    if (failed && lane == 0) {
        // a wait gave up: let the (at most two) copies this warp still has in flight land (bounded)
        for (int jj = j; jj < j + 2; jj++) mbar_wait_bounded(mybar + (jj & 1), (uint32_t)((jj >> 1) & 1));
    }
}

template <typename T, int BITS, int D>
int launch_shape(const AttendArgs &a, const AppendArgs *ap, int n_splits, int tps, cudaStream_t stream) {
    uint32_t *qfrag = a.qprep;
    float *qscal = reinterpret_cast<float *>(a.qprep + (size_t)a.batch * a.heads * 32 * 16);
    const int do_append = ap != nullptr;
    AppendArgs apv{};
    if (ap) apv = *ap;
    const int prep_warps = (do_append ? 2 : 0) + a.group;
    decode_prep_kernel<T, BITS, D><<<dim3(a.heads, a.batch), 32 * prep_warps, 0, stream>>>(a, apv, do_append,
                                                                                            qfrag, qscal);
    count_launch();
    int rc = check_cuda(cudaGetLastError(), "gqa decode prep launch");
    if (rc != SA_OK) return rc;

    using GG = WGeo<BITS, D>;
    auto kern = decode_stream_kernel<T, BITS, D>;
    const size_t smem = GG::SMEM;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "gqa decode smem attribute");
        if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
    }
    const int n_items = a.batch * a.heads * n_splits;
    int grid = 2 * a.sm_count;
    if (grid > n_items) grid = n_items;
    const int tpw = tps / kNW;
    kern<<<grid, kNW * 32, smem, stream>>>(a, n_splits, tps, tpw, n_items, qfrag, qscal);
    count_launch();
    int rc2 = check_cuda(cudaGetLastError(), "gqa decode launch");
    if (rc2 != SA_OK || n_splits == 1) return rc2;
    return launch_gqa_combine(a, n_splits, stream);
}

template <typename T>
int launch_dtype(const AttendArgs &a, const AppendArgs *ap, int n_splits, int tps, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch_shape<T, 4, 128>(a, ap, n_splits, tps, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch_shape<T, 8, 128>(a, ap, n_splits, tps, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch_shape<T, 4, 64>(a, ap, n_splits, tps, stream);
    return launch_shape<T, 8, 64>(a, ap, n_splits, tps, stream);
}

}  // namespace

// Whether the tensor-core decode handles this call.
bool decode_fast_eligible(const AttendArgs &a) {
    if (a.seq_len != 1 || a.group < 1 || a.group > 4) return false;
    if ((a.bits != 4 && a.bits != 8) || (a.head_dim != 64 && a.head_dim != 128)) return false;
    if (a.capacity % 64 != 0 || a.qprep == nullptr || a.dev_status == nullptr)
        return false;
    const int64_t total = a.pos0 + 1;
    if (total > (int64_t)kMaxSplits * kNW * kTPW) return false;
    // every split's partial must fit the workspace
    const int64_t units = (int64_t)a.batch * a.heads;
    return (size_t)((int64_t)kMaxSplits * units * a.group * (a.head_dim + 4)) <= a.workspace_floats;
}

// Prep (+ append when `ap` is given) and decode of one query token per row.
int launch_gqa_decode_fast(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    const int64_t total = a.pos0 + 1;
    const int64_t units = (int64_t)a.batch * a.heads;
    // splits: at most kNW * kTPW tokens each, a multiple of kNW * 64 (whole
    // chunks per warp); enough work items for ~8 per persistent CTA.
    const int64_t grain = (int64_t)kNW * 64, cap_tok = (int64_t)kNW * kTPW;
    int64_t n = (total + cap_tok - 1) / cap_tok;
    const int64_t want = (16LL * a.sm_count + units - 1) / units;
    const int64_t by_len = (total + grain - 1) / grain;
    const int64_t more = want < by_len ? want : by_len;
    if (n < more) n = more;
    if (n > kMaxSplits) n = kMaxSplits;
    int64_t tps = (total + n - 1) / n;
    tps = (tps + grain - 1) / grain * grain;
    n = (total + tps - 1) / tps;
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_dtype<float>(a, ap, (int)n, (int)tps, stream);
        case SA_DTYPE_FLOAT16: return launch_dtype<__half>(a, ap, (int)n, (int)tps, stream);
        default: return launch_dtype<__nv_bfloat16>(a, ap, (int)n, (int)tps, stream);
    }
}

}  // namespace sa

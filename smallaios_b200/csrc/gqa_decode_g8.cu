// Tensor-core decode attention for 5..8 query heads per KV head (the
// Llama-3-70B shape: 64 query heads over 8 KV heads): one query token per
// sequence, 4/8-bit codes, head_dim 64/128.
//
// Same three launches and the same integer arithmetic as the decode for up
// to four heads (gqa_decode_mma.cu); what changes is how eight heads share
// one pass over the KV stream:
//
//  decode_prep8_kernel: quantize-on-append of the new token, then the eight
//    query heads as three signed 8-bit digits each, laid out as the B
//    fragments of three n-tiles: n-tile 0 holds heads 0-3 (digits 0 and 1),
//    n-tile 1 heads 4-7 (digits 0 and 1), n-tile 2 digit 2 of all eight.
//    Lane (r, q) of the QK product then owns the dots of heads q and q + 4.
//
//  decode8_stream_kernel: one CTA of 12 warps per SM (12 x 15 KB of slots and
//    score buffers), the stream-K chunk ranges of the four-head kernel.  K
//    chunks are contracted against the three n-tiles (three mma per
//    16 tokens x 32 dimensions); the scores of the eight heads go to shared
//    memory.  The V chunks are contracted twice from shared memory, once per
//    half of the heads, with the four-head P tile (rows: digit j of head
//    4*half + i at row 4j + i), so the integer sums of one half (64
//    registers) are folded before the other half starts.  A warp's partial
//    record holds all eight heads.
//
//  decode_merge_kernel<T, D, 8>: one warp per query head.
#include "sa_append.cuh"
#include "sa_async.cuh"
#include "sa_decode_common.cuh"

namespace sa {

namespace {

using namespace dec;

constexpr int kNW8 = 12;    // warps per decode CTA (one CTA per SM)
constexpr int kTileW = 8;   // u32 words per row of a warp's P-digit tile (12 rows)

template <int BITS, int D>
struct G8Geo {
    static constexpr int KB = D * BITS / 8;             // code bytes per token
    static constexpr int CT = (KB > 64) ? 32 : 64;       // tokens per chunk
    static constexpr int TPW = 2 * CT;                   // tokens per sub-segment
    static constexpr int SCS = TPW + 8;                  // floats per head row of a warp's score buffer
    static constexpr int SLOT = CT * (KB + 16);          // K chunk: codes + K meta + V meta
    static constexpr int SEGW = KB / 16;                 // K words per quad per row
    static constexpr int NCH = D / 32;                   // QK k-chunks
    static constexpr int NTV = D / 8;                    // PV n-tiles
    static constexpr int NF = NTV;                       // float value sums per lane and half
    static constexpr int VV = ((BITS == 4) ? NTV / 2 : NTV) / 4;  // 16-byte V loads per 16-token block
    static constexpr int QW = NCH * 6;                   // q-digit words per lane: 3 n-tiles x 2 halves
    static constexpr int SCW = 8 * SCS;                  // floats of a warp's score buffer
    static constexpr int REC = RecGeo<D, 8>::REC;        // floats per partial record
    static constexpr int SMEM = kNW8 * 2 * SLOT + kNW8 * SCW * 4 + kNW8 * 12 * kTileW * 4 + 256;
    static_assert(SMEM <= 227 * 1024, "decode8 shared memory");
};

constexpr int kQWMax8 = 24;  // q-digit words per lane at head_dim 128

// B-fragment column (n-tile t, column fr) that carries digit dg of head g.
__device__ __forceinline__ void frag_column8(int g, int dg, int &t, int &fr) {
    if (g < 4) {
        t = dg == 2 ? 2 : 0;
        fr = dg == 2 ? 2 * g : 2 * g + dg;
    } else {
        t = dg == 2 ? 2 : 1;
        fr = dg == 2 ? 2 * (g - 4) + 1 : 2 * (g - 4) + dg;
    }
}

// ---- prep: append the new token + q digits of eight heads ----------------------
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(320) decode_prep8_kernel(AttendArgs a, AppendArgs ap, int do_append,
                                                           uint32_t *qfrag, float *qscal) {
    using GG = G8Geo<BITS, D>;
    constexpr int EPL = D / 32;
    __shared__ float s_q[8][D];
    __shared__ uint8_t s_codes[2][256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.x, b = blockIdx.y;
    const int G = a.group;
    const int q0w = do_append ? 2 : 0;
    const float *sg = a.signs + (int64_t)h * D;
    griddep_launch_dependents();
    griddep_wait();  // launched as a dependent of the kernel before it: q and the cache are ready
    if (do_append && warp < 2) {
        encode_append_vector<T, EPL>(ap, b, 0, h, warp, lane, s_codes[warp]);
        return;
    }
    const int g = warp - q0w;
    if (g < 0 || g >= 8) return;
    const int64_t bh = (int64_t)b * a.heads + h;
    uint32_t *frag = qfrag + bh * 32 * GG::QW;
    float sigma = 1.0f, inv_sigma = 0.0f, sum = 0.0f;
    if (g < G) {
        const int qheads = a.heads * G;
        const T *src = static_cast<const T *>(a.query) + ((int64_t)b * qheads + h * G + g) * D;
        float x[EPL];
#pragma unroll
        for (int r = 0; r < EPL; r++) x[r] = 0.0f;
        load_elems<T, EPL>(src + lane * EPL, x);
        if (a.do_rotary) rope_lane<EPL>(x, lane, D, a.pos0, a.cos_cache, a.sin_cache, a.interleaved);
#pragma unroll
        for (int r = 0; r < EPL; r++) x[r] *= sg[lane * EPL + r];
        warp_wht_butterfly<EPL>(x, lane, D);
        float mabs = 0.0f;
        const float *vtr = a.lr_vtr ? a.lr_vtr + bh * D : nullptr;
#pragma unroll
        for (int r = 0; r < EPL; r++) {
            x[r] *= a.wht_scale;
            s_q[g][lane * EPL + r] = x[r];
            sum += vtr ? x[r] * vtr[lane * EPL + r] : x[r];  // sum(q'), or q'.V^T with low-rank K
            mabs = fmaxf(mabs, fabsf(x[r]));
        }
        sum = warp_sum(sum);
        mabs = warp_max(mabs);
        sigma = mabs > 0.0f ? mabs / kQMax : 1.0f;
        inv_sigma = 1.0f / sigma;
    }
    if (lane == 0) {
        const float sl2 = a.scale * kLog2eF;
        qscal[bh * 16 + g] = g < G ? sigma * sl2 : 0.0f;
        qscal[bh * 16 + 8 + g] = g < G ? sum * sl2 : 0.0f;
    }
    __syncwarp();  // s_q[g] complete
    // Head g's words: for k-chunk c, fragment k-group fq and half hf, the
    // word of digit dg sits at fragment lane fr*4 + fq, index c*6 + t*2 + hf.
    for (int it = lane; it < 8 * GG::NCH; it += 32) {
        const int fq = it & 3, hf = (it >> 2) & 1, c = it >> 3;
        uint32_t w0 = 0, w1 = 0, w2 = 0;
        if (g < G) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int k = 16 * hf + 4 * fq + e;
                int qi = __float2int_rn(s_q[g][k_dim<BITS, D>(c, fq, k)] * inv_sigma);
                qi = min(max(qi, -(int)kQMax), (int)kQMax);
                const int d2 = (int)(int8_t)(qi & 0xff);
                const int rest = (qi - d2) >> 8;
                const int d1 = (int)(int8_t)(rest & 0xff);
                const int d0 = (rest - d1) >> 8;
                w0 |= ((uint32_t)(d0 & 0xff)) << (8 * e);
                w1 |= ((uint32_t)(d1 & 0xff)) << (8 * e);
                w2 |= ((uint32_t)(d2 & 0xff)) << (8 * e);
            }
        }
        const uint32_t wd[3] = {w0, w1, w2};
#pragma unroll
        for (int dg = 0; dg < 3; dg++) {
            int t, fr;
            frag_column8(g, dg, t, fr);
            frag[(fr * 4 + fq) * GG::QW + c * 6 + t * 2 + hf] = wd[dg];
        }
    }
}

// ---- decode: stream-K warp ranges over eight heads -------------------------------
template <typename T, int BITS, int D>
__global__ void __launch_bounds__(kNW8 * 32, 1)
    decode8_stream_kernel(AttendArgs a, int ncu, int F, int W, const uint32_t *__restrict__ qfrag,
                          const float *__restrict__ qscal) {
    using GG = G8Geo<BITS, D>;
    using RG = RecGeo<D, 8>;
    constexpr int KB = GG::KB, CT = GG::CT, SCS = GG::SCS;

    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned char *slots = smem + warp * 2 * GG::SLOT;
    float *scw = reinterpret_cast<float *>(smem + kNW8 * 2 * GG::SLOT) + warp * GG::SCW;
    uint32_t *tile = reinterpret_cast<uint32_t *>(smem + kNW8 * 2 * GG::SLOT + kNW8 * GG::SCW * 4) +
                     warp * 12 * kTileW;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kNW8 * 2 * GG::SLOT + kNW8 * GG::SCW * 4 +
                                                  kNW8 * 12 * kTileW * 4);  // [kNW8][2]
    uint64_t *mybar = bars + 2 * warp;

    const int r = lane >> 2, q = lane & 3;
    const int ph = lane >> 3, tq = lane & 7;  // P-digit role: head ph of a half, token quad tq
    const bool lo = lane < 16;

    if (tid == 0) {
        for (int i = 0; i < 2 * kNW8; i++) mbar_init(bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();  // the only block-wide barrier
    griddep_launch_dependents();
    const int w = blockIdx.x * kNW8 + warp;
    if (w >= W) return;
    const int f0 = (int)((int64_t)w * F / W), f1 = (int)((int64_t)(w + 1) * F / W);
    const int total = (int)a.pos0 + 1;

    unsigned pend = 0;
    bool failed = false;
    auto issue = [&](int s, int uu, int c, int kind) {
        constexpr uint32_t kCodeBytes = CT * KB, kMetaBytes = CT * 8;
        const int64_t row = (int64_t)uu * a.capacity + c * CT;
        uint64_t *bar = mybar + s;
        if (lane == 0) mbar_expect_tx(bar, kCodeBytes + (kind == 0 ? 2 * kMetaBytes : kMetaBytes));
        if (lane < 3 - kind) {
            const void *src;
            uint32_t nb = kMetaBytes, off;
            if (lane == 0) {
                src = (kind == 0 ? a.k_codes : a.v_codes) + row * KB;
                nb = kCodeBytes;
                off = 0;
            } else if (lane == 1) {
                src = (kind == 0 ? a.k_meta : a.v_meta) + row * 2;
                off = CT * KB;
            } else {
                src = a.v_meta + row * 2;
                off = CT * KB + CT * 8;
            }
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            bulk_g2s(slots + s * GG::SLOT + off, src, nb, bar);
        }
        pend |= 1u << (2 * s + kind);
    };
    auto issue_empty = [&](int s, int kind) {
        if (lane == 0) mbar_arrive(mybar + s);
        pend |= 1u << (2 * s + kind);
    };
    auto wait = [&](int s, int kind) {
        const bool ok = mbar_wait_bounded(mybar + s, (uint32_t)kind);
        if (__any_sync(0xffffffffu, !ok)) {
            failed = true;
            if (lane == 0) atomicOr(a.dev_status, 1);
        } else {
            pend &= ~(1u << (2 * s + kind));
        }
    };

    int u = f0 / ncu, ubase = u * ncu, fs = f0;
    int ns = min(2, min(f1, ubase + ncu) - fs);
    {
        const bool new0 = fs - ubase == ncu - 1, new1 = ns > 1 && fs - ubase + 1 == ncu - 1;
        if (!new0) issue(0, u, fs - ubase, 0);
        if (ns < 2) issue_empty(1, 0);
        else if (!new1) issue(1, u, fs - ubase + 1, 0);
        griddep_wait();
        if (new0) issue(0, u, fs - ubase, 0);
        if (new1) issue(1, u, fs - ubase + 1, 0);
    }

    float c1a = 0.0f, c2a = 0.0f, c1b = 0.0f, c2b = 0.0f;  // score constants of heads q, q + 4
    // per half hh: head 4*hh + ph's reference R, sum 2^(s-R), sum 2^(s-R)*vzp
    float Rr[2], Lr[2], Zr[2];
    float facc[2][GG::NF];  // per half: head 4*hh + ((lane>>2)&3)'s value sums in the frame of Rr
    bool fresh = true;
    while (!failed) {
        if (fresh) {
            c1a = qscal[(int64_t)u * 16 + q];
            c1b = qscal[(int64_t)u * 16 + 4 + q];
            c2a = qscal[(int64_t)u * 16 + 8 + q];
            c2b = qscal[(int64_t)u * 16 + 12 + q];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                Rr[hh] = -INFINITY;
                Lr[hh] = 0.0f;
                Zr[hh] = 0.0f;
#pragma unroll
                for (int k = 0; k < GG::NF; k++) facc[hh][k] = 0.0f;
            }
            fresh = false;
        }
        const int fn = fs + ns;
        int un = u, ubn = ubase, nsn = 0;
        if (fn < f1) {
            if (fn == ubase + ncu) {
                un = u + 1;
                ubn = ubase + ncu;
            }
            nsn = min(2, min(f1, ubn + ncu) - fn);
        }
        const int c0 = fs - ubase;
        const int n_w = min(total - c0 * CT, ns * CT);

        // ---------------- phase 1: scores of the eight heads ----------------
        float rma = -INFINITY, rmb = -INFINITY, vmax = 0.0f;  // max score of heads q, q + 4; max vscale
        {
            uint32_t bq[GG::QW];
            const uint4 *src = reinterpret_cast<const uint4 *>(qfrag + ((int64_t)u * 32 + lane) * GG::QW);
#pragma unroll
            for (int v = 0; v < GG::QW / 4; v++) {
                const uint4 x = src[v];
                bq[4 * v] = x.x;
                bq[4 * v + 1] = x.y;
                bq[4 * v + 2] = x.z;
                bq[4 * v + 3] = x.w;
            }
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                wait(cc, 0);
                if (failed) break;
                if (cc == 0 || cc < ns) {
                    const unsigned char *st = slots + cc * GG::SLOT;
                    const float *kms = reinterpret_cast<const float *>(st + CT * KB);
                    const float *vms = kms + 2 * CT;
#pragma unroll
                    for (int mt = 0; mt < CT / 16; mt++) {
                        uint32_t wv[2][GG::SEGW];
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {
                            const unsigned char *p = st + (16 * mt + r + 8 * hf) * KB + q * (KB / 4);
                            if constexpr (GG::SEGW == 2) {
                                const uint2 x = *reinterpret_cast<const uint2 *>(p);
                                wv[hf][0] = x.x;
                                wv[hf][1] = x.y;
                            } else {
#pragma unroll
                                for (int v = 0; v < GG::SEGW / 4; v++) {
                                    const uint4 x = reinterpret_cast<const uint4 *>(p)[v];
                                    wv[hf][4 * v] = x.x;
                                    wv[hf][4 * v + 1] = x.y;
                                    wv[hf][4 * v + 2] = x.z;
                                    wv[hf][4 * v + 3] = x.w;
                                }
                            }
                        }
                        int acc[3][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
                        for (int k = 0; k < GG::NCH; k++) {
                            uint32_t a0, a1, a2, a3;
                            if constexpr (BITS == 4) {
                                a0 = wv[0][k] & 0x0F0F0F0Fu;
                                a1 = wv[1][k] & 0x0F0F0F0Fu;
                                a2 = (wv[0][k] >> 4) & 0x0F0F0F0Fu;
                                a3 = (wv[1][k] >> 4) & 0x0F0F0F0Fu;
                            } else {
                                a0 = wv[0][2 * k];
                                a1 = wv[1][2 * k];
                                a2 = wv[0][2 * k + 1];
                                a3 = wv[1][2 * k + 1];
                            }
#pragma unroll
                            for (int t = 0; t < 3; t++)
                                mma_u8s8(acc[t], a0, a1, a2, a3, bq[k * 6 + t * 2], bq[k * 6 + t * 2 + 1]);
                        }
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {
                            const int row = 16 * mt + r + 8 * hf;
                            const int tl = cc * CT + row;
                            // head q: digits 0/1 in n-tile 0, digit 2 in n-tile 2 column 2q;
                            // head q + 4: n-tile 1, digit 2 in n-tile 2 column 2q + 1
                            const float da = fmaf((float)acc[0][2 * hf], 65536.0f,
                                                  (float)(acc[0][2 * hf + 1] * 256 + acc[2][2 * hf]));
                            const float db = fmaf((float)acc[1][2 * hf], 65536.0f,
                                                  (float)(acc[1][2 * hf + 1] * 256 + acc[2][2 * hf + 1]));
                            const float2 km = *reinterpret_cast<const float2 *>(kms + 2 * row);
                            const bool in = tl < n_w;
                            const float sa_ = in ? fmaf(km.x * c1a, da, km.y * c2a) : -INFINITY;
                            const float sb_ = in ? fmaf(km.x * c1b, db, km.y * c2b) : -INFINITY;
                            vmax = fmaxf(vmax, in ? vms[2 * row] : 0.0f);
                            scw[q * SCS + tl] = sa_;
                            scw[(q + 4) * SCS + tl] = sb_;
                            rma = fmaxf(rma, sa_);
                            rmb = fmaxf(rmb, sb_);
                        }
                    }
                }
                __syncwarp();
                if (cc < ns) issue(cc, u, c0 + cc, 1);
                else issue_empty(cc, 1);
            }
        }
        if (failed) break;
#pragma unroll
        for (int m = 4; m < 32; m <<= 1) {
            rma = fmaxf(rma, __shfl_xor_sync(0xffffffffu, rma, m));
            rmb = fmaxf(rmb, __shfl_xor_sync(0xffffffffu, rmb, m));
            vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, m));
        }
        // new references of heads ph and 4 + ph (lane ph holds the maxima of heads ph and ph + 4)
        float Rq[2];
        {
            const float lv = __log2f(vmax);
            const float mx[2] = {__shfl_sync(0xffffffffu, rma, ph), __shfl_sync(0xffffffffu, rmb, ph)};
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const float Rp = fmaxf(Rr[hh], mx[hh] + lv);
                Rq[hh] = Rp - kLog2UMax;
                const float fac = (Rr[hh] == -INFINITY) ? 0.0f : exp2f(Rr[hh] - Rp);
                Rr[hh] = Rp;
                Lr[hh] *= fac;
                Zr[hh] *= fac;
                const float fh = __shfl_sync(0xffffffffu, fac, 8 * ((lane >> 2) & 3));
#pragma unroll
                for (int k = 0; k < GG::NF; k++) facc[hh][k] *= fh;
            }
        }

        // ---------------- phase 2: values, one half of the heads at a time ----------------
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            int pacc[GG::NTV][4];
            const float *sch = scw + (4 * hh + ph) * SCS;
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                if (hh == 0) {
                    wait(cc, 1);
                    if (failed) break;
                }
                if (cc == 0 || cc < ns) {
                    const unsigned char *st = slots + cc * GG::SLOT;
                    const float *vms = reinterpret_cast<const float *>(st + CT * KB);
#pragma unroll
                    for (int sp = 0; sp < CT / 32; sp++) {
                        const int tc = 32 * sp + 4 * tq;
                        const int tb = cc * CT + tc;
                        uint32_t U[4];
                        {
                            const float4 s4 = *reinterpret_cast<const float4 *>(sch + tb);
                            const float4 m01 = *reinterpret_cast<const float4 *>(vms + 2 * tc);
                            const float4 m23 = *reinterpret_cast<const float4 *>(vms + 2 * tc + 4);
                            const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
                            const float vs[4] = {m01.x, m01.z, m23.x, m23.z}, vz[4] = {m01.y, m01.w, m23.y, m23.w};
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const float ee = ex2_approx(sv[e] - Rq[hh]);
                                Lr[hh] += ee;
                                Zr[hh] = fmaf(ee, vz[e], Zr[hh]);
                                U[e] = __float2uint_rn(fminf(ee * vs[e], kUMax));
                            }
                        }
                        const uint32_t lo0 = __byte_perm(U[0], U[1], 0x0062), hi0 = __byte_perm(U[2], U[3], 0x0062);
                        const uint32_t lo1 = __byte_perm(U[0], U[1], 0x0051), hi1 = __byte_perm(U[2], U[3], 0x0051);
                        const uint32_t lo2 = __byte_perm(U[0], U[1], 0x0040), hi2 = __byte_perm(U[2], U[3], 0x0040);
                        tile[(0 + ph) * kTileW + tq] = __byte_perm(lo0, hi0, 0x5410);
                        tile[(4 + ph) * kTileW + (tq ^ 4)] = __byte_perm(lo1, hi1, 0x5410);
                        tile[(8 + ph) * kTileW + tq] = __byte_perm(lo2, hi2, 0x5410);
                        __syncwarp();
                        const int sw = r & 4;
                        const uint32_t pa0 = tile[r * kTileW + (q ^ sw)], pa2 = tile[r * kTileW + ((4 + q) ^ sw)];
                        const uint32_t pa1 = r < 4 ? tile[(r + 8) * kTileW + q] : 0u;
                        const uint32_t pa3 = r < 4 ? tile[(r + 8) * kTileW + 4 + q] : 0u;
                        __syncwarp();
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
                                    if (cc == 0 && sp == 0) {
                                        mma_u8u8_z(pacc[2 * i], pa0, pa1, pa2, pa3, y0[jj], y1[jj]);
                                        mma_u8u8_z(pacc[2 * i + 1], pa0, pa1, pa2, pa3, y0[jj] & 0xF0F0F0F0u,
                                                   y1[jj] & 0xF0F0F0F0u);
                                    } else {
                                        mma_u8u8(pacc[2 * i], pa0, pa1, pa2, pa3, y0[jj], y1[jj]);
                                        mma_u8u8(pacc[2 * i + 1], pa0, pa1, pa2, pa3, y0[jj] & 0xF0F0F0F0u,
                                                 y1[jj] & 0xF0F0F0F0u);
                                    }
                                } else {
                                    if (cc == 0 && sp == 0) mma_u8u8_z(pacc[i], pa0, pa1, pa2, pa3, y0[jj], y1[jj]);
                                    else mma_u8u8(pacc[i], pa0, pa1, pa2, pa3, y0[jj], y1[jj]);
                                }
                            }
                        }
                    }
                }
                if (hh == 1) {
                    // both halves have read chunk cc: the slot takes the next K chunk
                    __syncwarp();
                    if (nsn > 0) {
                        if (cc < nsn) issue(cc, un, fn - ubn + cc, 0);
                        else issue_empty(cc, 0);
                    }
                }
            }
            if (failed) break;
            // fold this half's digit sums into its float sums (same layout as the four-head kernel)
            {
                const float w_a = lo ? 65536.0f : 256.0f;
                const float ntw = (BITS == 4 && !lo) ? 0.0625f : 1.0f;
#pragma unroll
                for (int np = 0; np < GG::NTV / 2; np++) {
                    if constexpr (BITS == 4) {
#pragma unroll
                        for (int x = 0; x < 4; x++) pacc[2 * np][x] -= pacc[2 * np + 1][x];
                    }
#pragma unroll
                    for (int cc = 0; cc < 2; cc++) {
                        // rows 12-15 of the P tile are zero, so c2/c3 of lanes >= 16 add nothing
                        const float fe = fmaf((float)pacc[2 * np][cc], w_a, (float)pacc[2 * np][2 + cc]);
                        const float fo = fmaf((float)pacc[2 * np + 1][cc], w_a, (float)pacc[2 * np + 1][2 + cc]);
                        const float recv = __shfl_xor_sync(0xffffffffu, lo ? fo : fe, 16);
                        facc[hh][2 * np + cc] = fmaf((lo ? fe : fo) + recv, ntw, facc[hh][2 * np + cc]);
                    }
                }
            }
        }
        if (failed) break;
        if (nsn == 0 || un != u) {
            // ---------------- the unit's partial record (eight heads) ----------------
            float *rec = a.workspace + (int64_t)(w + u) * GG::REC;
            const int hr = (lane >> 2) & 3;
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                float L = Lr[hh], Z = Zr[hh];
                L += __shfl_xor_sync(0xffffffffu, L, 1);
                L += __shfl_xor_sync(0xffffffffu, L, 2);
                L += __shfl_xor_sync(0xffffffffu, L, 4);
                Z += __shfl_xor_sync(0xffffffffu, Z, 1);
                Z += __shfl_xor_sync(0xffffffffu, Z, 2);
                Z += __shfl_xor_sync(0xffffffffu, Z, 4);
#pragma unroll
                for (int k = 0; k < GG::NF; k++)
                    rec[(4 * hh + hr) * D + v_dim<BITS, D>(2 * (k >> 1) + (lo ? 0 : 1), 2 * q + (k & 1))] =
                        facc[hh][k];
                if (tq == 0) {
                    rec[RG::R + 4 * hh + ph] = Rr[hh];
                    rec[RG::L + 4 * hh + ph] = L;
                    rec[RG::Z + 4 * hh + ph] = Z;
                }
            }
            fresh = true;
        }
        if (nsn == 0) break;
        fs = fn;
        u = un;
        ubase = ubn;
        ns = nsn;
    }

    if (failed && lane == 0) {
        // a wait gave up: let this warp's copies still in flight land (bounded)
        for (int b = 0; b < 4; b++)
            if (pend & (1u << b)) mbar_wait_bounded(mybar + (b >> 1), (uint32_t)(b & 1));
    }
}

struct DecodeGrid8 {
    int ncu, F, W, ctas;
};

template <int BITS, int D>
DecodeGrid8 decode8_grid(const AttendArgs &a) {
    using GG = G8Geo<BITS, D>;
    DecodeGrid8 g;
    const int64_t total = a.pos0 + 1;
    g.ncu = (int)((total + GG::CT - 1) / GG::CT);
    g.F = a.batch * a.heads * g.ncu;
    g.W = min(a.sm_count * kNW8, g.F);
    g.ctas = (g.W + kNW8 - 1) / kNW8;
    return g;
}

template <typename T, int BITS, int D>
int launch8_shape(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    using GG = G8Geo<BITS, D>;
    uint32_t *qfrag = a.qprep;
    float *qscal = reinterpret_cast<float *>(a.qprep + (size_t)a.batch * a.heads * 32 * kQWMax8);
    const int do_append = ap != nullptr;
    AppendArgs apv{};
    if (ap) apv = *ap;
    const int prep_warps = (do_append ? 2 : 0) + 8;
    // prep, decode and merge are programmatic dependents of the kernel before them
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.heads, a.batch);
    cfg.blockDim = dim3(32 * prep_warps);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    int rc = check_cuda(cudaLaunchKernelEx(&cfg, decode_prep8_kernel<T, BITS, D>, a, apv, do_append, qfrag, qscal),
                        "gqa decode8 prep launch");
    count_launch();
    if (rc != SA_OK) return rc;

    auto kern = decode8_stream_kernel<T, BITS, D>;
    const size_t smem = GG::SMEM;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "gqa decode8 smem attribute");
        if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
    }
    const DecodeGrid8 dg = decode8_grid<BITS, D>(a);
    cfg.gridDim = dim3((unsigned)dg.ctas);
    cfg.blockDim = dim3(kNW8 * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    rc = check_cuda(cudaLaunchKernelEx(&cfg, kern, a, dg.ncu, dg.F, dg.W, (const uint32_t *)qfrag,
                                       (const float *)qscal),
                    "gqa decode8 launch");
    count_launch();
    if (rc != SA_OK) return rc;
    cfg.gridDim = dim3((unsigned)(a.batch * a.heads));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    rc = check_cuda(cudaLaunchKernelEx(&cfg, decode_merge_kernel<T, D, 8>, a, dg.ncu, dg.F, dg.W),
                    "gqa decode8 merge launch");
    count_launch();
    return rc;
}

template <typename T>
int launch8_dtype(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch8_shape<T, 4, 128>(a, ap, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch8_shape<T, 8, 128>(a, ap, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch8_shape<T, 4, 64>(a, ap, stream);
    return launch8_shape<T, 8, 64>(a, ap, stream);
}

}  // namespace

// Records of the eight-head decode: one per warp of the grid plus one per unit.
size_t decode8_workspace_floats(int sm_count, int64_t units, int head_dim) {
    return (size_t)((int64_t)sm_count * kNW8 + units) * (size_t)(8 * head_dim + 32);
}

// q-digit words (and score constants) per unit of the eight-head prep.
size_t decode8_qprep_words() { return 32 * kQWMax8 + 16; }

int launch_gqa_decode8(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch8_dtype<float>(a, ap, stream);
        case SA_DTYPE_FLOAT16: return launch8_dtype<__half>(a, ap, stream);
        default: return launch8_dtype<__nv_bfloat16>(a, ap, stream);
    }
}

}  // namespace sa

// Tensor-core decode attention over the PolarQuant cache: one query token per
// sequence, 4/8-bit codes, head_dim 64/128, up to 4 query heads per KV head
// (5..8 heads: gqa_decode_g8.cu).
//
// Three launches per step:
//
//  decode_prep_kernel, one CTA per (KV head, batch row):
//    - quantize-on-append of the new token's K and V (same bit-exact encoder
//      as sa_kv_append), when the operator appends;
//    - RoPE + rotation of the G query heads, q' = H.S.q/sqrt(n), written as
//      three signed 8-bit digits of a 24-bit fixed-point number per head:
//      q' ~= sigma * (d0*2^16 + d1*2^8 + d2), |d| <= 127, stored already
//      arranged as each lane's mma B-fragment words.
//
//  decode_stream_kernel, two CTAs of 8 independent warps per SM.  Each warp
//  owns an equal share of all (row, KV head, chunk) work laid end to end and
//  streams it through two shared-memory slots of its own with 1-D bulk copies
//  (cp.async.bulk + mbarrier, no multicast), in sub-segments of 128 tokens:
//    phase 1 (K): K codes are unpacked to u8 in registers and contracted with
//      the q' digits by mma.m16n8k32 u8 x s8 -> exact int32 dots q'.c; the
//      score s = scale_t*sigma*(q'.c) + zp_t*sum(q') (log2 units) goes to
//      shared memory.
//    phase 2 (V): with a reference R >= max(s) + log2(max vscale) (running
//      over the sub-segments), every token gets e = 2^(s - R) and
//      u = e * vscale in (0, 1] as a 24-bit fixed-point number (three
//      unsigned digits); sum_t u_t * c_t is an exact int32 mma.m16n8k32
//      u8 x u8 over the 16-token-block V layout, L = sum e and
//      Z = sum e * vzp are float sums.  After the sub-segment the integer
//      sums are folded into float sums in the frame of R.
//    A warp leaves one partial record per unit its range touches.
//
//
//  decode_merge_kernel: per unit, merges the records, normalises, applies the
//  inverse rotation and stores.
//
//  Every mbarrier wait is bounded; a wait that gives up sets the cache's
//  device status, the warp stops issuing and writing and drains its copies.
#include "sa_append.cuh"
#include "sa_async.cuh"
#include "sa_decode_common.cuh"

namespace sa {

namespace {

using namespace dec;

constexpr int kNW = 8;            // warps per decode CTA
constexpr int kTileW = 8;         // u32 words per row of a warp's P-digit tile (12 rows)
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
    __shared__ uint8_t s_codes[2][256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.x, b = blockIdx.y;
    const int G = a.group;
    const int q0w = do_append ? 2 : 0;
    const float *sg = a.signs + (int64_t)h * D;
    // the decode kernel may start now: it waits for this grid before it
    // reads the q digits or the appended token
    griddep_launch_dependents();
    griddep_wait();  // launched as a dependent of the kernel before it: q and the cache are ready
    if (do_append && warp < 2) {
        encode_append_vector<T, EPL>(ap, b, 0, h, warp, lane, s_codes[warp]);
        return;
    }
    const int g = warp - q0w;
    if (g < 0 || g >= 4) return;
    const int64_t bh = (int64_t)b * a.heads + h;
    uint32_t *frag = qfrag + bh * 32 * GG::QW;
    // Fragment lane fl = (r, q) holds column r of the QK B operand: head
    // r >> 1; n-tile 0 column 2j -> (head j, digit 0), 2j+1 -> (head j,
    // digit 1); n-tile 1 column 2j -> (head j, digit 2), 2j+1 -> zero.  Warp g
    // writes the 8 fragment lanes of head g, each as four lanes of 4 words.
    const int fl = 8 * g + (lane >> 2);  // fragment lane
    const int fr = fl >> 2, fq = fl & 3;
    uint32_t *dst = frag + fl * GG::QW + (lane & 3) * (GG::QW / 4);
    if (g >= G) {  // no such head: zero columns
#pragma unroll
        for (int i = 0; i < GG::QW / 4; i++) dst[i] = 0u;
        if (lane == 0) {
            qscal[bh * 8 + g] = 0.0f;
            qscal[bh * 8 + 4 + g] = 0.0f;
        }
        return;
    }
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
    float sum = 0.0f, mabs = 0.0f;
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
    const float sigma = mabs > 0.0f ? mabs / kQMax : 1.0f;
    const float inv_sigma = 1.0f / sigma;
    if (lane == 0) {
        const float sl2 = a.scale * kLog2eF;
        qscal[bh * 8 + g] = sigma * sl2;
        qscal[bh * 8 + 4 + g] = sum * sl2;
    }
    __syncwarp();  // s_q[g] complete
    // this lane's words: index i of fragment lane fl is c*4 + t*2 + half,
    // for i in [(lane & 3) * QW/4, (lane & 3 + 1) * QW/4)
#pragma unroll
    for (int ii = 0; ii < GG::QW / 4; ii++) {
        const int i = (lane & 3) * (GG::QW / 4) + ii;
        const int c = i >> 2, t = (i >> 1) & 1, half = i & 1;
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int k = 16 * half + 4 * fq + e;
            int qi = __float2int_rn(s_q[g][k_dim<BITS, D>(c, fq, k)] * inv_sigma);
            qi = min(max(qi, -(int)kQMax), (int)kQMax);  // keep the top digit within int8
            const int d2 = (int)(int8_t)(qi & 0xff);
            const int rest = (qi - d2) >> 8;
            const int d1 = (int)(int8_t)(rest & 0xff);
            const int d0 = (rest - d1) >> 8;
            const int dg = t == 0 ? ((fr & 1) ? d1 : d0) : ((fr & 1) ? 0 : d2);
            word |= ((uint32_t)(dg & 0xff)) << (8 * e);
        }
        dst[ii] = word;
    }
}


// ---- decode: stream-K warp ranges ----------------------------------------------
// The context of every (row, KV head) unit is cut into chunks of CT tokens and
// the chunks of all units are laid end to end (F chunks).  Warp w of the grid
// (W warps) owns the contiguous range [w*F/W, (w+1)*F/W): every warp streams
// the same number of chunks whatever the batch, heads and context length, and
// no warp ever waits for another.  A range may start or end inside a unit and
// may cover several units; for each unit it touches the warp leaves one
// partial record (running max R, sums L and Z, un-normalised value sums) at
// record index w + u, and decode_merge_kernel merges each unit's records.
//
// Inside a unit the warp walks sub-segments of two chunks through its own two
// shared-memory slots: slot s holds K chunk s of a sub-segment, then its V
// chunk s, then K chunk s of the next sub-segment, and so on, so a slot's
// mbarrier always completes an even phase for a K chunk and an odd phase for
// a V chunk.  A sub-segment with a single chunk gives slot 1 empty phases (an
// arrive without data).  Phase 1 computes the scores from the K chunks
// (kept in shared memory), phase 2 streams the V chunks with the running
// reference R as the fixed-point frame; the integer accumulators are folded
// into float sums after every sub-segment.
template <int BITS, int D>
struct WGeo {
    static constexpr int KB = D * BITS / 8;             // code bytes per token
    static constexpr int CT = (KB > 64) ? 32 : 64;       // tokens per chunk
    static constexpr int TPW = 2 * CT;                   // tokens per sub-segment
    static constexpr int SCS = TPW + 8;                  // floats per head row of a warp's score buffer (bank offset)
    static constexpr int SLOT = CT * (KB + 16);          // K chunk: codes + K meta + V meta (a V chunk is smaller)
    static constexpr int SEGW = KB / 16;                 // K words per quad per row
    static constexpr int NCH = D / 32;                   // QK k-chunks
    static constexpr int NTV = D / 8;                    // PV n-tiles
    static constexpr int NF = NTV;                       // float value sums per lane
    static constexpr int VV = ((BITS == 4) ? NTV / 2 : NTV) / 4;  // 16-byte V loads per 16-token block
    static constexpr int QW = NCH * 4;                   // q-digit words per lane
    static constexpr int SCW = 4 * SCS;                  // floats of a warp's score buffer
    static constexpr int REC = RecGeo<D, 4>::REC;        // floats per partial record: [4][D] values, R/L/Z x 4
    static constexpr int SMEM = kNW * 2 * SLOT + kNW * SCW * 4 + kNW * 12 * kTileW * 4 + 256;
};

template <typename T, int BITS, int D>
__global__ void __launch_bounds__(kNW * 32, 2)
    decode_stream_kernel(AttendArgs a, int ncu, int F, int W, const uint32_t *__restrict__ qfrag,
                         const float *__restrict__ qscal) {
    using GG = WGeo<BITS, D>;
    constexpr int KB = GG::KB, CT = GG::CT, SCS = GG::SCS;

    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned char *slots = smem + warp * 2 * GG::SLOT;                                   // this warp's 2 slots
    float *scw = reinterpret_cast<float *>(smem + kNW * 2 * GG::SLOT) + warp * GG::SCW;  // scores of the sub-segment
    uint32_t *tile = reinterpret_cast<uint32_t *>(smem + kNW * 2 * GG::SLOT + kNW * GG::SCW * 4) +
                     warp * 12 * kTileW;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kNW * 2 * GG::SLOT + kNW * GG::SCW * 4 +
                                                  kNW * 12 * kTileW * 4);  // [kNW][2]
    uint64_t *mybar = bars + 2 * warp;

    const int G = a.group;
    const int r = lane >> 2, q = lane & 3;
    const int ph = lane >> 3, tq = lane & 7;  // P-digit role: head ph, token quad tq of a 32-token step
    const bool my_head = q < G;
    const bool lo = lane < 16;                // value sums: lanes < 16 keep even n-tiles, the rest odd ones

    if (tid == 0) {
        for (int i = 0; i < 2 * kNW; i++) mbar_init(bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();  // the only block-wide barrier: warps are independent from here on
    // The merge kernel may launch now (it waits for this grid).
    griddep_launch_dependents();
    const int w = blockIdx.x * kNW + warp;
    if (w >= W) return;
    const int f0 = (int)((int64_t)w * F / W), f1 = (int)((int64_t)(w + 1) * F / W);
    const int total = (int)a.pos0 + 1;

    // Copies of a chunk, one per lane: K chunk = codes (lane 0), K meta
    // (lane 1), V meta (lane 2); V chunk = codes (lane 0), V meta (lane 1).
    // `pend` has bit 2*slot + kind (0 = K, 1 = V) set while a phase is issued
    // and not yet waited for.
    unsigned pend = 0;
    bool failed = false;
    // Whole chunks are copied even past the context (the capacity is a
    // multiple of 64, the cache is zero-initialised): the extra tokens are
    // finite and masked by their -inf scores.
    auto issue = [&](int s, int uu, int c, int kind) {
        constexpr uint32_t kCodeBytes = CT * KB, kMetaBytes = CT * 8;
        const int64_t row = (int64_t)uu * a.capacity + c * CT;  // first token of the chunk
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
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // after the warp's reads of the slot
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
        // The first K chunks; one that holds the newest token (appended by
        // the prep kernel) is fetched after waiting for that kernel, the
        // older ones before.
        const bool new0 = fs - ubase == ncu - 1, new1 = ns > 1 && fs - ubase + 1 == ncu - 1;
        if (!new0) issue(0, u, fs - ubase, 0);
        if (ns < 2) issue_empty(1, 0);
        else if (!new1) issue(1, u, fs - ubase + 1, 0);
        griddep_wait();
        if (new0) issue(0, u, fs - ubase, 0);
        if (new1) issue(1, u, fs - ubase + 1, 0);
    }

    float c1 = 0.0f, c2 = 0.0f;
    float Rr = -INFINITY, Lr = 0.0f, Zr = 0.0f;  // head ph: reference R, sum 2^(s-R), sum 2^(s-R)*vzp
    float facc[GG::NF];                           // head (lane>>2)&3: value sums in the frame of Rr
    bool fresh = true;
    while (!failed) {
        if (fresh) {  // first sub-segment of a unit
            c1 = qscal[(int64_t)u * 8 + q];
            c2 = qscal[(int64_t)u * 8 + 4 + q];
            Rr = -INFINITY;
            Lr = 0.0f;
            Zr = 0.0f;
#pragma unroll
            for (int k = 0; k < GG::NF; k++) facc[k] = 0.0f;
            fresh = false;
        }
        // the next sub-segment (nsn = 0: none)
        const int fn = fs + ns;
        int un = u, ubn = ubase, nsn = 0;
        if (fn < f1) {
            if (fn == ubase + ncu) {
                un = u + 1;
                ubn = ubase + ncu;
            }
            nsn = min(2, min(f1, ubn + ncu) - fn);
        }
        const int c0 = fs - ubase;                           // first chunk within the unit
        const int n_w = min(total - c0 * CT, ns * CT);       // tokens in the sub-segment

        // ---------------- phase 1: scores ----------------
        float rmax = -INFINITY, vmax = 0.0f;  // max score of head q, max vscale
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
                if (cc == 0 || cc < ns) {  // a sub-segment has at least one chunk
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
                        int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
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
                            mma_u8s8(acc[0], a0, a1, a2, a3, bq[k * 4 + 0], bq[k * 4 + 1]);
                            mma_u8s8(acc[1], a0, a1, a2, a3, bq[k * 4 + 2], bq[k * 4 + 3]);
                        }
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {
                            const int row = 16 * mt + r + 8 * hf;  // token within the chunk
                            const int tl = cc * CT + row;          // token within the sub-segment
                            const float dot = fmaf((float)acc[0][2 * hf], 65536.0f,
                                                   (float)(acc[0][2 * hf + 1] * 256 + acc[1][2 * hf]));
                            const float2 km = *reinterpret_cast<const float2 *>(kms + 2 * row);
                            const bool in = tl < n_w;
                            const float s = in ? fmaf(km.x * c1, dot, km.y * c2) : -INFINITY;
                            vmax = fmaxf(vmax, in ? vms[2 * row] : 0.0f);
                            if (my_head) {
                                scw[q * SCS + tl] = s;
                                rmax = fmaxf(rmax, s);
                            }
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
            rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, m));
            vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, m));
        }
        // new reference of head ph (lane ph holds head ph's max; u = 2^(s - R) * vscale <= 1)
        // and the factor that moves earlier sums to it
        const float Rp = fmaxf(Rr, __shfl_sync(0xffffffffu, rmax, ph) + __log2f(vmax));
        const float Rq = Rp - kLog2UMax;  // sums and digits are kept in units of 1 / kUMax
        const float fac = (Rr == -INFINITY) ? 0.0f : exp2f(Rr - Rp);
        Rr = Rp;
        Lr *= fac;
        Zr *= fac;
        {
            const float fh = __shfl_sync(0xffffffffu, fac, 8 * ((lane >> 2) & 3));
#pragma unroll
            for (int k = 0; k < GG::NF; k++) facc[k] *= fh;
        }

        // ---------------- phase 2: values ----------------
        int pacc[GG::NTV][4];  // started by the first 32-token step (chunk 0 always holds tokens)
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            wait(cc, 1);
            if (failed) break;
            if (cc == 0 || cc < ns) {  // a sub-segment has at least one chunk
                const unsigned char *st = slots + cc * GG::SLOT;
                const float *vms = reinterpret_cast<const float *>(st + CT * KB);
#pragma unroll
                for (int sp = 0; sp < CT / 32; sp++) {
                    const int tc = 32 * sp + 4 * tq;  // this lane's first token within the chunk
                    const int tb = cc * CT + tc;      // ... within the sub-segment
                    // Tokens past the context have score -inf (e = 0).  Rows of heads >= G
                    // hold no scores; their sums are never read.
                    uint32_t U[4];
                    {
                        const float4 s4 = *reinterpret_cast<const float4 *>(scw + ph * SCS + tb);
                        const float4 m01 = *reinterpret_cast<const float4 *>(vms + 2 * tc);
                        const float4 m23 = *reinterpret_cast<const float4 *>(vms + 2 * tc + 4);
                        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
                        const float vs[4] = {m01.x, m01.z, m23.x, m23.z}, vz[4] = {m01.y, m01.w, m23.y, m23.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float ee = ex2_approx(sv[e] - Rq);  // kUMax * 2^(s - R)
                            Lr += ee;
                            Zr = fmaf(ee, vz[e], Zr);
                            U[e] = __float2uint_rn(fminf(ee * vs[e], kUMax));
                        }
                    }
                    // digit j of the 4 tokens -> one A-fragment word (row 4j + head, token quad tq)
                    const uint32_t lo0 = __byte_perm(U[0], U[1], 0x0062), hi0 = __byte_perm(U[2], U[3], 0x0062);
                    const uint32_t lo1 = __byte_perm(U[0], U[1], 0x0051), hi1 = __byte_perm(U[2], U[3], 0x0051);
                    const uint32_t lo2 = __byte_perm(U[0], U[1], 0x0040), hi2 = __byte_perm(U[2], U[3], 0x0040);
                    // row R keeps column c at word R*8 + (c ^ (R & 4)): the stores of
                    // rows x..x+3 and the fragment loads hit 32 distinct banks
                    tile[(0 + ph) * kTileW + tq] = __byte_perm(lo0, hi0, 0x5410);
                    tile[(4 + ph) * kTileW + (tq ^ 4)] = __byte_perm(lo1, hi1, 0x5410);
                    tile[(8 + ph) * kTileW + tq] = __byte_perm(lo2, hi2, 0x5410);
                    __syncwarp();
                    const int sw = r & 4;
                    const uint32_t pa0 = tile[r * kTileW + (q ^ sw)], pa2 = tile[r * kTileW + ((4 + q) ^ sw)];
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
                                // n-tile 2i sums the raw bytes (lo + 16 hi), n-tile 2i+1 the high
                                // nibbles in place (16 hi); the fold separates them
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
            __syncwarp();
            if (nsn > 0) {
                if (cc < nsn) issue(cc, un, fn - ubn + cc, 0);
                else issue_empty(cc, 0);
            }
        }
        if (failed) break;

        // ---------------- fold the digit sums into the float sums ----------------
        // Accumulator rows: r < 4 -> (digit 0, head r) in c0/c1 and (digit 2,
        // head r) in c2/c3; r >= 4 -> (digit 1, head r - 4) in c0/c1.  value =
        // (d0*2^16 + d1*2^8 + d2) / (2^24 - 1).  Lanes L and L^16 hold the
        // pieces of the same (head, column): each keeps one n-tile of every
        // pair and sends the other's piece across.
        {
            const float w_a = lo ? 65536.0f : 256.0f;  // digit weights (sums are in units of 1 / kUMax)
            const float ntw = (BITS == 4 && !lo) ? 0.0625f : 1.0f;  // high-nibble tiles hold 16 * code
#pragma unroll
            for (int np = 0; np < GG::NTV / 2; np++) {
                if constexpr (BITS == 4) {
#pragma unroll
                    for (int x = 0; x < 4; x++) pacc[2 * np][x] -= pacc[2 * np + 1][x];  // low nibbles
                }
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    // rows 12-15 of the P tile are zero, so c2/c3 of lanes >= 16 add nothing
                    const float fe = fmaf((float)pacc[2 * np][cc], w_a, (float)pacc[2 * np][2 + cc]);
                    const float fo = fmaf((float)pacc[2 * np + 1][cc], w_a, (float)pacc[2 * np + 1][2 + cc]);
                    const float recv = __shfl_xor_sync(0xffffffffu, lo ? fo : fe, 16);
                    facc[2 * np + cc] = fmaf((lo ? fe : fo) + recv, ntw, facc[2 * np + cc]);
                }
            }
        }
        if (nsn == 0 || un != u) {
            // ---------------- the unit's partial record ----------------
            Lr += __shfl_xor_sync(0xffffffffu, Lr, 1);
            Lr += __shfl_xor_sync(0xffffffffu, Lr, 2);
            Lr += __shfl_xor_sync(0xffffffffu, Lr, 4);
            Zr += __shfl_xor_sync(0xffffffffu, Zr, 1);
            Zr += __shfl_xor_sync(0xffffffffu, Zr, 2);
            Zr += __shfl_xor_sync(0xffffffffu, Zr, 4);
            if (!failed) {
                // record: value sums [head][dim], then R, L, Z of the four heads
                float *rec = a.workspace + (int64_t)(w + u) * GG::REC;
                const int hr = (lane >> 2) & 3;
                if (hr < G) {
#pragma unroll
                    for (int k = 0; k < GG::NF; k++)
                        rec[hr * D + v_dim<BITS, D>(2 * (k >> 1) + (lo ? 0 : 1), 2 * q + (k & 1))] = facc[k];
                }
                if (tq == 0) {
                    rec[4 * D + ph] = ph < G ? Rr : -INFINITY;
                    rec[4 * D + 4 + ph] = Lr;
                    rec[4 * D + 8 + ph] = Zr;
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
        // a wait gave up and nothing was issued since: let this warp's copies still in flight land (bounded)
        for (int b = 0; b < 4; b++)
            if (pend & (1u << b)) mbar_wait_bounded(mybar + (b >> 1), (uint32_t)(b & 1));
    }
}

// Grid of the decode kernel: two CTAs per SM, no more warps than chunks.
struct DecodeGrid {
    int ncu, F, W, ctas;
};

template <int BITS, int D>
DecodeGrid decode_grid(const AttendArgs &a) {
    using GG = WGeo<BITS, D>;
    DecodeGrid g;
    const int64_t total = a.pos0 + 1;
    g.ncu = (int)((total + GG::CT - 1) / GG::CT);
    g.F = a.batch * a.heads * g.ncu;  // fits int: decode_fast_eligible bounds it
    g.W = min(2 * a.sm_count * kNW, g.F);
    g.ctas = (g.W + kNW - 1) / kNW;
    return g;
}

template <typename T, int BITS, int D>
int launch_shape(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    uint32_t *qfrag = a.qprep;
    float *qscal = reinterpret_cast<float *>(a.qprep + (size_t)a.batch * a.heads * 32 * 16);
    const int do_append = ap != nullptr;
    AppendArgs apv{};
    if (ap) apv = *ap;
    const int prep_warps = (do_append ? 2 : 0) + 4;  // the append warps, then one warp per fragment head
    // All three launches are programmatic dependents of the kernel before them (prep of whatever
    // kernel precedes the call), so each launch overlaps the tail of the one before; each kernel
    // waits for its predecessor's grid before it reads what that grid wrote.
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
    int rc = check_cuda(cudaLaunchKernelEx(&cfg, decode_prep_kernel<T, BITS, D>, a, apv, do_append, qfrag, qscal),
                        "gqa decode prep launch");
    count_launch();
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
    const DecodeGrid dg = decode_grid<BITS, D>(a);
    cfg.gridDim = dim3((unsigned)dg.ctas);
    cfg.blockDim = dim3(kNW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    rc = check_cuda(cudaLaunchKernelEx(&cfg, kern, a, dg.ncu, dg.F, dg.W, (const uint32_t *)qfrag, (const float *)qscal),
                    "gqa decode launch");
    count_launch();
    if (rc != SA_OK) return rc;
    cfg.gridDim = dim3((unsigned)(a.batch * a.heads));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    rc = check_cuda(cudaLaunchKernelEx(&cfg, decode_merge_kernel<T, D, 4>, a, dg.ncu, dg.F, dg.W),
                    "gqa decode merge launch");
    count_launch();
    return rc;
}

template <typename T>
int launch_dtype(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch_shape<T, 4, 128>(a, ap, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch_shape<T, 8, 128>(a, ap, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch_shape<T, 4, 64>(a, ap, stream);
    return launch_shape<T, 8, 64>(a, ap, stream);
}

}  // namespace

// Floats of partial records the decode needs: one per warp of the grid plus
// one per unit (a warp's range touches one unit more than it crosses).
size_t decode_workspace_floats(int sm_count, int64_t units, int head_dim, int group) {
    if (group > 4) return decode8_workspace_floats(sm_count, units, head_dim);
    return (size_t)((int64_t)2 * sm_count * kNW + units) * (size_t)(4 * head_dim + 16);
}

// 32-bit words of the prep area per (row, KV head): the q-digit fragments of
// 32 lanes, then the score constants.
size_t decode_qprep_words(int group) { return group > 4 ? decode8_qprep_words() : 32 * 16 + 8; }

// Whether the tensor-core decode handles this call.
bool decode_fast_eligible(const AttendArgs &a) {
    if (a.seq_len != 1 || a.group < 1 || a.group > 8) return false;
    if ((a.bits != 4 && a.bits != 8) || (a.head_dim != 64 && a.head_dim != 128)) return false;
    if (a.capacity % 64 != 0 || a.qprep == nullptr || a.dev_status == nullptr) return false;
    const int64_t units = (int64_t)a.batch * a.heads;
    if (units * ((a.pos0 + 32) / 32) >= ((int64_t)1 << 31)) return false;  // flat chunk indices are int
    return decode_workspace_floats(a.sm_count, units, a.head_dim, a.group) <= a.workspace_floats;
}

// Prep (+ append when `ap` is given), decode and merge of one query token per row.
int launch_gqa_decode_fast(const AttendArgs &a, const AppendArgs *ap, cudaStream_t stream) {
    if (a.group > 4) return launch_gqa_decode8(a, ap, stream);
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_dtype<float>(a, ap, stream);
        case SA_DTYPE_FLOAT16: return launch_dtype<__half>(a, ap, stream);
        default: return launch_dtype<__nv_bfloat16>(a, ap, stream);
    }
}

}  // namespace sa

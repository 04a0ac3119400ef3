// Tensor-core decode attention over the PolarQuant cache (one query token,
// 4/8-bit codes, head_dim 64/128, up to 4 query heads per KV head).
//
// One CTA per (split of the context, KV head, batch row); each warp owns a
// contiguous token range of the split and runs two phases over it:
//
//  1. scores.  q' = H.S.q/sqrt(n) is written as three signed 8-bit digits
//     (24-bit fixed point per head, q' ~= sigma * (d0*2^16 + d1*2^8 + d2)),
//     so q'.c for 16 tokens x 4 heads is one exact int32 contraction:
//     mma.m16n8k32 u8 (K codes, unpacked in registers) x s8 (digits).  The
//     score of token t, head h is scale_t*(q'.c) + zp_t*sum(q'), in log2
//     units, kept in shared memory.
//  2. values.  With the warp's max R over max(s, s + log2 vscale), each token
//     gets u = 2^(s + log2 vscale - R) in (0, 1] as a 24-bit fixed-point
//     number (three unsigned 8-bit digits) and the PV product
//     sum_t u_t * c_t is again an exact int32 mma.m16n8k32 u8 x u8, with the
//     V codes of 4 consecutive tokens coming from one 32-bit word of the
//     4-token interleaved layout.  No online rescaling is needed inside a
//     warp because R is known before phase 2 starts.
//
// The warps of a CTA merge their (R, L, Z, acc) in shared memory; splits are
// merged by attend_combine_kernel (or the CTA writes the output directly when
// there is one split), which also applies the inverse rotation.
#include "sa_common.cuh"
#include "sa_internal.h"

namespace sa {

// defined in gqa_attend.cu
void choose_splits(const AttendArgs &a, int64_t total, int *n_splits, int *tps);
int launch_gqa_combine(const AttendArgs &a, int n_splits, cudaStream_t stream);

namespace {

constexpr int kNW = 8;           // warps per CTA
constexpr int kTPW = 256;        // max tokens per warp (phase-1 score buffer)
constexpr int kPRow = 48;        // bytes per row of the P-digit tile (bank-conflict free)
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kQMax = 8355711.0f;      // 127*65536 + 127*256 + 127
constexpr float kUMax = 16777215.0f;     // 2^24 - 1

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

__device__ __forceinline__ uint4 ldg_nc(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// The SEGW 32-bit words of one quad's share of a K row (8, 16 or 32 bytes).
template <int SEGW>
__device__ __forceinline__ void load_seg(const uint8_t *p, uint32_t (&w)[SEGW]) {
    if (SEGW == 2) {
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
    } else {
#pragma unroll
        for (int v = 0; v < SEGW / 4; v++) {
            const uint4 x = ldg_nc(p + 16 * v);
            w[4 * v] = x.x;
            w[4 * v + 1] = x.y;
            w[4 * v + 2] = x.z;
            w[4 * v + 3] = x.w;
        }
    }
}

__device__ __forceinline__ float2 ldg_f2(const float *p) {
    return __ldg(reinterpret_cast<const float2 *>(p));
}

// Physical dimension of logical k (0..31) in K-chunk c for quad q: the byte
// layout of one token's codes, as consumed by the A fragment.
template <int BITS, int D>
__device__ __forceinline__ int k_dim(int c, int q, int k) {
    constexpr int KB = D * BITS / 8;  // code bytes per token
    constexpr int SEG = KB / 4;       // bytes owned by one quad
    const int hi = k >> 4, e = k & 3;  // k = 4q+e (hi=0) or 16+4q+e (hi=1)
    if (BITS == 4) return 2 * (q * SEG + 4 * c + e) + hi;
    return q * SEG + 8 * c + 4 * hi + e;
}

// Word index (within a 4-token group) that gives n-tile `nt`, column `col`
// of the PV B fragment, and the dimension it carries.
template <int BITS, int D>
__device__ __forceinline__ int v_dim(int nt, int col) {
    if (BITS == 4) {
        const int i = nt >> 1, hi = nt & 1;
        const int w = 32 * (i >> 2) + 4 * col + (i & 3);
        return 2 * w + hi;
    }
    return 32 * (nt >> 2) + 4 * col + (nt & 3);
}

template <typename T, int BITS, int D>
__global__ void __launch_bounds__(kNW * 32, 2)
    decode_mma_kernel(AttendArgs a, int n_splits, int tokens_per_split, int tokens_per_warp) {
    constexpr int KB = D * BITS / 8;
    constexpr int SEGW = KB / 16;         // 32-bit words per quad per K row
    constexpr int NCH = D / 32;           // K chunks of 32 dims
    constexpr int NTV = D / 8;            // PV n-tiles
    constexpr int VW = (BITS == 4) ? NTV / 2 : NTV;  // V words per thread per 4-token group
    constexpr int VV = VW / 4;            // uint4 loads per thread per 4-token group
    constexpr int EPL = D / 32;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *s_q = reinterpret_cast<float *>(smem_raw);            // [4][D]
    float *s_qsum = s_q + 4 * D;                                  // [4]
    float *s_sigma = s_qsum + 4;                                  // [4]
    float *s_R = s_sigma + 4;                                     // [kNW][4]
    float *s_sc = s_R + kNW * 4;                                  // [kNW][kTPW][4]
    float *s_lv = s_sc + kNW * kTPW * 4;                          // [kNW][kTPW]
    unsigned char *s_p = reinterpret_cast<unsigned char *>(s_lv + kNW * kTPW);  // [kNW][16][kPRow]
    // merge area (reuses s_sc after phase 2): [kNW][4][D] acc + [kNW][4][3] R,L,Z
    float *m_acc = s_sc;
    float *m_rlz = s_sc + kNW * 4 * D;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = lane >> 2, q = lane & 3;
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int G = a.group;
    const int64_t qpos = a.pos0;  // single query token
    const int64_t total = qpos + 1;
    const float *sg = a.signs + (int64_t)h * D;
    const int qheads = a.heads * G;

    // ---- prologue: RoPE + rotation + digit scale of the G query heads ----
    if (warp < G) {
        const int g = warp;
        const T *src = static_cast<const T *>(a.query) + ((int64_t)b * qheads + h * G + g) * D;
        float x[EPL];
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) x[rr] = ld_f32(src + lane * EPL + rr);
        if (a.do_rotary) {
            const int half = D / 2;
            const float *cr = a.cos_cache + qpos * half;
            const float *sr = a.sin_cache + qpos * half;
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) {
                const int e = lane * EPL + rr;
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
                const float c = cr[pair], sn = sr[pair];
                const float xo = ld_f32(src + partner);
                x[rr] = first ? __fsub_rn(__fmul_rn(c, x[rr]), __fmul_rn(sn, xo))
                              : __fadd_rn(__fmul_rn(sn, xo), __fmul_rn(c, x[rr]));
            }
        }
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) x[rr] *= sg[lane * EPL + rr];
        warp_wht_butterfly<EPL>(x, lane, D);
        float sum = 0.0f, mabs = 0.0f;
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) {
            x[rr] *= a.wht_scale;
            s_q[g * D + lane * EPL + rr] = x[rr];
            sum += x[rr];
            mabs = fmaxf(mabs, fabsf(x[rr]));
        }
        sum = warp_sum(sum);
        mabs = warp_max(mabs);
        if (lane == 0) {
            s_qsum[g] = sum;
            s_sigma[g] = mabs > 0.0f ? mabs / kQMax : 1.0f;
        }
    }
    __syncthreads();

    // Q-digit B fragments: n-tile 0 column 2j -> (head j, digit 0), 2j+1 -> (head j, digit 1);
    // n-tile 1 column 2j -> (head j, digit 2), 2j+1 -> zero.  Column = r here.
    uint32_t bq[NCH][2][2];
    {
        const int hh = r >> 1;
        const bool has_head = hh < G;
        const float inv_sigma = has_head ? 1.0f / s_sigma[hh] : 0.0f;
#pragma unroll
        for (int c = 0; c < NCH; c++) {
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t w0 = 0, w1 = 0;  // n-tile 0, n-tile 1
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int k = 16 * half + 4 * q + e;
                    int qi = 0;
                    if (has_head) {
                        // |q'/sigma| <= kQMax up to rounding; clamp so the top digit stays in int8
                        qi = __float2int_rn(s_q[hh * D + k_dim<BITS, D>(c, q, k)] * inv_sigma);
                        qi = min(max(qi, -(int)kQMax), (int)kQMax);
                    }
                    // balanced base-256 digits: qi = d0*65536 + d1*256 + d2, each in [-127, 127]
                    const int d2 = (int)(int8_t)(qi & 0xff);
                    const int rest = (qi - d2) >> 8;
                    const int d1 = (int)(int8_t)(rest & 0xff);
                    const int d0 = (rest - d1) >> 8;
                    const int t0dig = (r & 1) ? d1 : d0;
                    const int t1dig = (r & 1) ? 0 : d2;
                    w0 |= ((uint32_t)(t0dig & 0xff)) << (8 * e);
                    w1 |= ((uint32_t)(t1dig & 0xff)) << (8 * e);
                }
                bq[c][0][half] = w0;
                bq[c][1][half] = w1;
            }
        }
    }
    const bool my_head = q < G;
    const float my_sigma = my_head ? s_sigma[q] : 0.0f;
    const float my_qsum = my_head ? s_qsum[q] : 0.0f;
    const float sl2 = a.scale * kLog2eF;

    const int64_t hrow = (int64_t)b * a.heads + h;
    const uint8_t *kc = a.k_codes + hrow * (int64_t)a.capacity * KB;
    const uint8_t *vc = a.v_codes + hrow * (int64_t)a.capacity * KB;
    const float *km = a.k_meta + hrow * (int64_t)a.capacity * 2;
    const float *vm = a.v_meta + hrow * (int64_t)a.capacity * 2;

    int64_t s_begin = (int64_t)split * tokens_per_split;
    int64_t s_end = s_begin + tokens_per_split;
    if (s_end > total) s_end = total;
    const int64_t tw0 = s_begin + (int64_t)warp * tokens_per_warp;
    int64_t tw1 = tw0 + tokens_per_warp;
    if (tw1 > s_end) tw1 = s_end;

    float *sc = s_sc + warp * kTPW * 4;
    float *lvb = s_lv + warp * kTPW;

    // ---- phase 1: scores ----
    float rmax = -INFINITY;
    for (int64_t t0 = tw0; t0 < tw1; t0 += 64) {
        uint32_t kr[4][2][SEGW];
        float2 kmt[4][2];
        float vsc[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                const int64_t t = t0 + 16 * i + r + 8 * hf;
                if (t < tw1) {
                    load_seg<SEGW>(kc + t * KB + q * (KB / 4), kr[i][hf]);
                    kmt[i][hf] = ldg_f2(km + 2 * t);
                    vsc[i][hf] = __ldg(vm + 2 * t);
                } else {
#pragma unroll
                    for (int w = 0; w < SEGW; w++) kr[i][hf][w] = 0u;
                    kmt[i][hf] = make_float2(0.0f, 0.0f);
                    vsc[i][hf] = 1.0f;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (t0 + 16 * i >= tw1) break;
            int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
            const uint32_t *w0 = kr[i][0];
            const uint32_t *w1 = kr[i][1];
#pragma unroll
            for (int c = 0; c < NCH; c++) {
                uint32_t a0, a1, a2, a3;
                if (BITS == 4) {
                    a0 = w0[c] & 0x0F0F0F0Fu;
                    a1 = w1[c] & 0x0F0F0F0Fu;
                    a2 = (w0[c] >> 4) & 0x0F0F0F0Fu;
                    a3 = (w1[c] >> 4) & 0x0F0F0F0Fu;
                } else {
                    a0 = w0[2 * c];
                    a1 = w1[2 * c];
                    a2 = w0[2 * c + 1];
                    a3 = w1[2 * c + 1];
                }
                mma_u8s8(acc[0], a0, a1, a2, a3, bq[c][0][0], bq[c][0][1]);
                mma_u8s8(acc[1], a0, a1, a2, a3, bq[c][1][0], bq[c][1][1]);
            }
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                const int64_t t = t0 + 16 * i + r + 8 * hf;
                const float dot =
                    fmaf((float)acc[0][2 * hf], 65536.0f, fmaf((float)acc[0][2 * hf + 1], 256.0f, (float)acc[1][2 * hf])) *
                    my_sigma;
                float s = (kmt[i][hf].x * dot + kmt[i][hf].y * my_qsum) * sl2;
                const float lv = __log2f(vsc[i][hf]);
                const bool valid = t < tw1;
                if (!valid || !my_head) s = -INFINITY;
                const int tl = (int)(t - tw0);
                if (valid) {
                    if (my_head) sc[tl * 4 + q] = s;
                    if (q == 0) lvb[tl] = lv;
                    rmax = fmaxf(rmax, fmaxf(s, s + lv));
                }
            }
        }
    }
    // warp max over the 8 token rows sharing a head (lanes with equal q)
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
    rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
    if (lane < 4) s_R[warp * 4 + lane] = rmax;
    __syncwarp();

    // ---- phase 2: values ----
    float Rh[4];
#pragma unroll
    for (int hh = 0; hh < 4; hh++) Rh[hh] = s_R[warp * 4 + hh];
    unsigned char *pb = s_p + warp * 16 * kPRow;
    // rows 12..15 of the P tile stay zero
    reinterpret_cast<uint32_t *>(pb + (12 + (lane >> 3)) * kPRow)[lane & 7] = 0u;
    int pacc[NTV][4];
#pragma unroll
    for (int nt = 0; nt < NTV; nt++) pacc[nt][0] = pacc[nt][1] = pacc[nt][2] = pacc[nt][3] = 0;
    float Lp[4] = {0.f, 0.f, 0.f, 0.f}, Zp[4] = {0.f, 0.f, 0.f, 0.f};
    const int64_t ngroups = a.capacity / kVGroup;

    for (int64_t t0 = tw0; t0 < tw1; t0 += 32) {
        // V codes of token groups (t0/4 + q) and (t0/4 + 4 + q)
        uint4 vw[2][VV];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            const int64_t grp = t0 / kVGroup + 4 * hf + q;
            const bool ok = grp * kVGroup < tw1 && grp < ngroups;
            const uint8_t *gbase = vc + grp * (int64_t)(KB * kVGroup);
#pragma unroll
            for (int v = 0; v < VV; v++)
                vw[hf][v] = ok ? ldg_nc(gbase + 128 * v + 16 * r) : make_uint4(0, 0, 0, 0);
        }
        // P digits: lane = token
        {
            const int64_t t = t0 + lane;
            const bool valid = t < tw1;
            const int tl = (int)(t - tw0);
            float4 s4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            float lv = 0.0f, vz = 0.0f;
            if (valid) {
                s4 = *reinterpret_cast<const float4 *>(sc + tl * 4);
                lv = lvb[tl];
                vz = __ldg(vm + 2 * t + 1);
            }
            const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int hh = 0; hh < 4; hh++) {
                uint32_t U = 0;
                if (hh < G && valid) {
                    const float p = exp2f(sv[hh] - Rh[hh]);
                    const float u = exp2f(sv[hh] + lv - Rh[hh]);
                    Lp[hh] += p;
                    Zp[hh] = fmaf(p, vz, Zp[hh]);
                    U = __float2uint_rn(fminf(u, 1.0f) * kUMax);
                }
                pb[(0 + hh) * kPRow + lane] = (unsigned char)(U >> 16);
                pb[(4 + hh) * kPRow + lane] = (unsigned char)((U >> 8) & 0xffu);
                pb[(8 + hh) * kPRow + lane] = (unsigned char)(U & 0xffu);
            }
        }
        __syncwarp();
        const uint32_t pa0 = *reinterpret_cast<const uint32_t *>(pb + r * kPRow + 4 * q);
        const uint32_t pa1 = *reinterpret_cast<const uint32_t *>(pb + (r + 8) * kPRow + 4 * q);
        const uint32_t pa2 = *reinterpret_cast<const uint32_t *>(pb + r * kPRow + 16 + 4 * q);
        const uint32_t pa3 = *reinterpret_cast<const uint32_t *>(pb + (r + 8) * kPRow + 16 + 4 * q);
        __syncwarp();
#pragma unroll
        for (int v = 0; v < VV; v++) {
            const uint32_t x0[4] = {vw[0][v].x, vw[0][v].y, vw[0][v].z, vw[0][v].w};
            const uint32_t x1[4] = {vw[1][v].x, vw[1][v].y, vw[1][v].z, vw[1][v].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int i = 4 * v + j;  // word index within the thread's VW words
                if (BITS == 4) {
                    mma_u8u8(pacc[2 * i], pa0, pa1, pa2, pa3, x0[j] & 0x0F0F0F0Fu, x1[j] & 0x0F0F0F0Fu);
                    mma_u8u8(pacc[2 * i + 1], pa0, pa1, pa2, pa3, (x0[j] >> 4) & 0x0F0F0F0Fu,
                             (x1[j] >> 4) & 0x0F0F0F0Fu);
                } else {
                    mma_u8u8(pacc[i], pa0, pa1, pa2, pa3, x0[j], x1[j]);
                }
            }
        }
    }

    // ---- warp partial -> shared memory ----
#pragma unroll
    for (int hh = 0; hh < 4; hh++) {
        Lp[hh] = warp_sum(Lp[hh]);
        Zp[hh] = warp_sum(Zp[hh]);
    }
    __syncthreads();  // every warp is done with s_sc before it becomes the merge area
    float *macc = m_acc + warp * 4 * D;
    // rows: r<4 -> (digit 0, head r) and (digit 2, head r); r>=4 -> (digit 1, head r-4)
#pragma unroll
    for (int nt = 0; nt < NTV; nt++) {
#pragma unroll
        for (int cc = 0; cc < 2; cc++) {
            const int mid = __shfl_down_sync(0xffffffffu, pacc[nt][cc], 16);
            if (r < 4 && r < G) {
                const float v = fmaf((float)pacc[nt][cc], 65536.0f, fmaf((float)mid, 256.0f, (float)pacc[nt][2 + cc]));
                macc[r * D + v_dim<BITS, D>(nt, 2 * q + cc)] = v * (1.0f / kUMax);
            }
        }
    }
    if (lane < 4) {
        m_rlz[(warp * 4 + lane) * 3 + 0] = Rh[lane];
        m_rlz[(warp * 4 + lane) * 3 + 1] = Lp[lane];
        m_rlz[(warp * 4 + lane) * 3 + 2] = Zp[lane];
    }
    __syncthreads();

    // ---- merge warps; warp g finishes head g ----
    if (warp < G) {
        const int g = warp;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kNW; w++) M = fmaxf(M, m_rlz[(w * 4 + g) * 3]);
        float wt[kNW], L = 0.0f, Z = 0.0f;
#pragma unroll
        for (int w = 0; w < kNW; w++) {
            const float Rw = m_rlz[(w * 4 + g) * 3];
            wt[w] = (Rw == -INFINITY) ? 0.0f : exp2f(Rw - M);
            L = fmaf(wt[w], m_rlz[(w * 4 + g) * 3 + 1], L);
            Z = fmaf(wt[w], m_rlz[(w * 4 + g) * 3 + 2], Z);
        }
        float x[EPL];
#pragma unroll
        for (int rr = 0; rr < EPL; rr++) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kNW; w++) s = fmaf(wt[w], m_acc[(w * 4 + g) * D + lane * EPL + rr], s);
            x[rr] = s;
        }
        if (n_splits == 1) {
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) x[rr] = L > 0.0f ? (x[rr] + Z) * inv : 0.0f;
            warp_wht_butterfly<EPL>(x, lane, D);
            T *dst = static_cast<T *>(a.out) + ((int64_t)b * qheads + h * G + g) * D;
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) st_from_f32(dst + lane * EPL + rr, x[rr] * a.wht_scale * sg[lane * EPL + rr]);
        } else {
            float *ws = a.workspace + ((((int64_t)b * a.heads + h) * n_splits + split) * G + g) * (D + 4);
#pragma unroll
            for (int rr = 0; rr < EPL; rr++) ws[lane * EPL + rr] = x[rr];
            if (lane == 0) {
                ws[D] = M;
                ws[D + 1] = L;
                ws[D + 2] = Z;
            }
        }
    }
}

size_t decode_smem_bytes(int d) {
    return sizeof(float) * ((size_t)4 * d + 4 + 4 + kNW * 4 + (size_t)kNW * kTPW * 4 + (size_t)kNW * kTPW) +
           (size_t)kNW * 16 * kPRow;
}

template <typename T, int BITS, int D>
int launch_decode(const AttendArgs &a, int n_splits, int tps, int tpw, cudaStream_t stream) {
    auto kern = decode_mma_kernel<T, BITS, D>;
    const size_t smem = decode_smem_bytes(D);
    static int configured[64];  // per device: the shared-memory opt-in is set once
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "gqa_decode_mma smem attribute");
        if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
    }
    dim3 grid(n_splits, a.heads, a.batch);
    kern<<<grid, kNW * 32, smem, stream>>>(a, n_splits, tps, tpw);
    count_launch();
    int rc = check_cuda(cudaGetLastError(), "gqa_decode_mma launch");
    if (rc != SA_OK || n_splits == 1) return rc;
    return launch_gqa_combine(a, n_splits, stream);
}

template <typename T>
int launch_by_shape(const AttendArgs &a, int n_splits, int tps, int tpw, cudaStream_t stream) {
    if (a.bits == 4 && a.head_dim == 128) return launch_decode<T, 4, 128>(a, n_splits, tps, tpw, stream);
    if (a.bits == 8 && a.head_dim == 128) return launch_decode<T, 8, 128>(a, n_splits, tps, tpw, stream);
    if (a.bits == 4 && a.head_dim == 64) return launch_decode<T, 4, 64>(a, n_splits, tps, tpw, stream);
    return launch_decode<T, 8, 64>(a, n_splits, tps, tpw, stream);
}

}  // namespace

int launch_gqa_decode_fast(const AttendArgs &a, cudaStream_t stream, bool *handled) {
    *handled = false;
    if (a.seq_len != 1 || a.group > 4 || (a.bits != 4 && a.bits != 8) || (a.head_dim != 64 && a.head_dim != 128))
        return SA_OK;
    if (a.capacity % 64 != 0) return SA_OK;
    const int64_t total = a.pos0 + 1;
    const int64_t units = (int64_t)a.batch * a.heads;
    // splits: every warp holds at most kTPW tokens; enough CTAs for ~7 waves
    // of 2 CTAs per SM; partials must fit the workspace.
    int64_t n_min = (total + (int64_t)kNW * kTPW - 1) / ((int64_t)kNW * kTPW);
    int64_t n_want = (14LL * a.sm_count + units - 1) / units;
    int64_t n_len = (total + kNW * 16 - 1) / (kNW * 16);  // at least 16 tokens per warp
    int64_t n = n_want < n_len ? n_want : n_len;
    if (n < n_min) n = n_min;
    if (n > kMaxSplits) n = kMaxSplits;
    if (n < n_min) return SA_OK;  // context too long for the split limit: generic path
    const int64_t per_split = (int64_t)a.group * (a.head_dim + 4) * units;
    if (n > 1 && (size_t)(n * per_split) > a.workspace_floats) {
        n = (int64_t)(a.workspace_floats / (size_t)per_split);
        if (n < n_min || n < 1) return SA_OK;
    }
    // tokens per warp: multiple of 16; tokens per split = kNW * tokens per warp
    int64_t tpw = (total + n * kNW - 1) / (n * kNW);
    tpw = (tpw + 15) / 16 * 16;
    if (tpw > kTPW) return SA_OK;
    const int64_t tps = tpw * kNW;
    n = (total + tps - 1) / tps;
    *handled = true;
    switch (a.dtype) {
        case SA_DTYPE_FLOAT: return launch_by_shape<float>(a, (int)n, (int)tps, (int)tpw, stream);
        case SA_DTYPE_FLOAT16: return launch_by_shape<__half>(a, (int)n, (int)tps, (int)tpw, stream);
        default: return launch_by_shape<__nv_bfloat16>(a, (int)n, (int)tps, (int)tpw, stream);
    }
}

}  // namespace sa

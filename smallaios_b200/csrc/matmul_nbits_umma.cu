// MatMulNBits on the 5th-generation tensor cores (tcgen05, sm_100a): int4
// weights, block 32, fp16/bf16 activations with scales of the same type,
// default zero point 8, 17 or more activation rows (blocks of up to 128).
//
// The product is computed transposed (weights as the MMA's M side):
//   D[n, m] = sum_k W[n, k] * A[m, k],  W[n, k] = (q[n, k] - 8) * s[n, k / 32]
// One CTA owns 128 weight rows (UMMA M = 128) and a block of BN (32..128)
// activation rows (UMMA N; grid.y walks the blocks), over the whole K:
//
//  warp 0     TMA producer: per stage of 256 k, the [128 rows x 128 B] code
//             tile (128-byte swizzle), the [128 x 8] scale tile and four
//             [BN x 64] activation tiles in the canonical K-major SW128
//             layout the MMA reads directly.
//  warps 1,10 warp 1 allocates 512 TMEM columns; one elected lane of each
//             issues the MMAs of the even / odd sub-chunks
//             (tcgen05.mma kind::f16, A from TMEM, B from shared memory,
//             D = f32 in TMEM: 256 / BN accumulators of BN columns taken in
//             turn, so that back-to-back MMAs are independent) and commits
//             their completion to the mbarriers that recycle the buffers.
//  warps 2-9  dequantize: each thread owns one weight row (its TMEM lane)
//             and writes 64 k of it per buffer into TMEM (tcgen05.st), four
//             buffers in flight.  Warps 2-5 take the even 64-k sub-chunks,
//             warps 6-9 the odd ones; warps 2-5 also run the epilogue
//             (tcgen05.ld of the accumulators, their sum, bias, conversion,
//             store).
//
// Exact weights: a scale s (fp16: 11 significant bits, bf16: 8) is split as
// s = s1 + s2 with s1 = s with its low three mantissa bits cleared.  q - 8
// has at most three significant bits, so (q-8)*s1 and (q-8)*s2 are exact in
// the 16-bit type, and the MMA's products are exact in fp32: two MMAs per
// k step (A1 = (q-8)*s1, A2 = (q-8)*s2) give the f32 dequantized product
// with f32 accumulation.
//
// Every mbarrier wait is bounded; a wait that gives up sets a shared abort
// flag (all roles leave their loops), the kernel lets its copies and MMAs
// land, frees TMEM and returns without writing y.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "sa_async.cuh"
#include "sa_common.cuh"
#include "sa_internal.h"
#include "sa_tcgen05.cuh"
#include "sa_tma.cuh"

namespace sa {

namespace {

constexpr int kUmBM = 128;                  // weight rows per CTA (UMMA M)
constexpr int kUmKC = 256;                  // k per TMA stage
constexpr int kUmNA = 4;                    // A buffers in TMEM (an even number: buffer q % NA belongs to group q % 2)
constexpr int kUmCodeTile = kUmBM * 128;    // [128 rows][128 B]
constexpr int kUmScaleTile = kUmBM * 16;    // [128 rows][8 scales]
constexpr int kUmDqWarps = 8;
constexpr int kUmThreads = 32 * (3 + kUmDqWarps);  // + the TMA warp and two MMA warps
constexpr uint32_t kUmTmemCols = 512;       // accumulators in [0, 256), A buffers in [256, 512)
constexpr uint32_t kUmAcol = 256;

__device__ int g_umma_status;  // bit 0: a bounded wait gave up

template <int BN>
struct UmGeo {
    static constexpr int NS = BN <= 32 ? 4 : (BN <= 64 ? 3 : 2);   // TMA stages
    // independent f32 accumulators in TMEM columns [0, 256): consecutive MMAs go to
    // different ones, so they do not wait for each other's accumulation
    static constexpr int NACC = 256 / BN;
    static constexpr int ACT_SUB = BN * 128;                       // one [BN][64] activation tile
    static constexpr int STAGE = kUmCodeTile + kUmScaleTile + 4 * ACT_SUB;
    // at least 116 KB, so that one CTA (holding 512 TMEM columns) runs per SM
    static constexpr int SMEM = (1024 + NS * STAGE + 256) > 116 * 1024 ? (1024 + NS * STAGE + 256) : 116 * 1024;
    static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
};

// Instruction descriptor, kind::f16: D f32, A and B of type T (K-major), N = BN, M = 128.
template <typename T, int BN>
__host__ __device__ constexpr uint32_t umma_idesc() {
    return (1u << 4) | ((std::is_same<T, __half>::value ? 0u : 1u) << 7) |
           ((std::is_same<T, __half>::value ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(kUmBM >> 4) << 24);
}

// Barrier over every thread of every CTA of the cluster (release / acquire:
// shared and global writes before it are visible after it).
__device__ __forceinline__ void cluster_sync_all() {
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Generic address of the same shared-memory location in CTA 0 of the cluster.
__device__ __forceinline__ float *map_to_rank0(float *p) {
    uint64_t out;
    asm volatile("mapa.u64 %0, %1, 0;\n" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)));
    return reinterpret_cast<float *>(out);
}

constexpr uint64_t kUmWaitNs = 2000000000ull;

// Bounded wait that also gives up when another role has aborted; the bound is
// 2 s of %globaltimer.
__device__ __forceinline__ bool um_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (um_try(bar, parity)) return true;
    const uint64_t t0 = um_clock_ns();
    for (uint32_t it = 1;; ++it) {
        if (um_try(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (*abort_flag) return false;
            if (um_clock_ns() - t0 > kUmWaitNs) break;
        }
    }
    *abort_flag = 1;
    atomicOr(&g_umma_status, 1);
    return false;
}

// ---- dequantization: two k of one byte -> a packed pair, split by the scale halves ----
template <typename T>
struct UmDq {
    static constexpr uint32_t kMagic = std::is_same<T, __half>::value ? 0x64006400u : 0x43004300u;  // 1024 | 128 + q
    static constexpr uint16_t kBias = std::is_same<T, __half>::value ? 0x6408 : 0x4308;            // 1032 | 136
};

template <typename T>
__device__ __forceinline__ uint32_t um_sub8(uint32_t x) {
    if constexpr (std::is_same<T, __half>::value) {
        __half2 h = *reinterpret_cast<__half2 *>(&x);
        h = __hsub2(h, __halves2half2(__ushort_as_half(UmDq<T>::kBias), __ushort_as_half(UmDq<T>::kBias)));
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&x);
        h = __hsub2(h, __halves2bfloat162(__ushort_as_bfloat16(UmDq<T>::kBias), __ushort_as_bfloat16(UmDq<T>::kBias)));
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

template <typename T>
__device__ __forceinline__ uint32_t um_mul(uint32_t x, uint32_t s) {
    if constexpr (std::is_same<T, __half>::value) {
        __half2 h = __hmul2(*reinterpret_cast<__half2 *>(&x), *reinterpret_cast<__half2 *>(&s));
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = __hmul2(*reinterpret_cast<__nv_bfloat162 *>(&x), *reinterpret_cast<__nv_bfloat162 *>(&s));
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

// Scale halves of one 16-bit scale as packed pairs (s1, s1) and (s2, s2).
template <typename T>
__device__ __forceinline__ void um_split_scale(uint16_t s, uint32_t &p1, uint32_t &p2) {
    const uint16_t s1 = s & 0xFFF8u;
    uint16_t s2;
    if constexpr (std::is_same<T, __half>::value) {
        s2 = __half_as_ushort(__hsub(__ushort_as_half(s), __ushort_as_half(s1)));
    } else {
        s2 = __bfloat16_as_ushort(__hsub(__ushort_as_bfloat16(s), __ushort_as_bfloat16(s1)));
    }
    p1 = (uint32_t)s1 | ((uint32_t)s1 << 16);
    p2 = (uint32_t)s2 | ((uint32_t)s2 << 16);
}

// FUSED: the QKV projection of a decode step.  The CTA's 128 output columns
// are 128 / head_dim whole heads of one kind; the epilogue stores them
// (rounded) straight into q_out, k_out or v_out.  The rotary and the
// quantize-on-append then run as a programmatic dependent launch, one warp
// per head vector (qkv_finish_kernel): measured on B200 at the Llama-3-8B
// layer shape (batch 64), finishing the vectors inside this kernel's
// epilogue took 36.7 us for the projection against 22.6 us + a 3 us launch,
// the vector encode being latency-bound with a few warps per tile.
template <typename T, int BN, bool FUSED>
__global__ void __launch_bounds__(kUmThreads, 1)
    mnb_umma_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
                    const __grid_constant__ CUtensorMap tm_act, const T *__restrict__ bias, T *__restrict__ y, int m,
                    int n, int k, const __grid_constant__ QkvArgs qa) {
    using GG = UmGeo<BN>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + GG::NS * GG::STAGE);  // [NS] TMA landed
    uint64_t *empty = full + GG::NS;                                            // [NS] stage consumed
    uint64_t *afull = empty + GG::NS;                                           // [NA] A buffer written
    uint64_t *aempty = afull + kUmNA;                                           // [NA] A buffer read by its MMAs
    uint64_t *dfull = aempty + kUmNA;                                           // all MMAs complete
    uint32_t *tslot = reinterpret_cast<uint32_t *>(dfull + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    // split-K over a thread-block cluster: CTA `rank` of a cluster of `nsplit`
    // (consecutive blockIdx.x) takes chunks [cb, ce) of the tile's K
    uint32_t rank = 0, nsplit = 1;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(rank));
    asm volatile("mov.u32 %0, %%cluster_nctarank;\n" : "=r"(nsplit));
    const int n0 = (blockIdx.x / nsplit) * kUmBM;
    const int m0 = blockIdx.y * BN;  // first activation row of this CTA
    const int cb = (int)(rank * (k / kUmKC) / nsplit), ce = (int)((rank + 1) * (k / kUmKC) / nsplit);
    const int nchunks = ce - cb, nsub = 4 * nchunks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < GG::NS; i++) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kUmDqWarps + 2);
        }
        for (int i = 0; i < kUmNA; i++) {
            mbar_init(afull + i, 4);
            mbar_init(aempty + i, 1);
        }
        mbar_init(dfull, 2);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tslot, kUmTmemCols);
    tc_fence_before();
    __syncthreads();
    // a dependent launch (the fused projection's finishing kernel) may start; it waits for this grid
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    tc_fence_after();
    const uint32_t tbase = *tslot;

    int issued = 0;  // producer: stages issued
    if (warp == 0) {
        if (lane == 0) {
            auto load_act = [&](int c) {
                unsigned char *st = smem + (c % GG::NS) * GG::STAGE;
#pragma unroll
                for (int j = 0; j < 4; j++)
                    tma_load_2d(st + kUmCodeTile + kUmScaleTile + j * GG::ACT_SUB, &tm_act, (cb + c) * kUmKC + 64 * j,
                                m0, full + c % GG::NS);
            };
            // The weights do not depend on the kernel before this one (a programmatic dependent
            // launch may run this grid while it finishes): the first stages' codes and scales are
            // requested before the wait for the activations.
            const int pre = nchunks < GG::NS ? nchunks : GG::NS;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % GG::NS;
                if (c >= GG::NS && !um_wait(empty + s, (uint32_t)(((c / GG::NS) - 1) & 1), abort_flag)) break;
                unsigned char *st = smem + s * GG::STAGE;
                mbar_expect_tx(full + s, (uint32_t)GG::STAGE);
                const int cg = cb + c;  // chunk of the tile's K
                tma_load_2d(st, &tm_codes, cg * 128, n0, full + s);
                tma_load_2d(st + kUmCodeTile, &tm_scales, cg * 8, n0, full + s);
                if (c + 1 == pre) {
                    asm volatile("griddepcontrol.wait;\n" ::: "memory");
                    for (int c2 = 0; c2 < pre; c2++) load_act(c2);
                } else if (c >= pre) {
                    load_act(c);
                }
                issued = c + 1;
            }
        }
    } else if (warp == 1 || warp == 10) {
        // two MMA warps take the even and the odd sub-chunks, each into its own half of the
        // accumulators (issuing from two warps is 6-9% faster than from one); the whole warp
        // runs the loop (uniform descriptors) and one elected lane issues
        const int par = warp == 1 ? 0 : 1;
        constexpr uint32_t idesc = umma_idesc<T, BN>();
        for (int q = par; q < nsub; q += 2) {
            const int c = q >> 2, j = q & 3, s = c % GG::NS, ab = q % kUmNA;
            bool ok = j != par || um_wait(full + s, (uint32_t)((c / GG::NS) & 1), abort_flag);
            if (ok) ok = um_wait(afull + ab, (uint32_t)((q / kUmNA) & 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const uint32_t act = smem_u32(smem + s * GG::STAGE + kUmCodeTile + kUmScaleTile + j * GG::ACT_SUB);
            const uint32_t ta = tbase + kUmAcol + (uint32_t)ab * 64;
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t bdesc = sw128_kmajor_desc(act + 32 * kk);
#pragma unroll
                    for (int h = 0; h < 2; h++) {  // A1 = (q-8)*s1, A2 = (q-8)*s2
                        const int idx = (q >> 1) * 8 + 2 * kk + h;  // this warp's MMA count
                        constexpr int HA = GG::NACC / 2;
                        umma_ts(tbase + (uint32_t)((par * HA + idx % HA) * BN), ta + 32 * h + 8 * kk, bdesc, idesc,
                                idx >= HA ? 1u : 0u);
                    }
                }
                umma_commit(aempty + ab);
                if (j >= 2) umma_commit(empty + s);  // each MMA warp's last sub-chunk of the chunk
            }
            __syncwarp();
        }
        if (elect_one()) umma_commit(dfull);
        __syncwarp();
        // the MMAs always complete: wait for them (bounded) before TMEM is freed
        const uint64_t t0 = um_clock_ns();
        while (!um_try(dfull, 0) && um_clock_ns() - t0 < kUmWaitNs) {
        }
    } else {
        const int g = (warp - 2) >> 2, sp = warp & 3;
        const int row = 32 * sp + lane;                              // weight row in the tile = TMEM lane
        const uint32_t tl = tbase + ((uint32_t)(32 * sp) << 16);     // this warp's lane quarter
        // Software pipeline: sub-chunk q's TMEM stores drain while sub-chunk q + 2 is
        // dequantized into the other register set.
        // dq: wait for the stage, dequantize 64 k of this row into r (A1 in
        // r[0..31], A2 in r[32..63]).
        auto dq = [&](int q, uint32_t (&r)[64]) -> bool {
            const int c = q >> 2, j = q & 3, s = c % GG::NS;
            const bool ok = um_wait(full + s, (uint32_t)((c / GG::NS) & 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) return false;
            const unsigned char *st = smem + s * GG::STAGE;
            // 64 codes of this row: 16-byte units 2j and 2j+1 of its swizzled 128-byte line
            const uint4 u0 = *reinterpret_cast<const uint4 *>(st + row * 128 + (((2 * j) ^ (row & 7)) << 4));
            const uint4 u1 = *reinterpret_cast<const uint4 *>(st + row * 128 + (((2 * j + 1) ^ (row & 7)) << 4));
            const uint32_t sc = *reinterpret_cast<const uint32_t *>(st + kUmCodeTile + row * 16 + j * 4);
            uint32_t s1[2], s2[2];
            um_split_scale<T>((uint16_t)(sc & 0xFFFFu), s1[0], s2[0]);
            um_split_scale<T>((uint16_t)(sc >> 16), s1[1], s2[1]);
            const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int wi = 0; wi < 8; wi++) {  // words 0-3: block 2j, words 4-7: block 2j + 1
                const uint32_t w = wv[wi], wh = w >> 4;
#pragma unroll
                for (int p = 0; p < 4; p++) {
                    // byte p of w: its low nibble (k = 8wi + 2p) in half 0, high nibble in half 1
                    const uint32_t t = __byte_perm(w, wh, (uint32_t)(p | (p << 4) | ((4 + p) << 8) | ((4 + p) << 12)));
                    uint32_t x;
                    asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x) : "r"(t), "r"(0x000F000Fu), "r"(UmDq<T>::kMagic));
                    x = um_sub8<T>(x);
                    r[4 * wi + p] = um_mul<T>(x, s1[wi >> 2]);
                    r[32 + 4 * wi + p] = um_mul<T>(x, s2[wi >> 2]);
                }
            }
            return true;
        };
        // put: wait until buffer q % NA is free, store r into it
        auto put = [&](int q, const uint32_t (&r)[64]) -> bool {
            const int ab = q % kUmNA;
            const bool ok = q < kUmNA || um_wait(aempty + ab, (uint32_t)(((q / kUmNA) - 1) & 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) return false;
            tc_fence_after();
            const uint32_t abuf = tl + kUmAcol + (uint32_t)ab * 64;
            tmem_st16(abuf, r);
            tmem_st16(abuf + 16, r + 16);
            tmem_st16(abuf + 32, r + 32);
            tmem_st16(abuf + 48, r + 48);
            return true;
        };
        // fin: the stores of q have landed: hand the buffer to the MMA warp
        auto fin = [&](int q) {
            const int c = q >> 2, j = q & 3, s = c % GG::NS, ab = q % kUmNA;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(afull + ab);
                if (j >= 2) mbar_arrive(empty + s);
            }
        };
        uint32_t ra[64], rb[64];
        int q = g;
        if (q < nsub && dq(q, ra)) {
            for (;;) {
                if (!put(q, ra)) break;
                const int q2 = q + 2;
                const bool more2 = q2 < nsub && dq(q2, rb);
                fin(q);
                if (!more2 || !put(q2, rb)) break;
                const int q3 = q2 + 2;
                const bool more3 = q3 < nsub && dq(q3, ra);
                fin(q2);
                if (!more3) break;
                q = q3;
            }
        }
    }

    // ---- epilogue (every thread of the CTA comes here) ----
    // warps 2-5 hold TMEM lane quarters (warp & 3) = weight rows of the tile
    const bool epi = warp >= 2 && warp < 6;
    const int row = 32 * (warp & 3) + lane;
    const uint32_t tl = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
    bool ok = true;
    if (epi) {
        asm volatile("griddepcontrol.wait;\n" ::: "memory");  // y (and bias) may belong to the previous kernel
        ok = um_wait(dfull, 0, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
    }
    // this CTA's f32 sums of output column n0 + row, 16 activation rows at a time
    // (the accumulators' sum, in accumulator order; up to four TMEM loads in flight per wait)
    auto load_sums = [&](int c0, float (&acc)[16]) {
        constexpr int G = GG::NACC < 4 ? GG::NACC : 4;
#pragma unroll
        for (int i = 0; i < 16; i++) acc[i] = 0.0f;
#pragma unroll
        for (int d0 = 0; d0 < GG::NACC; d0 += G) {
            uint32_t v[G][16];
#pragma unroll
            for (int d = 0; d < G; d++) tmem_ld16(tl + (uint32_t)((d0 + d) * BN + c0), v[d]);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < G; d++)
#pragma unroll
                for (int i = 0; i < 16; i++) acc[i] += __uint_as_float(v[d][i]);
        }
    };
    // split-K: ranks 1.. store their sums into rank 0's shared memory ([rank-1][column][row], the
    // stages are idle after the first cluster barrier), rank 0 adds them
    float *part = reinterpret_cast<float *>(smem);
    if (nsplit > 1) {
        cluster_sync_all();
        if (epi && rank != 0 && ok && !*abort_flag) {
            float *dst = map_to_rank0(part) + (size_t)(rank - 1) * BN * kUmBM;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float acc[16];
                load_sums(c0, acc);
#pragma unroll
                for (int i = 0; i < 16; i++) dst[(c0 + i) * kUmBM + row] = acc[i];
            }
        }
        cluster_sync_all();
    }
    if (epi && rank == 0) {
        // destination of output column n0 + row: y, or the q / k / v output of the fused projection
        T *dst = y;
        int64_t ld = n, col = n0 + row;
        if constexpr (FUSED) {
            const int64_t qc = (int64_t)qa.q_heads * qa.ap.head_dim, kc = (int64_t)qa.ap.heads * qa.ap.head_dim;
            if (col < qc) {
                dst = static_cast<T *>(qa.q_out);
                ld = qc;
            } else if (col < qc + kc) {
                dst = static_cast<T *>(const_cast<void *>(qa.ap.key));
                ld = kc;
                col -= qc;
            } else {
                dst = static_cast<T *>(const_cast<void *>(qa.ap.value));
                ld = kc;
                col -= qc + kc;
            }
        }
        if (ok && !*abort_flag) {
            const float bv = bias ? DT<T>::to_f32(bias[n0 + row]) : 0.0f;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float acc[16];
                load_sums(c0, acc);
                for (uint32_t r = 1; r < nsplit; r++)
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[i] += part[((size_t)(r - 1) * BN + c0 + i) * kUmBM + row];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int mi = m0 + c0 + i;
                    if (mi < m) dst[(int64_t)mi * ld + col] = DT<T>::from_f32(acc[i] + bv);
                }
            }
        }
    }
    // teardown: copies still in flight after an abort land before the CTA exits
    if (warp == 0 && lane == 0 && *abort_flag) {
        for (int c = (issued > GG::NS ? issued - GG::NS : 0); c < issued; c++)
            mbar_wait_bounded(full + c % GG::NS, (uint32_t)((c / GG::NS) & 1));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, kUmTmemCols);
    }
}

template <typename T, int BN, bool FUSED>
int launch_umma_bn(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m,
                   int64_t n, int64_t k, const QkvArgs &qa, cudaStream_t stream) {
    using GG = UmGeo<BN>;
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(SA_ERR_CUDA, "MatMulNBits: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm_codes, tm_scales, tm_act;
    const cuuint32_t ones[2] = {1, 1};
    const cuuint64_t cdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n}, cstride[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t cbox[2] = {128, (cuuint32_t)kUmBM};
    CUresult r = encode(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(b), cdim, cstride, cbox,
                        ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits umma: code tensor map (%d)", (int)r);
    const cuuint64_t sdim[2] = {(cuuint64_t)(k / 32), (cuuint64_t)n}, sstride[1] = {(cuuint64_t)(k / 32) * 2};
    const cuuint32_t sbox[2] = {8, (cuuint32_t)kUmBM};
    r = encode(&tm_scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(scales), sdim, sstride, sbox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits umma: scale tensor map (%d)", (int)r);
    const cuuint64_t adim[2] = {(cuuint64_t)k, (cuuint64_t)m}, astride[1] = {(cuuint64_t)k * 2};
    const cuuint32_t abox[2] = {64, (cuuint32_t)BN};
    r = encode(&tm_act, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(a), adim, astride, abox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits umma: activation tensor map (%d)", (int)r);
    auto kern = mnb_umma_kernel<T, BN, FUSED>;
    static int configured[64];
    static int max_clusters[64][5];  // co-resident clusters of 2..4 CTAs
    int dev = 0;
    cudaGetDevice(&dev);
    const int tiles = (int)(n / kUmBM);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(kUmThreads);
    cfg.dynamicSmemBytes = GG::SMEM;
    cfg.stream = stream;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GG::SMEM);
        if (e != cudaSuccess) return check_cuda(e, "MatMulNBits umma smem attribute");
        if (dev >= 0 && dev < 64) {
            for (int sc = 2; sc <= 4; sc++) {
                at[0].val.clusterDim.x = (unsigned)sc;
                at[0].val.clusterDim.y = at[0].val.clusterDim.z = 1;
                cfg.gridDim = dim3((unsigned)(sc * 64));
                int nc = 0;
                if (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    nc = 0;
                }
                max_clusters[dev][sc] = nc;
            }
            __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
        }
    }
    // K split over a cluster: the largest of 2..4 CTAs per tile that keeps one
    // wave (every cluster co-resident) and whose partial sums fit in the stages
    int split = 1;
    int sm_count = 148;
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64)
        for (int sc = 2; sc <= 4; sc++)
            if (m <= BN && sc <= k / kUmKC && tiles * sc <= sm_count && tiles <= max_clusters[dev][sc] &&
                (sc - 1) * BN * kUmBM * 4 <= GG::NS * GG::STAGE)
                split = sc;
    at[0].val.clusterDim.x = (unsigned)split;
    at[0].val.clusterDim.y = at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(tiles * split), (unsigned)((m + BN - 1) / BN));
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tm_codes, tm_scales, tm_act, static_cast<const T *>(bias),
                                       static_cast<T *>(y), (int)m, (int)n, (int)k, qa);
    count_launch();
    return check_cuda(e, "MatMulNBits umma launch");
}

template <typename T, bool FUSED>
int launch_umma_t(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m,
                  int64_t n, int64_t k, const QkvArgs &qa, cudaStream_t stream) {
    if (m <= 32) return launch_umma_bn<T, 32, FUSED>(a, b, scales, bias, y, m, n, k, qa, stream);
    if (m <= 64) return launch_umma_bn<T, 64, FUSED>(a, b, scales, bias, y, m, n, k, qa, stream);
    return launch_umma_bn<T, 128, FUSED>(a, b, scales, bias, y, m, n, k, qa, stream);
}

}  // namespace

// fp16/bf16, block 32, default zero point, m >= 17 (blocks of 128 rows above
// 128), N a multiple of 128, K a multiple of 256, codes / scales /
// activations 16-byte aligned.
// (Up to 16 rows the mma.sync kernels are faster: a tile here pays the whole
// per-CTA dequant of its 128 weight rows and K/8 MMAs whatever the row count.)
bool matmul_nbits_umma_eligible(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, int dtype,
                                int64_t m, int64_t n, int64_t k, int block_size) {
    if (dtype != SA_DTYPE_FLOAT16 && dtype != SA_DTYPE_BFLOAT16) return false;
    if (zp || block_size != 32 || m < 17 || m > (1 << 22)) return false;  // grid.y = m / 128 blocks
    if (n % kUmBM != 0 || k % kUmKC != 0 || n > (1 << 30) || k > (1 << 24)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(scales);
    return (al & 15) == 0;
}

int launch_matmul_nbits_umma(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y,
                             int dtype, int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
    const QkvArgs none{};
    if (dtype == SA_DTYPE_FLOAT16) return launch_umma_t<__half, false>(a, b, scales, bias, y, m, n, k, none, stream);
    return launch_umma_t<__nv_bfloat16, false>(a, b, scales, bias, y, m, n, k, none, stream);
}

// The fused QKV projection: x [batch][k] times the packed [n][k] weights
// (q rows, then k rows, then v rows), epilogue per qkv_finish_vector.  The
// caller checked matmul_nbits_umma_eligible and that every 128-column tile
// holds whole heads of one kind (q_heads*D and kv_heads*D multiples of 128).
int launch_qkv_umma_fused(const void *x, const uint8_t *w_codes, const void *w_scales, const QkvArgs &a,
                          int64_t n, int64_t k, cudaStream_t stream) {
    const int64_t m = a.ap.batch;
    const int rc = a.ap.dtype == SA_DTYPE_FLOAT16
                       ? launch_umma_t<__half, true>(x, w_codes, w_scales, nullptr, nullptr, m, n, k, a, stream)
                       : launch_umma_t<__nv_bfloat16, true>(x, w_codes, w_scales, nullptr, nullptr, m, n, k, a, stream);
    if (rc != SA_OK) return rc;
    return launch_qkv_finish(a, stream);
}

}  // namespace sa

// MatMulNBits (ORT com.microsoft.MatMulNBits contract), int4 weights with
// per-(column, k-block) scales and optional packed zero points.
//
// tcgen05 path (matmul_nbits_umma.cu): fp16/bf16, block 32, default zero
// point, 17 <= m <= 128, N % 128 == 0, K % 256 == 0.  mma.sync path (m <= 64,
// the same types, N % 16 == 0): mnb_mma_kernel below.  Other shapes take the
// CUDA-core path:
//
// GEMV path (m <= 8 rows per pass): one warp per output column streams that
// column's packed codes with 128-bit loads (16 bytes = 32 codes per lane per
// step) and keeps the activation rows in registers/L1.  The block scale is
// factored out of the inner sum: y = sum_blk s_blk * (sum_k a_k*(q_k - zp)),
// so each code costs one integer extract and one FMA.  HBM-bound: the codes
// and scales are read exactly once.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "sa_async.cuh"
#include "sa_common.cuh"
#include "sa_internal.h"
#include "sa_tma.cuh"

namespace sa {

namespace {

constexpr int kGemvWarps = 8;

template <typename T>
__device__ __forceinline__ float scale_at(const T *s, int64_t i) {
    return DT<T>::to_f32(s[i]);
}

// grid.x covers columns (one warp each); rows [m0, m0 + MT) of A.
template <typename T, int MT>
__global__ void __launch_bounds__(32 * kGemvWarps)
    mnb_gemv_kernel(const T *__restrict__ a, const uint8_t *__restrict__ b, const T *__restrict__ scales,
                    const uint8_t *__restrict__ zps, const T *__restrict__ bias, T *__restrict__ y, int64_t m,
                    int64_t m0, int64_t n, int64_t k, int block_size) {
    const int lane = threadIdx.x & 31;
    const int64_t col = (int64_t)blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (col >= n) return;
    const int64_t nblk = k / block_size;
    const int64_t row_bytes = k / 2;
    const int64_t zp_row = (nblk * 4 + 7) / 8;
    const uint8_t *bcol = b + col * row_bytes;
    float acc[MT];
#pragma unroll
    for (int r = 0; r < MT; r++) acc[r] = 0.0f;

    // Each lane owns 32 consecutive k per step (16 bytes of codes); a block of
    // block_size >= 16 codes spans whole 16-element halves of that chunk.
    for (int64_t k0 = (int64_t)lane * 32; k0 < k; k0 += 32 * 32) {
        const uint4 w = *reinterpret_cast<const uint4 *>(bcol + k0 / 2);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        float part[MT][2];
#pragma unroll
        for (int r = 0; r < MT; r++) part[r][0] = part[r][1] = 0.0f;
        float zf[2];
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int64_t blk = (k0 + hlf * 16) / block_size;
            uint32_t zp = 8u;
            if (zps) {
                const uint8_t zb = zps[col * zp_row + blk / 2];
                zp = (blk & 1) ? (uint32_t)(zb >> 4) : (uint32_t)(zb & 15u);
            }
            zf[hlf] = (float)zp;
        }
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
            const int hlf = wi >> 1;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float qv = (float)((words[wi] >> (4 * j)) & 15u) - zf[hlf];
                const int64_t kk = k0 + wi * 8 + j;
#pragma unroll
                for (int r = 0; r < MT; r++) {
                    if (m0 + r < m) part[r][hlf] += ld_f32(a + (m0 + r) * k + kk) * qv;
                }
            }
        }
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int64_t blk = (k0 + hlf * 16) / block_size;
            const float s = scale_at(scales, col * nblk + blk);
#pragma unroll
            for (int r = 0; r < MT; r++) acc[r] += s * part[r][hlf];
        }
    }
#pragma unroll
    for (int r = 0; r < MT; r++) {
        float v = warp_sum(acc[r]);
        if (lane == 0 && m0 + r < m) {
            if (bias) v += ld_f32(bias + col);
            st_from_f32(y + (m0 + r) * n + col, v);
        }
    }
}

// ---- tensor-core path ---------------------------------------------------------
// One CTA owns a 16-column tile of N (the A operand of mma.m16n8k16: rows =
// output columns, k = the reduction) and SPLIT warps; warp w reduces over
// k-blocks [w*nbw, (w+1)*nbw).  Each warp streams its 16 columns' packed codes
// and block scales through kMnbSlots shared-memory slots, 8 blocks (128 B of
// codes per column) per chunk: one 2-D TMA copy of the 16 x 128 B code tile
// (128-byte swizzle, so the fragment loads hit distinct banks) and one of the
// 16 x 8 scales.  A 32-bit word of codes gives four fp16 (or bf16) pairs
// (q - 8) with a shift, a logic op that ORs the nibble into the mantissa of
// 1024 (128 for bf16), and a packed subtract: nibbles i and i+4 form one
// pair, and the activations are fed in the same k order.  Products and the
// per-block sums are exact fp32 (tensor-core accumulate); the block scale
// multiplies each block's sum in fp32.  The activations (B operand, columns =
// rows of A) come with each chunk too: a third TMA copy of the m x 256 tile.
constexpr int kMnbMaxSplit = 4;                    // warps (K splits) per CTA, at most
constexpr int kMnbChunk = 8;                       // k-blocks per chunk (128 B of codes per column)
constexpr int kMnbCodeTile = 16 * kMnbChunk * 16;  // 2048 B, 1024-aligned in shared memory
constexpr int kMnbScaleTile = 16 * kMnbChunk * 2;  // 256 B
constexpr int kMnbActRow = kMnbChunk * 32 * 2;     // 512 B: one activation row of a chunk

// Chunks in flight per warp (two: the CTA count is what keeps HBM busy).
__host__ __device__ constexpr int mnb_slots(int mrows) { return 2 + 0 * mrows; }
// K splits (warps) per CTA: more warps for one m-tile, fewer when the
// activation tiles are large.
[[maybe_unused]] constexpr int mnb_split(int mt) { return mt == 1 ? 4 : 2; }

template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1, bool zero_c) {
    if constexpr (std::is_same<T, __half>::value) {
        if (zero_c)
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%10,%10,%10,%10};\n"
                : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
        else
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};\n"
                : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        if (zero_c)
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%10,%10,%10,%10};\n"
                : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
        else
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};\n"
                : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// Nibbles i and i+4 of w as a packed pair (q - 8), exact in fp16 / bf16.
template <typename T>
__device__ __forceinline__ uint32_t dq_pair(uint32_t w, int i) {
    uint32_t x;
    if constexpr (std::is_same<T, __half>::value) {
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x) : "r"(w >> (4 * i)), "r"(0x000F000Fu), "r"(0x64006400u));
        __half2 h = *reinterpret_cast<__half2 *>(&x);
        h = __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));  // 1032
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x) : "r"(w >> (4 * i)), "r"(0x000F000Fu), "r"(0x43004300u));
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&x);
        h = __hsub2(h, __halves2bfloat162(__ushort_as_bfloat16(0x4308), __ushort_as_bfloat16(0x4308)));  // 136
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

// The four pairs of word w: p[0] = (n0, n4), p[1] = (n1, n5), p[2] = (n2, n6),
// p[3] = (n3, n7) as (q - 8).  fp16 takes nibbles 1, 5, 3, 7 in place (bits
// 4-7 of the mantissa, one shift less per word) as 16 (q - 8); the matching
// activations are divided by 16 (mnb_act_scale_odd), which is exact.
template <typename T>
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t (&p)[4]) {
    if constexpr (std::is_same<T, __half>::value) {
        const uint32_t w8 = w >> 8;
        const __half2 o1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
        const __half2 o1152 = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
        uint32_t x[4];
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x[0]) : "r"(w), "r"(0x000F000Fu), "r"(0x64006400u));
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x[1]) : "r"(w), "r"(0x00F000F0u), "r"(0x64006400u));
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x[2]) : "r"(w8), "r"(0x000F000Fu), "r"(0x64006400u));
        asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(x[3]) : "r"(w8), "r"(0x00F000F0u), "r"(0x64006400u));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __half2 h = *reinterpret_cast<__half2 *>(&x[i]);
            h = __hsub2(h, (i & 1) ? o1152 : o1032);
            p[i] = *reinterpret_cast<uint32_t *>(&h);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) p[i] = dq_pair<T>(w, i);
    }
}

// Activation pair registers that meet the in-place high nibbles (b1, b3 of
// a block) are scaled by 1/16 for fp16 (exact: a power of two).
template <typename T>
__device__ __forceinline__ uint32_t mnb_act_scale_odd(uint32_t v) {
    if constexpr (std::is_same<T, __half>::value) {
        __half2 h = *reinterpret_cast<__half2 *>(&v);
        h = __hmul2(h, __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00)));  // 1/16
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        return v;
    }
}

// (fma.rn.f32x2) d = s * a + d on two lanes of packed f32.
__device__ __forceinline__ void ffma2(float &d0, float &d1, float s, float a0, float a1) {
    asm("{\n.reg .b64 dd, aa, ss;\nmov.b64 aa, {%2, %3};\nmov.b64 ss, {%4, %4};\nmov.b64 dd, {%0, %1};\n"
        "fma.rn.f32x2 dd, aa, ss, dd;\nmov.b64 {%0, %1}, dd;\n}\n"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(s));
}

// NT = 16-column tiles per warp (they share the activation fragments);
// SUB = 128-byte code sub-tiles per chunk (a chunk is 8 * SUB k-blocks, so
// each row of a chunk is SUB * 128 contiguous bytes of HBM).
template <typename T, int MT, int NS, int SPLIT, int NT, int SUB>
__global__ void __launch_bounds__(32 * SPLIT)
    mnb_mma_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
                   const __grid_constant__ CUtensorMap tm_act, const T *__restrict__ bias, T *__restrict__ y, int m,
                   int n, int k) {
    constexpr int CHUNK = kMnbChunk * SUB;                       // k-blocks per chunk
    constexpr int SUBTILE = NT * kMnbCodeTile;                   // one [16 NT][128 B] code sub-tile
    constexpr int CODE_TILE = SUB * SUBTILE, SCALE_TILE = NT * SUB * kMnbScaleTile;
    constexpr int ACT_ROW = SUB * kMnbActRow;                    // bytes of one activation row per chunk
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the 128-byte swizzle pattern assumes 1024-byte aligned tiles: align the base explicitly
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // [SPLIT][NS] code tiles (1024-aligned for the swizzle), then the scale
    // and activation tiles, barriers, the reduction area
    const int mrows = m;
    const int act_bytes = ((mrows * ACT_ROW + 127) / 128) * 128;
    unsigned char *codes = smem + warp * NS * CODE_TILE;
    unsigned char *scl = smem + SPLIT * NS * CODE_TILE + warp * NS * (SCALE_TILE + act_bytes);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SPLIT * NS * (CODE_TILE + SCALE_TILE + act_bytes)) +
                     warp * NS;
    float *red = reinterpret_cast<float *>(smem + SPLIT * NS * (CODE_TILE + SCALE_TILE + act_bytes) +
                                           SPLIT * NS * 8);

    const int n0 = blockIdx.x * 16 * NT;
    const int nblk = k / 32;
    const int nbw = nblk / SPLIT;  // a multiple of CHUNK
    const int b0 = warp * nbw;
    const int nchunks = nbw / CHUNK;
    if (lane == 0) {
        for (int i = 0; i < NS; i++) mbar_init(bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int c) {  // lane 0: chunk c -> slot c % NS
        const int s = c % NS;
        const int blk = b0 + c * CHUNK;
        unsigned char *st = scl + s * (SCALE_TILE + act_bytes);
        mbar_expect_tx(bars + s, CODE_TILE + SCALE_TILE + mrows * ACT_ROW);
#pragma unroll
        for (int sb = 0; sb < SUB; sb++)
            tma_load_2d(codes + s * CODE_TILE + sb * SUBTILE, &tm_codes, (blk + kMnbChunk * sb) * 16, n0, bars + s);
        tma_load_2d(st, &tm_scales, blk, n0, bars + s);
#pragma unroll
        for (int sb = 0; sb < SUB; sb++)  // [SUB][m][256] activation sub-tiles
            tma_load_2d(st + SCALE_TILE + sb * mrows * kMnbActRow, &tm_act, (blk + kMnbChunk * sb) * 32, 0, bars + s);
    };
    if (lane == 0)
        for (int c = 0; c < NS && c < nchunks; c++) issue(c);

    float tot[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++) tot[mt][nt][0] = tot[mt][nt][1] = tot[mt][nt][2] = tot[mt][nt][3] = 0.0f;
    bool ok = true;
    int c = 0;
    for (; c < nchunks; c++) {
        const int s = c % NS;
        if (ok && !mbar_wait_bounded(bars + s, (uint32_t)((c / NS) & 1))) ok = false;
        if (__any_sync(0xffffffffu, !ok)) break;  // a copy never landed: give up (output left unwritten)
#pragma unroll
      for (int sb = 0; sb < SUB; sb++) {
        const unsigned char *ct = codes + s * CODE_TILE + sb * SUBTILE;
        const unsigned char *sc = scl + s * (SCALE_TILE + act_bytes);
        const unsigned char *at = sc + SCALE_TILE + sb * mrows * kMnbActRow;  // [mrows][256] activations
        // this lane's scales of the sub-tile's 8 blocks, rows 16 nt + g and 16 nt + g + 8
        uint4 srow[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            srow[nt][0] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g) * CHUNK * 2 + sb * 16);
            srow[nt][1] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g + 8) * CHUNK * 2 + sb * 16);
        }
#pragma unroll
        for (int bi = 0; bi < kMnbChunk; bi++) {
            // the activation fragments of block bi, shared by the NT tiles
            uint32_t bf[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                const int row = mt * 8 + g;
                uint4 x = make_uint4(0u, 0u, 0u, 0u);
                if (row < m) x = *reinterpret_cast<const uint4 *>(at + row * kMnbActRow + bi * 64 + 16 * t);
                bf[mt][0] = __byte_perm(x.x, x.z, 0x5410);
                bf[mt][1] = mnb_act_scale_odd<T>(__byte_perm(x.x, x.z, 0x7632));
                bf[mt][2] = __byte_perm(x.y, x.w, 0x5410);
                bf[mt][3] = mnb_act_scale_odd<T>(__byte_perm(x.y, x.w, 0x7632));
            }
            // rows g and g+8 of each 128-byte-swizzled 16-row tile: 16-byte unit bi sits at unit bi ^ (row & 7)
            const int u = ((bi ^ g) & 7) * 16 + 4 * t;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint32_t w0 = *reinterpret_cast<const uint32_t *>(ct + (16 * nt + g) * 128 + u);
                const uint32_t w1 = *reinterpret_cast<const uint32_t *>(ct + (16 * nt + g + 8) * 128 + u);
                uint32_t q0[4], q1[4];
                dq_word<T>(w0, q0);
                dq_word<T>(w1, q1);
                const uint32_t p00 = q0[0], p10 = q1[0], p01 = q0[1], p11 = q1[1];
                const uint32_t p02 = q0[2], p12 = q1[2], p03 = q0[3], p13 = q1[3];
                const uint32_t sw0 = (&srow[nt][0].x)[bi >> 1], sw1 = (&srow[nt][1].x)[bi >> 1];
                const T s0 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw0) + (bi & 1));
                const T s1 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw1) + (bi & 1));
                const float sg = DT<T>::to_f32(s0), sg8 = DT<T>::to_f32(s1);
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    float acc[4];
                    mma_16816<T>(acc, p00, p10, p01, p11, bf[mt][0], bf[mt][1], true);
                    mma_16816<T>(acc, p02, p12, p03, p13, bf[mt][2], bf[mt][3], false);
                    ffma2(tot[mt][nt][0], tot[mt][nt][1], sg, acc[0], acc[1]);
                    ffma2(tot[mt][nt][2], tot[mt][nt][3], sg8, acc[2], acc[3]);
                }
            }
        }
      }
        __syncwarp();
        if (lane == 0 && c + NS < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            issue(c + NS);
        }
    }
    if (!ok && lane == 0) {
        // chunk c never landed: let this warp's copies still in flight land (bounded)
        for (int cc = c; cc < c + NS && cc < nchunks; cc++)
            mbar_wait_bounded(bars + cc % NS, (uint32_t)((cc / NS) & 1));
    }
    // sum the K splits: warps 1.. leave their sums in shared memory, warp 0 adds and stores
    constexpr int PER = MT * NT * 4;
    if (warp > 0) {
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    red[((warp - 1) * 32 + lane) * PER + (mt * NT + nt) * 4 + j] = tot[mt][nt][j];
    }
    __syncthreads();
    if (warp != 0 || !ok) return;
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float v = tot[mt][nt][j];
                for (int w = 1; w < SPLIT; w++) v += red[((w - 1) * 32 + lane) * PER + (mt * NT + nt) * 4 + j];
                const int row = mt * 8 + 2 * t + (j & 1);
                const int col = n0 + 16 * nt + g + ((j & 2) ? 8 : 0);
                if (row < m) {
                    if (bias) v += DT<T>::to_f32(bias[col]);
                    st_from_f32(y + (int64_t)row * n + col, v);
                }
            }
        }
    }
}

constexpr size_t mnb_mma_smem(int mt, int ns, int split, int nt, int sub, int mrows) {
    return 1024 +
           (size_t)split * ns *
               (nt * sub * (kMnbCodeTile + kMnbScaleTile) + ((mrows * sub * kMnbActRow + 127) / 128) * 128) +
           split * ns * 8 + (size_t)(split - 1) * 32 * mt * nt * 4 * 4;
}

template <typename T, int MT, int NT, int SUB = 1, int SPLIT = mnb_split(MT)>
int launch_mma(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m,
               int64_t n, int64_t k, cudaStream_t stream) {
    if (k % (32 * SPLIT * kMnbChunk * SUB) != 0) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: K split");
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(SA_ERR_CUDA, "MatMulNBits: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm_codes, tm_scales, tm_act;
    const cuuint64_t cdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n}, cstride[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t cbox[2] = {kMnbChunk * 16, 16 * NT}, ones[2] = {1, 1};
    CUresult r = encode(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(b), cdim, cstride, cbox,
                        ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: code tensor map (%d)", (int)r);
    const cuuint64_t sdim[2] = {(cuuint64_t)(k / 32), (cuuint64_t)n}, sstride[1] = {(cuuint64_t)(k / 32) * 2};
    const cuuint32_t sbox[2] = {kMnbChunk * SUB, 16 * NT};
    r = encode(&tm_scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(scales), sdim, sstride, sbox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: scale tensor map (%d)", (int)r);
    const cuuint64_t adim[2] = {(cuuint64_t)k, (cuuint64_t)m}, astride[1] = {(cuuint64_t)k * 2};
    const cuuint32_t abox[2] = {kMnbChunk * 32, (cuuint32_t)m};
    r = encode(&tm_act, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(a), adim, astride, abox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: activation tensor map (%d)", (int)r);
    const int mrows = (int)m;
    const size_t smem = mnb_mma_smem(MT, mnb_slots(mrows), SPLIT, NT, SUB, mrows);
    auto kern = mnb_mma_kernel<T, MT, 2, SPLIT, NT, SUB>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "MatMulNBits smem attribute");
    }
    kern<<<(unsigned)(n / (16 * NT)), 32 * SPLIT, smem, stream>>>(tm_codes, tm_scales, tm_act,
                                                                  static_cast<const T *>(bias), static_cast<T *>(y),
                                                                  (int)m, (int)n, (int)k);
    count_launch();
    return check_cuda(cudaGetLastError(), "MatMulNBits mma launch");
}

// ---- tensor-core path, 17..64 rows: the activation tile is shared by the CTA ----
// One CTA = 4 warps = 64 output columns over the whole K.  Thread 0 fetches,
// per chunk of 8 k-blocks, the 64 x 128 B code tile (128-byte swizzle), the
// 64 x 8 scales and the activations as four m x 64 sub-tiles (128-byte
// swizzle, so the fragment loads of 8 rows hit distinct banks); every warp
// dequantizes its 16 columns once per block and runs the m-tiles against it.
// A block-wide barrier after each chunk frees its slot for the next copy.
constexpr int kMnbWideWarps = 4;
constexpr int kMnbWideSlots = 2;

template <typename T, int MT>
__global__ void __launch_bounds__(32 * kMnbWideWarps)
    mnb_mma_wide_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
                        const __grid_constant__ CUtensorMap tm_act, const T *__restrict__ bias, T *__restrict__ y,
                        int m, int n, int k) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int mpad = (m + 7) & ~7;
    const int act_sub = mpad * 128;                         // one m x 64 activation sub-tile
    const int code_bytes = 64 * 128, scale_bytes = 64 * kMnbChunk * 2;
    const int slot_bytes = code_bytes + 4 * act_sub + ((scale_bytes + 1023) & ~1023);  // keeps 1024 alignment
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kMnbWideSlots * slot_bytes);
    const int n0 = blockIdx.x * 64;
    const int nchunks = k / (32 * kMnbChunk);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMnbWideSlots; i++) mbar_init(full + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](int c) {  // thread 0
        const int sl = c % kMnbWideSlots;
        unsigned char *base = smem + sl * slot_bytes;
        const int blk = c * kMnbChunk;
        mbar_expect_tx(full + sl, code_bytes + scale_bytes + 4 * m * 128);
        tma_load_2d(base, &tm_codes, blk * 16, n0, full + sl);
        for (int sb = 0; sb < 4; sb++) tma_load_2d(base + code_bytes + sb * act_sub, &tm_act, blk * 32 + sb * 64, 0, full + sl);
        tma_load_2d(base + code_bytes + 4 * act_sub, &tm_scales, blk, n0, full + sl);
    };
    if (threadIdx.x == 0)
        for (int c = 0; c < kMnbWideSlots && c < nchunks; c++) issue(c);

    float tot[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; mt++) tot[mt][0] = tot[mt][1] = tot[mt][2] = tot[mt][3] = 0.0f;
    const int r0 = 16 * warp + g;  // this lane's rows (output columns) of the 64-row tiles: r0, r0 + 8
    bool ok = true;
    int c = 0;
    for (; c < nchunks; c++) {
        const int sl = c % kMnbWideSlots;
        if (ok && !mbar_wait_bounded(full + sl, (uint32_t)((c / kMnbWideSlots) & 1))) ok = false;
        const int fail = __syncthreads_or(!ok);
        if (fail) {
            ok = false;
            break;
        }
        const unsigned char *ct = smem + sl * slot_bytes;
        const unsigned char *at = ct + code_bytes;
        const T *st = reinterpret_cast<const T *>(ct + code_bytes + 4 * act_sub);
#pragma unroll 2
        for (int bi = 0; bi < kMnbChunk; bi++) {
            const int u = ((bi ^ g) & 7) * 16 + 4 * t;
            const uint32_t w0 = *reinterpret_cast<const uint32_t *>(ct + r0 * 128 + u);
            const uint32_t w1 = *reinterpret_cast<const uint32_t *>(ct + (r0 + 8) * 128 + u);
            uint32_t q0[4], q1[4];
            dq_word<T>(w0, q0);
            dq_word<T>(w1, q1);
            const uint32_t p00 = q0[0], p10 = q1[0], p01 = q0[1], p11 = q1[1];
            const uint32_t p02 = q0[2], p12 = q1[2], p03 = q0[3], p13 = q1[3];
            const float sg = DT<T>::to_f32(st[r0 * kMnbChunk + bi]);
            const float sg8 = DT<T>::to_f32(st[(r0 + 8) * kMnbChunk + bi]);
            // activation row r of block bi: sub-tile bi/2, 16-byte unit (bi&1)*4 + t, swizzled with r & 7
            const unsigned char *ab = at + (bi >> 1) * act_sub + ((((bi & 1) * 4 + t) ^ g) & 7) * 16;
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                const int row = mt * 8 + g;
                uint4 x = make_uint4(0u, 0u, 0u, 0u);
                if (row < m) x = *reinterpret_cast<const uint4 *>(ab + row * 128);
                float acc[4];
                mma_16816<T>(acc, p00, p10, p01, p11, __byte_perm(x.x, x.z, 0x5410),
                             mnb_act_scale_odd<T>(__byte_perm(x.x, x.z, 0x7632)), true);
                mma_16816<T>(acc, p02, p12, p03, p13, __byte_perm(x.y, x.w, 0x5410),
                             mnb_act_scale_odd<T>(__byte_perm(x.y, x.w, 0x7632)), false);
                tot[mt][0] = fmaf(sg, acc[0], tot[mt][0]);
                tot[mt][1] = fmaf(sg, acc[1], tot[mt][1]);
                tot[mt][2] = fmaf(sg8, acc[2], tot[mt][2]);
                tot[mt][3] = fmaf(sg8, acc[3], tot[mt][3]);
            }
        }
        __syncthreads();  // every warp is done with this slot
        if (threadIdx.x == 0 && c + kMnbWideSlots < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            issue(c + kMnbWideSlots);
        }
    }
    if (!ok) {
        // chunk c never landed for some thread: let chunks c .. c + slots - 1 (issued, not consumed) land
        if (threadIdx.x == 0)
            for (int cc = c; cc < c + kMnbWideSlots && cc < nchunks; cc++)
                mbar_wait_bounded(full + cc % kMnbWideSlots, (uint32_t)((cc / kMnbWideSlots) & 1));
        return;
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int row = mt * 8 + 2 * t + (j & 1);
            const int col = n0 + r0 + ((j & 2) ? 8 : 0);
            if (row < m) {
                float v = tot[mt][j];
                if (bias) v += DT<T>::to_f32(bias[col]);
                st_from_f32(y + (int64_t)row * n + col, v);
            }
        }
    }
}

size_t mnb_wide_smem(int m) {
    const int mpad = (m + 7) & ~7;
    const size_t slot = 64 * 128 + 4 * (size_t)mpad * 128 + (((size_t)64 * kMnbChunk * 2 + 1023) & ~(size_t)1023);
    return 1024 + kMnbWideSlots * slot + kMnbWideSlots * 8;
}

template <typename T, int MT>
int launch_mma_wide(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m,
                    int64_t n, int64_t k, cudaStream_t stream) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(SA_ERR_CUDA, "MatMulNBits: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm_codes, tm_scales, tm_act;
    const cuuint32_t ones[2] = {1, 1};
    const cuuint64_t cdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n}, cstride[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t cbox[2] = {kMnbChunk * 16, 64};
    CUresult r = encode(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(b), cdim, cstride, cbox,
                        ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: code tensor map (%d)", (int)r);
    const cuuint64_t sdim[2] = {(cuuint64_t)(k / 32), (cuuint64_t)n}, sstride[1] = {(cuuint64_t)(k / 32) * 2};
    const cuuint32_t sbox[2] = {kMnbChunk, 64};
    r = encode(&tm_scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(scales), sdim, sstride, sbox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: scale tensor map (%d)", (int)r);
    const cuuint64_t adim[2] = {(cuuint64_t)k, (cuuint64_t)m}, astride[1] = {(cuuint64_t)k * 2};
    const cuuint32_t abox[2] = {64, (cuuint32_t)m};
    r = encode(&tm_act, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(a), adim, astride, abox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: activation tensor map (%d)", (int)r);
    const size_t smem = mnb_wide_smem((int)m);
    auto kern = mnb_mma_wide_kernel<T, MT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "MatMulNBits smem attribute");
    }
    kern<<<(unsigned)(n / 64), 32 * kMnbWideWarps, smem, stream>>>(tm_codes, tm_scales, tm_act,
                                                                  static_cast<const T *>(bias), static_cast<T *>(y),
                                                                  (int)m, (int)n, (int)k);
    count_launch();
    return check_cuda(cudaGetLastError(), "MatMulNBits wide mma launch");
}

// ---- prepacked weights -------------------------------------------------------
// Model weights are constant, so a host framework can repack them once at load
// (ONNX Runtime's MatMulNBits prepacks too).  The packed layout makes every
// chunk a warp streams one contiguous 9 KB run of HBM: per 32-column tile and
// per 16 k-blocks (512 codes), the 32 columns' 256-byte code runs followed by
// their 32 x 16 fp16 scales.  Inside a column's run, 16-byte unit u is stored
// at unit (u & 8) | ((u ^ column) & 7), so the fragment loads of 8 columns hit
// 32 distinct shared-memory banks.  A tile's chunks are consecutive.
constexpr int kPackCols = 32;                                 // columns per tile
constexpr int kPackBlocks = 16;                               // k-blocks per chunk
constexpr int kPackCodeBytes = kPackCols * kPackBlocks * 16;  // 8192
constexpr int kPackChunkBytes = kPackCodeBytes + kPackCols * kPackBlocks * 2;  // + scales = 9216
constexpr int kPackSplit = 2;                                 // warps (K splits) per CTA

__host__ __device__ inline int64_t pack_chunk_offset(int64_t tile, int64_t chunk, int64_t nchunks) {
    return (tile * nchunks + chunk) * kPackChunkBytes;
}

template <typename T>
__global__ void __launch_bounds__(256) mnb_prepack_kernel(const uint8_t *__restrict__ b, const T *__restrict__ scales,
                                                          uint8_t *__restrict__ packed, int n, int k) {
    const int64_t nchunks = k / (32 * kPackBlocks);
    const int64_t tile = blockIdx.y, chunk = blockIdx.x;
    uint8_t *dst = packed + pack_chunk_offset(tile, chunk, nchunks);
    const int nblk = k / 32;
    // codes: 32 columns x 16 units of 16 bytes
    for (int i = threadIdx.x; i < kPackCols * kPackBlocks; i += blockDim.x) {
        const int col = i / kPackBlocks, u = i % kPackBlocks;
        const int64_t ncol = tile * kPackCols + col;
        const uint4 v = *reinterpret_cast<const uint4 *>(b + ncol * (k / 2) + (chunk * kPackBlocks + u) * 16);
        const int us = (u & 8) | ((u ^ col) & 7);
        *reinterpret_cast<uint4 *>(dst + col * kPackBlocks * 16 + us * 16) = v;
    }
    // scales: [32 columns][16 blocks]
    T *sd = reinterpret_cast<T *>(dst + kPackCodeBytes);
    for (int i = threadIdx.x; i < kPackCols * kPackBlocks; i += blockDim.x) {
        const int col = i / kPackBlocks, bi = i % kPackBlocks;
        sd[i] = scales[(tile * kPackCols + col) * (int64_t)nblk + chunk * kPackBlocks + bi];
    }
}

// m <= 8 rows against prepacked weights: one CTA = one 32-column tile and
// kPackSplit warps splitting K; per chunk, one 1-D bulk copy of the packed
// run and two TMA copies of the m x 256 activation halves.
template <typename T>
__global__ void __launch_bounds__(32 * kPackSplit)
    mnb_packed_kernel(const uint8_t *__restrict__ packed, const __grid_constant__ CUtensorMap tm_act,
                      const T *__restrict__ bias, T *__restrict__ y, int m, int n, int k) {
    constexpr int NS = 2;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int act_row = kPackBlocks * 64;  // bytes of one activation row per chunk
    const int slot_bytes = kPackChunkBytes + ((m * act_row + 127) / 128) * 128;
    unsigned char *slots = smem + warp * NS * slot_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kPackSplit * NS * slot_bytes) + warp * NS;
    float *red = reinterpret_cast<float *>(smem + kPackSplit * NS * slot_bytes + kPackSplit * NS * 8);

    const int64_t tile = blockIdx.x;
    const int n0 = (int)tile * kPackCols;
    const int nchunks_all = k / (32 * kPackBlocks);
    const int nchunks = nchunks_all / kPackSplit;
    const int c0 = warp * nchunks;
    if (lane == 0) {
        for (int i = 0; i < NS; i++) mbar_init(bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int c) {  // lane 0: chunk c -> slot c % NS
        const int s = c % NS;
        unsigned char *dst = slots + s * slot_bytes;
        mbar_expect_tx(bars + s, kPackChunkBytes + m * act_row);
        bulk_g2s(dst, packed + pack_chunk_offset(tile, c0 + c, nchunks_all), kPackChunkBytes, bars + s);
        const int kk = (c0 + c) * kPackBlocks * 32;
        tma_load_2d(dst + kPackChunkBytes, &tm_act, kk, 0, bars + s);
        tma_load_2d(dst + kPackChunkBytes + m * 512, &tm_act, kk + 256, 0, bars + s);
    };
    if (lane == 0)
        for (int c = 0; c < NS && c < nchunks; c++) issue(c);

    float tot[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++) tot[nt][0] = tot[nt][1] = tot[nt][2] = tot[nt][3] = 0.0f;
    bool ok = true;
    int c = 0;
    for (; c < nchunks; c++) {
        const int s = c % NS;
        if (ok && !mbar_wait_bounded(bars + s, (uint32_t)((c / NS) & 1))) ok = false;
        if (__any_sync(0xffffffffu, !ok)) break;
        const unsigned char *ct = slots + s * slot_bytes;
        const unsigned char *sc = ct + kPackCodeBytes;
#pragma unroll
        for (int sb = 0; sb < 2; sb++) {
            const unsigned char *at = ct + kPackChunkBytes + sb * m * 512;  // [m][256] activations
            uint4 srow[2][2];
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                srow[nt][0] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g) * kPackBlocks * 2 + sb * 16);
                srow[nt][1] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g + 8) * kPackBlocks * 2 + sb * 16);
            }
#pragma unroll
            for (int bj = 0; bj < 8; bj++) {
                const int bi = sb * 8 + bj;
                uint4 x = make_uint4(0u, 0u, 0u, 0u);
                if (g < m) x = *reinterpret_cast<const uint4 *>(at + g * 512 + bj * 64 + 16 * t);
                const uint32_t bf0 = __byte_perm(x.x, x.z, 0x5410),
                               bf1 = mnb_act_scale_odd<T>(__byte_perm(x.x, x.z, 0x7632));
                const uint32_t bf2 = __byte_perm(x.y, x.w, 0x5410),
                               bf3 = mnb_act_scale_odd<T>(__byte_perm(x.y, x.w, 0x7632));
                const int u = ((bi & 8) | ((bi ^ g) & 7)) * 16 + 4 * t;  // same unit for rows g and g + 8
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const uint32_t w0 = *reinterpret_cast<const uint32_t *>(ct + (16 * nt + g) * 256 + u);
                    const uint32_t w1 = *reinterpret_cast<const uint32_t *>(ct + (16 * nt + g + 8) * 256 + u);
                    uint32_t q0[4], q1[4];
                    dq_word<T>(w0, q0);
                    dq_word<T>(w1, q1);
                    const uint32_t p00 = q0[0], p10 = q1[0], p01 = q0[1], p11 = q1[1];
                    const uint32_t p02 = q0[2], p12 = q1[2], p03 = q0[3], p13 = q1[3];
                    const uint32_t sw0 = (&srow[nt][0].x)[bj >> 1], sw1 = (&srow[nt][1].x)[bj >> 1];
                    const T s0 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw0) + (bj & 1));
                    const T s1 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw1) + (bj & 1));
                    float acc[4];
                    mma_16816<T>(acc, p00, p10, p01, p11, bf0, bf1, true);
                    mma_16816<T>(acc, p02, p12, p03, p13, bf2, bf3, false);
                    ffma2(tot[nt][0], tot[nt][1], DT<T>::to_f32(s0), acc[0], acc[1]);
                    ffma2(tot[nt][2], tot[nt][3], DT<T>::to_f32(s1), acc[2], acc[3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && c + NS < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            issue(c + NS);
        }
    }
    if (!ok && lane == 0)
        for (int cc = c; cc < c + NS && cc < nchunks; cc++)
            mbar_wait_bounded(bars + cc % NS, (uint32_t)((cc / NS) & 1));
    if (warp > 0) {
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) red[((warp - 1) * 32 + lane) * 8 + nt * 4 + j] = tot[nt][j];
    }
    __syncthreads();
    if (warp != 0 || !ok) return;
#pragma unroll
    for (int nt = 0; nt < 2; nt++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float v = tot[nt][j];
            for (int w = 1; w < kPackSplit; w++) v += red[((w - 1) * 32 + lane) * 8 + nt * 4 + j];
            const int row = 2 * t + (j & 1);
            const int col = n0 + 16 * nt + g + ((j & 2) ? 8 : 0);
            if (row < m) {
                if (bias) v += DT<T>::to_f32(bias[col]);
                st_from_f32(y + (int64_t)row * n + col, v);
            }
        }
    }
}

template <typename T>
int launch_packed(const void *a, const uint8_t *packed, const void *bias, void *y, int64_t m, int64_t n, int64_t k,
                  cudaStream_t stream) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(SA_ERR_CUDA, "MatMulNBits: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm_act;
    const cuuint64_t adim[2] = {(cuuint64_t)k, (cuuint64_t)m}, astride[1] = {(cuuint64_t)k * 2};
    const cuuint32_t abox[2] = {256, (cuuint32_t)m}, ones[2] = {1, 1};
    CUresult r = encode(&tm_act, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(a), adim, astride, abox, ones,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: activation tensor map (%d)", (int)r);
    const size_t slot = kPackChunkBytes + ((m * kPackBlocks * 64 + 127) / 128) * 128;
    const size_t smem = (size_t)kPackSplit * 2 * slot + kPackSplit * 2 * 8 + (size_t)(kPackSplit - 1) * 32 * 8 * 4;
    auto kern = mnb_packed_kernel<T>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "MatMulNBits packed smem attribute");
    }
    kern<<<(unsigned)(n / kPackCols), 32 * kPackSplit, smem, stream>>>(packed, tm_act, static_cast<const T *>(bias),
                                                                       static_cast<T *>(y), (int)m, (int)n, (int)k);
    count_launch();
    return check_cuda(cudaGetLastError(), "MatMulNBits packed launch");
}

// ---- decode GEMV path, m <= 4 rows -------------------------------------------
// The decode projections (one token per sequence, or a few) stream each weight
// byte once, so they are HBM-bound if the per-code arithmetic stays below the
// issue budget.  One CTA = 4 warps over 32 output columns; warp w reduces over
// the w-th quarter of K and streams its 32 columns' codes and scales through
// two shared-memory slots, 8 k-blocks (128 B of codes per column) per chunk:
// one 2-D TMA copy of the 32 x 128 B code tile (128-byte swizzle) and one of
// the 32 x 8 scales.  One ldmatrix.x4 gives a lane the fragment words of two
// k-blocks for its rows g and g + 8 (the swizzle keeps the eight rows of each
// 8 x 16 B matrix on distinct banks).  The dequant and the mma.m16n8k16 with
// exact products and fp32 block sums are those of mnb_mma_kernel; the block
// scale multiplies each block's sum in fp32.  The activation rows are turned
// into B fragments once per CTA (permuted to the dequant's k order, odd pairs
// pre-divided by 16 for fp16) and read with one 16-byte load per block.  The
// weight copies are issued before the kernel waits for the previous grid (it
// is a programmatic dependent launch): only the activations come from it.
constexpr int kGvSplit = 4;                          // warps per CTA, each over a quarter of K
constexpr int kGvCols = 32;                          // output columns per CTA (two 16-row MMA tiles)
constexpr int kGvChunk = 8;                          // k-blocks per chunk
constexpr int kGvSlots = 2;                          // chunks in flight per warp
constexpr int kGvCodeTile = kGvCols * 128;           // 4096 B, 1024-aligned for the swizzle
constexpr int kGvScaleTile = kGvCols * kGvChunk * 2; // 512 B
// One activation row: with more rows the staged fragments push the CTA past four per SM and
// the K-split kernel below is as fast (B200, C2 shape: m = 2 and 4 measured 14.1 and 14.6 us
// here, with two warps of four slots 12.4 and 18.8 us).
constexpr int kGvMaxM = 1;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <typename T>
__global__ void __launch_bounds__(32 * kGvSplit)
    mnb_gemv_tc_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_scales,
                       const T *__restrict__ a, const T *__restrict__ bias, T *__restrict__ y, int m, int n, int k) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nblk = k / 32;
    const int nbw = nblk / kGvSplit;  // k-blocks of this warp: a multiple of kGvChunk
    const int nchunks = nbw / kGvChunk;
    unsigned char *codes = smem + warp * kGvSlots * kGvCodeTile;
    unsigned char *scl = smem + kGvSplit * kGvSlots * kGvCodeTile + warp * kGvSlots * kGvScaleTile;
    uint4 *afrag = reinterpret_cast<uint4 *>(smem + kGvSplit * kGvSlots * (kGvCodeTile + kGvScaleTile));
    uint64_t *bar_base = reinterpret_cast<uint64_t *>(afrag + (size_t)nblk * 4 * m);
    uint64_t *bars = bar_base + warp * kGvSlots;
    uint64_t *act_bar = bar_base + kGvSplit * kGvSlots;
    float *red = reinterpret_cast<float *>(act_bar + 1);
    const int n0 = blockIdx.x * kGvCols;
    const int b0 = warp * nbw;
    if (lane == 0) {
        for (int i = 0; i < kGvSlots; i++) mbar_init(bars + i, 1);
        if (warp == 0) mbar_init(act_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    auto issue = [&](int c) {  // lane 0: chunk c -> slot c % kGvSlots
        const int s = c % kGvSlots;
        const int blk = b0 + c * kGvChunk;
        mbar_expect_tx(bars + s, kGvCodeTile + kGvScaleTile);
        tma_load_2d(codes + s * kGvCodeTile, &tm_codes, blk * 16, n0, bars + s);
        tma_load_2d(scl + s * kGvScaleTile, &tm_scales, blk, n0, bars + s);
    };
    // the weights do not depend on the kernel before this one: start streaming them now
    if (lane == 0)
        for (int c = 0; c < kGvSlots && c < nchunks; c++) issue(c);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the activations
    // The m activation rows, one bulk copy each, then every 16-byte unit turned in place into the B
    // fragment words of its k-block: [row][blk][t] = halves 8t..8t+7 as (h0,h4), (h1,h5)/16,
    // (h2,h6), (h3,h7)/16 (the dequant's pair order; the 1/16 meets the in-place fp16 high nibbles).
    if (threadIdx.x == 0) {
        mbar_expect_tx(act_bar, (uint32_t)(m * k * 2));
        for (int r = 0; r < m; r++)
            bulk_g2s(afrag + (size_t)r * nblk * 4, a + (int64_t)r * k, (uint32_t)(k * 2), act_bar);
    }
    bool ok = mbar_wait_bounded(act_bar, 0u);
    if (ok) {
        for (int i = threadIdx.x; i < nblk * 4 * m; i += blockDim.x) {
            const uint4 x = afrag[i];
            uint4 f;
            f.x = __byte_perm(x.x, x.z, 0x5410);
            f.y = mnb_act_scale_odd<T>(__byte_perm(x.x, x.z, 0x7632));
            f.z = __byte_perm(x.y, x.w, 0x5410);
            f.w = mnb_act_scale_odd<T>(__byte_perm(x.y, x.w, 0x7632));
            afrag[i] = f;
        }
    }
    __syncthreads();

    // ldmatrix row addresses: lane L feeds row (L & 7) + 8 * ((L >> 3) & 1) of a 16-row tile, at
    // 16-byte unit (block) + (L >> 4); the 128-byte swizzle puts unit u of row r at u ^ (r & 7)
    const int lrow = (lane & 7) + 8 * ((lane >> 3) & 1), lunit = lane >> 4;
    const bool has_row = g < m;
    float tot[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++) tot[nt][0] = tot[nt][1] = tot[nt][2] = tot[nt][3] = 0.0f;
    int c = 0;
    for (; c < nchunks; c++) {
        const int s = c % kGvSlots;
        if (ok && !mbar_wait_bounded(bars + s, (uint32_t)((c / kGvSlots) & 1))) ok = false;
        if (__any_sync(0xffffffffu, !ok)) break;  // a copy never landed: give up (output left unwritten)
        const uint32_t ct = smem_u32(codes + s * kGvCodeTile);
        const unsigned char *sc = scl + s * kGvScaleTile;
        // this lane's scales of the chunk's 8 blocks, rows 16 nt + g and 16 nt + g + 8
        uint4 srow[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            srow[nt][0] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g) * kGvChunk * 2);
            srow[nt][1] = *reinterpret_cast<const uint4 *>(sc + (16 * nt + g + 8) * kGvChunk * 2);
        }
        const int blk0 = b0 + c * kGvChunk;
#pragma unroll
        for (int bp = 0; bp < kGvChunk; bp += 2) {
            uint4 bf[2];
#pragma unroll
            for (int h = 0; h < 2; h++)
                bf[h] = has_row ? afrag[((size_t)g * nblk + blk0 + bp + h) * 4 + t] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                const int row = 16 * nt + lrow;
                uint32_t w[4];  // rows g, g+8 of block bp; rows g, g+8 of block bp+1
                ldsm_x4(w, ct + row * 128 + (((bp + lunit) ^ (row & 7)) << 4));
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    uint32_t q0[4], q1[4];
                    dq_word<T>(w[2 * h], q0);
                    dq_word<T>(w[2 * h + 1], q1);
                    const int bi = bp + h;
                    const uint32_t sw0 = (&srow[nt][0].x)[bi >> 1], sw1 = (&srow[nt][1].x)[bi >> 1];
                    const T s0 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw0) + (bi & 1));
                    const T s1 = *reinterpret_cast<const T *>(reinterpret_cast<const uint16_t *>(&sw1) + (bi & 1));
                    float acc[4];
                    mma_16816<T>(acc, q0[0], q1[0], q0[1], q1[1], bf[h].x, bf[h].y, true);
                    mma_16816<T>(acc, q0[2], q1[2], q0[3], q1[3], bf[h].z, bf[h].w, false);
                    ffma2(tot[nt][0], tot[nt][1], DT<T>::to_f32(s0), acc[0], acc[1]);
                    ffma2(tot[nt][2], tot[nt][3], DT<T>::to_f32(s1), acc[2], acc[3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && c + kGvSlots < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            issue(c + kGvSlots);
        }
    }
    if (!ok && lane == 0) {
        // a copy never landed: let this warp's copies still in flight land (bounded)
        for (int cc = c; cc < c + kGvSlots && cc < nchunks; cc++)
            mbar_wait_bounded(bars + cc % kGvSlots, (uint32_t)((cc / kGvSlots) & 1));
        if (warp == 0) mbar_wait_bounded(act_bar, 0u);
    }
    // sum the K quarters: warps 1.. leave their sums in shared memory, warp 0 adds and stores
    if (warp > 0) {
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) red[((warp - 1) * 32 + lane) * 8 + nt * 4 + j] = tot[nt][j];
    }
    const int bad = __syncthreads_or(!ok);
    if (warp != 0 || bad) return;
#pragma unroll
    for (int nt = 0; nt < 2; nt++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int row = 2 * t + (j & 1);
            if (row < m) {
                float v = tot[nt][j];
#pragma unroll
                for (int w = 1; w < kGvSplit; w++) v += red[((w - 1) * 32 + lane) * 8 + nt * 4 + j];
                const int col = n0 + 16 * nt + g + ((j & 2) ? 8 : 0);
                if (bias) v += DT<T>::to_f32(bias[col]);
                st_from_f32(y + (int64_t)row * n + col, v);
            }
        }
    }
}

size_t mnb_gemv_tc_smem(int64_t m, int64_t k) {
    return 1024 + (size_t)kGvSplit * kGvSlots * (kGvCodeTile + kGvScaleTile) + (size_t)(k / 32) * 4 * m * 16 +
           (kGvSplit * kGvSlots + 1) * 8 + (size_t)(kGvSplit - 1) * 32 * 8 * 4;
}

bool mnb_gemv_tc_eligible(int64_t m, int64_t n, int64_t k) {
    return m >= 1 && m <= kGvMaxM && n % kGvCols == 0 && k % (32 * kGvSplit * kGvChunk) == 0 &&
           mnb_gemv_tc_smem(m, k) <= 200 * 1024;
}

template <typename T>
int launch_gemv_tc(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m, int64_t n,
                   int64_t k, cudaStream_t stream) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return set_error(SA_ERR_CUDA, "MatMulNBits: cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm_codes, tm_scales;
    const cuuint32_t ones[2] = {1, 1};
    const cuuint64_t cdim[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n}, cstride[1] = {(cuuint64_t)(k / 2)};
    const cuuint32_t cbox[2] = {kGvChunk * 16, kGvCols};
    CUresult r = encode(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(b), cdim, cstride, cbox,
                        ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: code tensor map (%d)", (int)r);
    const cuuint64_t sdim[2] = {(cuuint64_t)(k / 32), (cuuint64_t)n}, sstride[1] = {(cuuint64_t)(k / 32) * 2};
    const cuuint32_t sbox[2] = {kGvChunk, kGvCols};
    r = encode(&tm_scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(scales), sdim, sstride, sbox, ones,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "MatMulNBits: scale tensor map (%d)", (int)r);
    const size_t smem = mnb_gemv_tc_smem(m, k);
    auto kern = mnb_gemv_tc_kernel<T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "MatMulNBits gemv smem attribute");
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n / kGvCols));
    cfg.blockDim = dim3(32 * kGvSplit);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tm_codes, tm_scales, static_cast<const T *>(a), static_cast<const T *>(bias),
                           static_cast<T *>(y), (int)m, (int)n, (int)k);
    count_launch();
    return check_cuda(e, "MatMulNBits gemv launch");
}

template <typename T>
int launch_mma_rows(const void *a, const uint8_t *b, const void *scales, const void *bias, void *y, int64_t m,
                    int64_t n, int64_t k, cudaStream_t stream) {
    if (mnb_gemv_tc_eligible(m, n, k)) return launch_gemv_tc<T>(a, b, scales, bias, y, m, n, k, stream);
    if (m <= 8) {
        // (chunks of two 128-byte sub-tiles per row, SUB = 2, measured slower on B200: 20.8 vs 16.8 us at m = 8)
        if (n % 32 == 0) return launch_mma<T, 1, 2>(a, b, scales, bias, y, m, n, k, stream);
        return launch_mma<T, 1, 1>(a, b, scales, bias, y, m, n, k, stream);
    }
    if (m <= 16) return launch_mma<T, 2, 1>(a, b, scales, bias, y, m, n, k, stream);
    if (n % 64 == 0) {  // the CTA shares one activation tile among 64 columns
        if (m <= 32) return launch_mma_wide<T, 4>(a, b, scales, bias, y, m, n, k, stream);
        return launch_mma_wide<T, 8>(a, b, scales, bias, y, m, n, k, stream);
    }
    if (m <= 32) return launch_mma<T, 4, 1>(a, b, scales, bias, y, m, n, k, stream);
    return launch_mma<T, 8, 1>(a, b, scales, bias, y, m, n, k, stream);
}

// The tensor-core path takes fp16/bf16 activations with block 32, no zero
// points, m <= 64, N a multiple of 16 and K a multiple of 1024 (whole chunks
// per warp), the codes, activations and scales 16-byte aligned.
bool mnb_mma_eligible(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, int dtype,
                      int64_t m, int64_t n, int64_t k, int block_size) {
    if (dtype != SA_DTYPE_FLOAT16 && dtype != SA_DTYPE_BFLOAT16) return false;
    if (zp || block_size != 32 || m < 1 || m > 64) return false;
    if (n % 16 != 0 || k % (32 * kMnbMaxSplit * kMnbChunk) != 0 || n > (1 << 30) || k > (1 << 24)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(scales);
    return (al & 15) == 0;
}

template <typename T>
int launch_t(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, const void *bias, void *y,
             int64_t m, int64_t n, int64_t k, int block_size, cudaStream_t stream) {
    if (k % 32 != 0) return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: K must be a multiple of 32");
    if ((reinterpret_cast<uintptr_t>(b) & 15) != 0 || ((k / 2) % 16) != 0)
        return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: packed B rows must be 16-byte aligned");
    const int64_t blocks = (n + kGemvWarps - 1) / kGemvWarps;
    for (int64_t m0 = 0; m0 < m; m0 += 8) {
        const int64_t mt = m - m0;
        dim3 grid((unsigned)blocks), block(32 * kGemvWarps);
        const T *A = static_cast<const T *>(a);
        const T *S = static_cast<const T *>(scales);
        const T *Bi = static_cast<const T *>(bias);
        T *Y = static_cast<T *>(y);
        if (mt == 1)
            mnb_gemv_kernel<T, 1><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else if (mt <= 2)
            mnb_gemv_kernel<T, 2><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else if (mt <= 4)
            mnb_gemv_kernel<T, 4><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        else
            mnb_gemv_kernel<T, 8><<<grid, block, 0, stream>>>(A, b, S, zp, Bi, Y, m, m0, n, k, block_size);
        count_launch();
        int rc = check_cuda(cudaGetLastError(), "MatMulNBits gemv launch");
        if (rc != SA_OK) return rc;
    }
    return SA_OK;
}

}  // namespace

int launch_matmul_nbits(const void *a, const uint8_t *b, const void *scales, const uint8_t *zp, const void *bias,
                        void *y, int dtype, int64_t m, int64_t n, int64_t k, int block_size, cudaStream_t stream) {
    if (matmul_nbits_umma_eligible(a, b, scales, zp, dtype, m, n, k, block_size))
        return launch_matmul_nbits_umma(a, b, scales, bias, y, dtype, m, n, k, stream);
    if (mnb_mma_eligible(a, b, scales, zp, dtype, m, n, k, block_size)) {
        if (dtype == SA_DTYPE_FLOAT16) return launch_mma_rows<__half>(a, b, scales, bias, y, m, n, k, stream);
        return launch_mma_rows<__nv_bfloat16>(a, b, scales, bias, y, m, n, k, stream);
    }
    switch (dtype) {
        case SA_DTYPE_FLOAT: return launch_t<float>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        case SA_DTYPE_FLOAT16: return launch_t<__half>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        case SA_DTYPE_BFLOAT16:
            return launch_t<__nv_bfloat16>(a, b, scales, zp, bias, y, m, n, k, block_size, stream);
        default: return set_error(SA_ERR_UNSUPPORTED, "MatMulNBits: dtype %d not supported", dtype);
    }
}

bool matmul_nbits_packable(int dtype, int64_t n, int64_t k, int block_size) {
    return (dtype == SA_DTYPE_FLOAT16 || dtype == SA_DTYPE_BFLOAT16) && block_size == 32 && n > 0 &&
           n % kPackCols == 0 && k > 0 && k % (32 * kPackBlocks * kPackSplit) == 0 && n <= (1 << 30) &&
           k <= (1 << 24);
}

size_t matmul_nbits_packed_bytes(int64_t n, int64_t k) {
    return (size_t)(n / kPackCols) * (size_t)(k / (32 * kPackBlocks)) * kPackChunkBytes;
}

int launch_matmul_nbits_prepack(const uint8_t *b, const void *scales, void *packed, int dtype, int64_t n, int64_t k,
                                cudaStream_t stream) {
    const dim3 grid((unsigned)(k / (32 * kPackBlocks)), (unsigned)(n / kPackCols));
    if (dtype == SA_DTYPE_FLOAT16)
        mnb_prepack_kernel<__half><<<grid, 256, 0, stream>>>(b, static_cast<const __half *>(scales),
                                                            static_cast<uint8_t *>(packed), (int)n, (int)k);
    else
        mnb_prepack_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(b, static_cast<const __nv_bfloat16 *>(scales),
                                                                   static_cast<uint8_t *>(packed), (int)n, (int)k);
    count_launch();
    return check_cuda(cudaGetLastError(), "MatMulNBits prepack launch");
}

int launch_matmul_nbits_packed(const void *a, const void *packed, const void *bias, void *y, int dtype, int64_t m,
                               int64_t n, int64_t k, cudaStream_t stream) {
    const uint8_t *p = static_cast<const uint8_t *>(packed);
    if (dtype == SA_DTYPE_FLOAT16) return launch_packed<__half>(a, p, bias, y, m, n, k, stream);
    return launch_packed<__nv_bfloat16>(a, p, bias, y, m, n, k, stream);
}

}  // namespace sa

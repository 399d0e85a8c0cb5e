// kquant.cu -- the dequant seam on the GPU (roofline.c src/dequant.c:5-80,
// with the Q4_K / Q6_K arms of ggml's block formats) and the fused K-quant
// dequant-matvec.
//
// Layout of one warp's work: a group of 8 superblocks (1152 B of Q4_K or
// 1680 B of Q6_K) is loaded with 128-bit loads while the previous group is
// decoded, then copied to shared memory, and every lane decodes 8 consecutive
// weights of each superblock (lane l owns weights 8l..8l+7) and writes them as
// two float4.
// Arithmetic is the rounding sequence of the C restatement with no
// contraction: Q4_K w = (d*sc)*q - (dmin*m), Q6_K w = (d*sc)*q.
#include "tcg_common.cuh"
#include "tcg_internal.h"
#include "numerics.cuh"

#include <cuda_fp16.h>
#include <string.h>

namespace tcg {

constexpr int QK = 256;
constexpr int GROUP = 8;          // superblocks staged per warp
constexpr int WARPS = 8;          // warps per CTA

template <int TYPE> struct KQ;
template <> struct KQ<GGML_TYPE_Q4_K> { static constexpr int BYTES = 144; };
template <> struct KQ<GGML_TYPE_Q6_K> { static constexpr int BYTES = 210; };

// Packed fp32 pairs (low word = first element), each half rounded to nearest
// like the scalar instruction.
typedef unsigned long long u64;
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c)
{
    u64 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b)
{
    u64 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// bytes j and j+1 of w as the float pair (2^23 + byte_j, 2^23 + byte_j+1)
__device__ __forceinline__ u64 magic2(uint32_t w, int j)
{
    const uint32_t a = __byte_perm(w, 0x4B000000u, 0x7440u | (unsigned)j);
    const uint32_t b = __byte_perm(w, 0x4B000000u, 0x7440u | (unsigned)(j + 1));
    return (u64)a | ((u64)b << 32);
}

// Exact binary16 -> binary32 by bit manipulation (tc_f16_to_f32,
// src/dequant.c:5-38): subnormals renormalised, NaN payloads kept.
__device__ __forceinline__ float f16_to_f32_exact(uint32_t h)
{
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, f = h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (f << 13);
    } else if (e != 0u) {
        bits = sign | ((e + 112u) << 23) | (f << 13);
    } else if (f == 0u) {
        bits = sign;
    } else {
        const uint32_t shift = 10u - (31u - (uint32_t)__clz(f));  // leading one to bit 10
        bits = sign | ((113u - shift) << 23) | (((f << shift) & 0x3FFu) << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t ld_u8(const uint8_t *s, int i) { return s[i]; }
__device__ __forceinline__ uint32_t ld_u16(const uint8_t *s, int i) { return (uint32_t)s[i] | ((uint32_t)s[i + 1] << 8); }

// Copy `bytes` bytes from global to this warp's shared buffer using the
// widest load the source alignment allows. `bytes` is even for every caller.
__device__ __forceinline__ void stage(uint8_t *dst, const uint8_t *src, int bytes, int lane)
{
    if (((uintptr_t)src & 15) == 0 && (bytes & 15) == 0) {
        const uint4 *s = reinterpret_cast<const uint4 *>(src);
        uint4 *d = reinterpret_cast<uint4 *>(dst);
        for (int i = lane; i < bytes / 16; i += 32) d[i] = __ldg(s + i);
    } else if (((uintptr_t)src & 1) == 0) {
        const uint16_t *s = reinterpret_cast<const uint16_t *>(src);
        uint16_t *d = reinterpret_cast<uint16_t *>(dst);
        for (int i = lane; i < bytes / 2; i += 32) d[i] = __ldg(s + i);
    } else {
        for (int i = lane; i < bytes; i += 32) dst[i] = __ldg(src + i);
    }
}

// The 8 weights of superblock `b` (staged at `blk`) that belong to `lane`.
template <int TYPE>
__device__ __forceinline__ void decode8(const uint8_t *blk, int lane, float w[8]);

template <>
__device__ __forceinline__ void decode8<GGML_TYPE_Q4_K>(const uint8_t *blk, int lane, float w[8])
{
    // lane = 8g + 4*half + p/8: group g of 64, low (half 0) or high nibbles,
    // bytes p..p+7 of that group's 32 quant bytes.
    const int g = lane >> 3, half = (lane >> 2) & 1, p = (lane & 3) * 8;
    const float d = f16_to_f32_exact(ld_u16(blk, 0));
    const float dmin = f16_to_f32_exact(ld_u16(blk, 2));
    const uint8_t *s = blk + 4;
    const int j = 2 * g + half;
    int sc, mn;
    if (j < 4) {
        sc = s[j] & 0x3F;
        mn = s[j + 4] & 0x3F;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const float a = __fmul_rn(d, (float)sc);
    const float c = __fmul_rn(dmin, (float)mn);
    const uint8_t *q = blk + 16 + 32 * g + p;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int nib = half ? (q[i] >> 4) : (q[i] & 0x0F);
        w[i] = __fsub_rn(__fmul_rn(a, (float)nib), c);
    }
}

template <>
__device__ __forceinline__ void decode8<GGML_TYPE_Q6_K>(const uint8_t *blk, int lane, float w[8])
{
    // lane = 16h + i/8 with i = 32r + l0: half h, row r of 32, offset l0.
    const int h = lane >> 4, i0 = (lane & 15) * 8, r = i0 >> 5, l0 = i0 & 31;
    const uint8_t *ql = blk + 64 * h + l0 + 32 * (r & 1);
    const uint8_t *qh = blk + 128 + 32 * h + l0;
    const int8_t sc = (int8_t)blk[192 + 8 * h + 2 * r + (l0 >> 4)];
    const float d = f16_to_f32_exact(ld_u16(blk, 208));
    const float s = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int lo = (r < 2) ? (ql[i] & 0x0F) : (ql[i] >> 4);
        const int hi = (qh[i] >> (2 * r)) & 3;
        w[i] = __fmul_rn(s, (float)((lo | (hi << 4)) - 32));
    }
}

// Warps stride over chunks of GROUP superblocks (chunk c to warp c mod
// warps, so the grid sweeps one contiguous window of the tensor). The
// 16-byte-aligned span covering a warp's next chunk is loaded into registers
// while the current one is decoded from its shared buffer (an aligned 16-byte
// word that holds a byte of the tensor lies in the same page as that byte, so
// the span's edges cannot fault); each lane writes its 8 weights of every
// superblock as two float4.
// With SPLIT, each weight goes out as its tf32 pair instead (dst the hi
// half, lo the lo half): the operand a 3xTF32 GEMM reads.
template <int TYPE, bool SPLIT = false>
__global__ void __launch_bounds__(WARPS * 32)
dequant_kq_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst, size_t nblocks, float *__restrict__ lo = nullptr)
{
    constexpr int BB = KQ<TYPE>::BYTES;
    constexpr int C = GROUP;
    constexpr int SPAN = (C * BB + 30) / 16 * 16;            // bytes of the widest aligned span
    constexpr int LPL = (SPAN / 16 + 31) / 32;               // 16-byte loads per lane
    __shared__ __align__(16) uint8_t buf[WARPS][SPAN];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const size_t nw = (size_t)gridDim.x * WARPS;
    const size_t nchunks = (nblocks + C - 1) / C;
    const uintptr_t base = (uintptr_t)src;
    uint4 r[LPL];
    auto span = [&](size_t c, uintptr_t &a0, size_t &b0, int &nb) {
        b0 = c * C;
        nb = (int)min((size_t)C, nblocks - b0);
        a0 = (base + b0 * BB) & ~(uintptr_t)15;
        return (int)((((base + (b0 + nb) * BB + 15) & ~(uintptr_t)15) - a0) / 16);
    };
    auto load = [&](size_t c) {
        uintptr_t a0; size_t b0; int nb;
        const int n16 = span(c, a0, b0, nb);
#pragma unroll
        for (int u = 0; u < LPL; u++)
            if (lane + 32 * u < n16) r[u] = __ldg(reinterpret_cast<const uint4 *>(a0) + lane + 32 * u);
    };
    size_t c = (size_t)blockIdx.x * WARPS + wid;
    if (c < nchunks) load(c);
    for (; c < nchunks; c += nw) {
        uintptr_t a0; size_t b0; int nb;
        const int n16 = span(c, a0, b0, nb);
        const int off = (int)((base + b0 * BB) - a0);
        __syncwarp();                                        // the previous chunk is decoded
#pragma unroll
        for (int u = 0; u < LPL; u++)
            if (lane + 32 * u < n16) reinterpret_cast<uint4 *>(buf[wid])[lane + 32 * u] = r[u];
        __syncwarp();
        if (c + nw < nchunks) load(c + nw);                  // in flight during the decode below
        for (int b = 0; b < nb; b++) {
            float w[8];
            decode8<TYPE>(buf[wid] + off + b * BB, lane, w);
            float4 *o = reinterpret_cast<float4 *>(dst + (b0 + b) * QK + 8 * lane);
            if constexpr (SPLIT) {
                float h[8], l[8];
#pragma unroll
                for (int i = 0; i < 8; i++) split_tf32(w[i], h[i], l[i]);
                float4 *ol = reinterpret_cast<float4 *>(lo + (b0 + b) * QK + 8 * lane);
                o[0] = make_float4(h[0], h[1], h[2], h[3]);
                o[1] = make_float4(h[4], h[5], h[6], h[7]);
                ol[0] = make_float4(l[0], l[1], l[2], l[3]);
                ol[1] = make_float4(l[4], l[5], l[6], l[7]);
            } else {
                o[0] = make_float4(w[0], w[1], w[2], w[3]);
                o[1] = make_float4(w[4], w[5], w[6], w[7]);
            }
        }
    }
}

__global__ void f16_to_f32_kernel(const uint16_t *__restrict__ src, float *__restrict__ dst, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = f16_to_f32_exact(src[i]);
}

// y[row] = sum_k W[row, k] x[k]. WPR warps share a row: warp w of the row
// takes superblock groups w, w+WPR, ...; partial sums meet in shared memory.
template <int TYPE, int WPR>
__global__ void __launch_bounds__(WARPS * 32)
matvec_kq_kernel(const uint8_t *__restrict__ W, const float *__restrict__ x, float *__restrict__ y,
                 int N, int K)
{
    constexpr int BB = KQ<TYPE>::BYTES;
    constexpr int ROWS = WARPS / WPR;           // rows per CTA pass
    __shared__ __align__(16) uint8_t buf[WARPS][GROUP * BB];
    __shared__ float part[WARPS];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int sub = wid % WPR, slot = wid / WPR;
    const int bpr = K / QK;                      // superblocks per row
    const int gpr = (bpr + GROUP - 1) / GROUP;   // groups per row
    const size_t row_bytes = (size_t)bpr * BB;

    for (int row0 = blockIdx.x * ROWS; row0 < N; row0 += gridDim.x * ROWS) {
        const int row = row0 + slot;
        float acc = 0.0f;
        if (row < N) {
            const uint8_t *wr = W + (size_t)row * row_bytes;
            for (int g = sub; g < gpr; g += WPR) {
                const int nb = min(GROUP, bpr - g * GROUP);
                stage(buf[wid], wr + (size_t)g * GROUP * BB, nb * BB, lane);
                __syncwarp();
                for (int b = 0; b < nb; b++) {
                    float w[8];
                    decode8<TYPE>(buf[wid] + b * BB, lane, w);
                    const float4 *xv = reinterpret_cast<const float4 *>(x + (size_t)(g * GROUP + b) * QK + 8 * lane);
                    const float4 x0 = __ldg(xv), x1 = __ldg(xv + 1);
                    acc = fmaf(w[0], x0.x, acc); acc = fmaf(w[1], x0.y, acc);
                    acc = fmaf(w[2], x0.z, acc); acc = fmaf(w[3], x0.w, acc);
                    acc = fmaf(w[4], x1.x, acc); acc = fmaf(w[5], x1.y, acc);
                    acc = fmaf(w[6], x1.z, acc); acc = fmaf(w[7], x1.w, acc);
                }
                __syncwarp();
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (WPR == 1) {
            if (lane == 0 && row < N) y[row] = acc;
        } else {
            if (lane == 0) part[wid] = acc;
            __syncthreads();
            if (sub == 0 && lane == 0 && row < N) {
                float s = 0.0f;
                for (int i = 0; i < WPR; i++) s += part[slot * WPR + i];
                y[row] = s;
            }
            __syncthreads();
        }
    }
}

// ----------------------------------------------------- streaming matvec
// Persistent CTAs of 16 warps, one per SM. x stays in shared memory for the
// whole launch, its float4 units XOR-swizzled so that the x loads of a warp
// spread over all eight 16-byte bank groups (for Q4_K also the sum of every 32
// consecutive x, for the min term). Every warp streams its weight segments (a
// part of a row of Q4_K, a whole row of Q6_K) through a cp.async ring of two to four slots
// and computes one slot while the next lands. Four lanes share a superblock,
// 64 weights per lane (its scales decoded once), and a warp works on eight
// consecutive superblocks at a time. The quant bytes are turned into floats 2^23 + q with byte permutes,
// shifted back exactly with packed f32x2 adds, and dotted with x by packed
// f32x2 FMAs:
//   Q4_K  sum (a q - c) x  =  a * sum(q x) - c * sum(x)   per sub-block of 32
//   Q6_K  sum (d sc) q x   =  (d sc) * sum(q x)           per sub-block of 16
constexpr int MV_WARPS = 24;       // 24 warps: Q6_K 3% faster than 16; 32 (64 registers) spills

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }


// sum_i (v_i - off) x_i over the 8 bytes v of (w0, w1); x 16-byte aligned in
// shared memory; neg_off2 holds -(2^23 + off) twice.
__device__ __forceinline__ float dot8(uint32_t w0, uint32_t w1, u64 neg_off2, const float *x)
{
    const ulonglong2 xa = *reinterpret_cast<const ulonglong2 *>(x);
    const ulonglong2 xb = *reinterpret_cast<const ulonglong2 *>(x + 4);
    u64 acc = 0ull;
    acc = fma2(add2(magic2(w0, 0), neg_off2), xa.x, acc);
    acc = fma2(add2(magic2(w0, 2), neg_off2), xa.y, acc);
    acc = fma2(add2(magic2(w1, 0), neg_off2), xb.x, acc);
    acc = fma2(add2(magic2(w1, 2), neg_off2), xb.y, acc);
    return __uint_as_float((uint32_t)acc) + __uint_as_float((uint32_t)(acc >> 32));
}


// x is stored by float4 unit u at u ^ swz(u): Q4_K lanes differ in u's bits
// 2 (half of a 32-weight group), 4-5 (group) and 6-7 (superblock); Q6_K lanes
// in bits 1-2, 5 and 6-7. XOR-ing the bank-group bits 0-2 with bits 4-6 (Q4_K)
// or 5-7 (Q6_K) leaves at most four distinct units per bank group in a warp's
// float4 load, the minimum for 512 bytes.
template <int TYPE>
__device__ __forceinline__ int xswz(int u)
{
    return TYPE == GGML_TYPE_Q4_K ? u ^ ((u >> 4) & 7) : u ^ ((u >> 5) & 7);
}

// acc += sum over the 8 bytes v of (w0, w1) of (v - off) * x, x in xa, xb
// (four f32x2 pairs); neg_off2 holds -(2^23 + off) twice.
__device__ __forceinline__ u64 dot8acc(uint32_t w0, uint32_t w1, u64 neg_off2, ulonglong2 xa, ulonglong2 xb, u64 acc)
{
    acc = fma2(add2(magic2(w0, 0), neg_off2), xa.x, acc);
    acc = fma2(add2(magic2(w0, 2), neg_off2), xa.y, acc);
    acc = fma2(add2(magic2(w1, 0), neg_off2), xb.x, acc);
    acc = fma2(add2(magic2(w1, 2), neg_off2), xb.y, acc);
    return acc;
}
__device__ __forceinline__ float pair_sum(u64 a)
{
    return __uint_as_float((uint32_t)a) + __uint_as_float((uint32_t)(a >> 32));
}
// the float4 unit at physical index u of the swizzled x
__device__ __forceinline__ ulonglong2 ldxu(const float *xs, int u)
{
    return reinterpret_cast<const ulonglong2 *>(xs)[u];
}

// Lane g (0..3) of Q4_K superblock b in R rows at once (their copies in the
// ring rstride bytes apart): its 32 quant bytes 32g .. 32g + 31 of a row hold
// weights 64g + i of sub-block 2g (low nibbles) and 64g + 32 + i of sub-block
// 2g + 1 (high nibbles), i < 32. Every x load serves the R rows, which halves
// the shared-memory traffic of x (4 bytes per weight, against 0.56 bytes of
// quants) at R = 2. x unit 64b + 16g + m (+ 8 for the high half) sits at
// physical unit (64b + 16g + 8 hi) + (m ^ f), f = (4b + g) & 7. acc[r] gains
// the row's partial dot product.
template <int R>
__device__ __forceinline__ void lane_dot_q4k(const uint8_t *blk, int rstride, int g, const float *xs,
                                             const float *x32, int b, float *acc)
{
    const int k = 2 * (g & 1);
    float a[R][2], c[R][2];
    uint32_t w[R][8];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const uint8_t *p = blk + r * rstride;
        const uint4 hd = *reinterpret_cast<const uint4 *>(p);
        const uint4 qa = *reinterpret_cast<const uint4 *>(p + 16 + 32 * g);
        const uint4 qb = *reinterpret_cast<const uint4 *>(p + 32 + 32 * g);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint32_t by = (hd.y >> (8 * (k + u))) & 0xFFu, bz = (hd.z >> (8 * (k + u))) & 0xFFu;
            const uint32_t bw = (hd.w >> (8 * (k + u))) & 0xFFu;
            const uint32_t sc = g < 2 ? (by & 63u) : ((bw & 15u) | ((by >> 6) << 4));
            const uint32_t mn = g < 2 ? (bz & 63u) : ((bw >> 4) | ((bz >> 6) << 4));
            a[r][u] = d * (float)sc;
            c[r][u] = dmin * (float)mn;
        }
        w[r][0] = qa.x; w[r][1] = qa.y; w[r][2] = qa.z; w[r][3] = qa.w;
        w[r][4] = qb.x; w[r][5] = qb.y; w[r][6] = qb.z; w[r][7] = qb.w;
    }
    const u64 neg = 0xCB000000CB000000ull;          // (-2^23, -2^23)
    const int base = 64 * b + 16 * g, f = (4 * b + g) & 7;
    // four independent accumulator chains per row (low/high nibbles x
    // even/odd words) so that the permute -> subtract -> FMA latency of one
    // overlaps the others
    u64 al0[R], al1[R], ah0[R], ah1[R];
#pragma unroll
    for (int r = 0; r < R; r++) al0[r] = al1[r] = ah0[r] = ah1[r] = 0ull;
#pragma unroll
    for (int m = 0; m < 8; m += 2) {
        const ulonglong2 l0 = ldxu(xs, base + (m ^ f)), l1 = ldxu(xs, base + ((m + 1) ^ f));
        const ulonglong2 h0 = ldxu(xs, base + 8 + (m ^ f)), h1 = ldxu(xs, base + 8 + ((m + 1) ^ f));
#pragma unroll
        for (int r = 0; r < R; r++) {
            const uint32_t lo0 = w[r][m] & 0x0F0F0F0Fu, lo1 = w[r][m + 1] & 0x0F0F0F0Fu;
            const uint32_t hi0 = (w[r][m] >> 4) & 0x0F0F0F0Fu, hi1 = (w[r][m + 1] >> 4) & 0x0F0F0F0Fu;
            al0[r] = fma2(add2(magic2(lo0, 0), neg), l0.x, al0[r]);
            al1[r] = fma2(add2(magic2(lo1, 0), neg), l1.x, al1[r]);
            ah0[r] = fma2(add2(magic2(hi0, 0), neg), h0.x, ah0[r]);
            ah1[r] = fma2(add2(magic2(hi1, 0), neg), h1.x, ah1[r]);
            al0[r] = fma2(add2(magic2(lo0, 2), neg), l0.y, al0[r]);
            al1[r] = fma2(add2(magic2(lo1, 2), neg), l1.y, al1[r]);
            ah0[r] = fma2(add2(magic2(hi0, 2), neg), h0.y, ah0[r]);
            ah1[r] = fma2(add2(magic2(hi1, 2), neg), h1.y, ah1[r]);
        }
    }
    const float s0 = x32[8 * b + 2 * g], s1 = x32[8 * b + 2 * g + 1];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const u64 al = add2(al0[r], al1[r]), ah = add2(ah0[r], ah1[r]);
        float v = a[r][0] * pair_sum(al);
        v = fmaf(-c[r][0], s0, v);
        v = fmaf(a[r][1], pair_sum(ah), v);
        acc[r] += fmaf(-c[r][1], s1, v);
    }
}

// 16 bytes at a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint4 lds16_unaligned(const uint8_t *p)
{
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// Lane g (0..3) of a Q6_K superblock b: half h = g / 2, l0 = 16 (g % 2); its
// 16 bytes ql[64h + l0 ..], ql[64h + 32 + l0 ..] and qh[32h + l0 ..] give the
// weights 128h + 32c + l0 + i (c = 0..3, i < 16), each group of 16 one
// sub-block. x unit 64b + 32h + 8c + 4(g % 2) + j sits at physical
// (64b + 32h + 8c) + ((4(g % 2) + j) ^ f), f = (2b + h) & 7.
__device__ __forceinline__ float lane_dot_q6k(const uint8_t *blk, int g, const float *xs, int b)
{
    const int h = g >> 1, e = g & 1, l0 = 16 * e;
    const uint4 q0 = lds16_unaligned(blk + 64 * h + l0);
    const uint4 q1 = lds16_unaligned(blk + 64 * h + 32 + l0);
    const uint4 qh = lds16_unaligned(blk + 128 + 32 * h + l0);
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(blk + 208)));
    const int sb = 192 + 8 * h + e;
    const u64 neg = 0xCB000020CB000020ull;          // (-(2^23 + 32), twice)
    const int base = 64 * b + 32 * h, f = (2 * b + h) & 7;
    const uint32_t lw0[4] = { q0.x, q0.y, q0.z, q0.w }, lw1[4] = { q1.x, q1.y, q1.z, q1.w };
    const uint32_t hw[4] = { qh.x, qh.y, qh.z, qh.w };
    float r = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint32_t *lo = (c & 1) ? lw1 : lw0;
        const int ls = (c >> 1) * 4, hs = 2 * c;
        u64 acc = 0ull;
#pragma unroll
        for (int m = 0; m < 4; m += 2) {
            const uint32_t v0 = ((lo[m] >> ls) & 0x0F0F0F0Fu) | (((hw[m] >> hs) & 0x03030303u) << 4);
            const uint32_t v1 = ((lo[m + 1] >> ls) & 0x0F0F0F0Fu) | (((hw[m + 1] >> hs) & 0x03030303u) << 4);
            const ulonglong2 xa = ldxu(xs, base + 8 * c + ((4 * e + m) ^ f));
            const ulonglong2 xb = ldxu(xs, base + 8 * c + ((4 * e + m + 1) ^ f));
            acc = dot8acc(v0, v1, neg, xa, xb, acc);
        }
        r = fmaf(d * (float)(int8_t)blk[sb + 2 * c], pair_sum(acc), r);
    }
    return r;
}

// x into shared memory (XOR-swizzled float4 units, every load of a thread
// issued before its stores) and, for Q4_K, the sums of x over each 32-weight
// sub-block. Ends with the CTA synchronised.
template <int TYPE>
__device__ __forceinline__ void stage_x(const float *__restrict__ x, float *xs, float *x32, int K)
{
    for (int i0 = threadIdx.x; i0 < K / 4; i0 += 8 * blockDim.x) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * blockDim.x;
            if (i < K / 4) v[u] = __ldg(reinterpret_cast<const float4 *>(x) + i);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = i0 + u * blockDim.x;
            if (i < K / 4) reinterpret_cast<float4 *>(xs)[xswz<TYPE>(i)] = v[u];
        }
    }
    __syncthreads();
    if (TYPE == GGML_TYPE_Q4_K) {
        for (int i = threadIdx.x; i < K / 32; i += blockDim.x) {
            float s = 0.0f;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float4 v = reinterpret_cast<const float4 *>(xs)[xswz<TYPE>(8 * i + u)];
                s += v.x; s += v.y; s += v.z; s += v.w;
            }
            x32[i] = s;
        }
        __syncthreads();
    }
}

// Barrier of the SEGS warps of one row group (named barrier 1 + rloc; 0 is
// the CTA-wide one): the other row groups of the CTA run on.
template <int SEGS>
__device__ __forceinline__ void group_sync(int rloc)
{
    static_assert(MV_WARPS / SEGS < 16, "one named barrier per row group");
    asm volatile("bar.sync %0, %1;" ::"r"(1 + rloc), "n"(SEGS * 32) : "memory");
}

template <int TYPE, int SEGS, int NSLOT, int ROWS>
__global__ void __launch_bounds__(MV_WARPS * 32, 1)
matvec_stream_kernel(const uint8_t *__restrict__ W, const float *__restrict__ x, float *__restrict__ y,
                     int N, int K)
{
    static_assert(ROWS == 1 || TYPE == GGML_TYPE_Q4_K, "row groups are a Q4_K shape");
    constexpr int BB = KQ<TYPE>::BYTES;
    constexpr int RPI = MV_WARPS / SEGS * ROWS;          // rows per CTA iteration
    extern __shared__ uint4 sm4[];
    float *xs = reinterpret_cast<float *>(sm4);
    float *x32 = xs + K;
    const int bpr = K / QK, bps = bpr / SEGS;            // superblocks per row / segment
    const int seg_bytes = bps * BB;                      // one row's segment
    const int slot_bytes = seg_bytes * ROWS;             // a warp's ROWS segments
    uint8_t *ring = reinterpret_cast<uint8_t *>(x32 + ((K / 32 + 3) & ~3));
    __shared__ float part[MV_WARPS * ROWS];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int sbi = lane >> 2, g4 = lane & 3;           // superblock of the eight, lane within it
    const int seg = wid % SEGS, rloc = wid / SEGS;
    uint8_t *slots = ring + (size_t)wid * NSLOT * slot_bytes;   // this warp's NSLOT-deep ring

    // the segments of rows it * RPI + rloc * ROWS + r (r < ROWS) that exist
    auto prefetch = [&](int it, uint8_t *dst) {
        const int row0 = it * RPI + rloc * ROWS;
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            if (row0 + r < N) {
                const uint8_t *src = W + ((size_t)(row0 + r) * bpr + (size_t)seg * bps) * BB;
                const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst + r * seg_bytes);
                for (int i = lane; i < seg_bytes / 16; i += 32) cp_async16(d + 16 * i, src + 16 * i);
            }
        }
        cp_commit();
    };

    int it = blockIdx.x;
#pragma unroll
    for (int i = 0; i < NSLOT - 1; i++) prefetch(it + i * (int)gridDim.x, slots + (size_t)i * slot_bytes);
    stage_x<TYPE>(x, xs, x32, K);

    for (int n = 0; it * RPI < N; it += gridDim.x, n++) {
        // NSLOT - 1 iterations ahead, into the slot the previous iteration read
        prefetch(it + (NSLOT - 1) * (int)gridDim.x, slots + (size_t)((n + NSLOT - 1) % NSLOT) * slot_bytes);
        asm volatile("cp.async.wait_group %0;" ::"n"(NSLOT - 1) : "memory");
        __syncwarp();
        const uint8_t *buf = slots + (size_t)(n % NSLOT) * slot_bytes;
        const int row0 = it * RPI + rloc * ROWS;
        float acc[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; r++) acc[r] = 0.0f;
        // a missing second row of a group computes on stale ring bytes and
        // is never stored
        if (row0 < N) {
            for (int b = sbi; b < bps; b += 8) {
                const int bg = seg * bps + b;               // superblock index within the row
                if (TYPE == GGML_TYPE_Q4_K) lane_dot_q4k<ROWS>(buf + (size_t)b * BB, seg_bytes, g4, xs, x32, bg, acc);
                else acc[0] += lane_dot_q6k(buf + (size_t)b * BB, g4, xs, bg);
            }
        }
        __syncwarp();
#pragma unroll
        for (int r = 0; r < ROWS; r++)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xFFFFFFFFu, acc[r], o);
        if constexpr (SEGS == 1) {
#pragma unroll
            for (int r = 0; r < ROWS; r++)
                if (lane == 0 && row0 + r < N) y[row0 + r] = acc[r];
        } else {
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < ROWS; r++) part[wid * ROWS + r] = acc[r];
            }
            group_sync<SEGS>(rloc);
            if (seg == 0 && lane == 0) {
#pragma unroll
                for (int r = 0; r < ROWS; r++) {
                    if (row0 + r < N) {
                        float s = 0.0f;
                        for (int j = 0; j < SEGS; j++) s += part[(wid + j) * ROWS + r];
                        y[row0 + r] = s;
                    }
                }
            }
            group_sync<SEGS>(rloc);
        }
    }
    cp_wait0();
}

int g_mv_last = 0;         // kernel of the latest matvec: 2 segment stream, 3 staged, 4 tensor cores,
                           // 5 Q4_K integer mma.sync, 6 Q6_K integer mma.sync

template <int TYPE, int SEGS, int NSLOT, int ROWS>
static bool launch_matvec_stream(float *y, const void *W, const float *x, int N, int K, size_t smem)
{
    static unsigned done[64];
    const int dev = ctx().device & 63;
    if (!done[dev]) {
        if (cudaFuncSetAttribute(matvec_stream_kernel<TYPE, SEGS, NSLOT, ROWS>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        done[dev] = 1;
    }
    constexpr int RPI = MV_WARPS / SEGS * ROWS;
    const long iters = ((long)N + RPI - 1) / RPI;
    const int grid = (int)(iters < ctx().sms ? iters : ctx().sms);
    matvec_stream_kernel<TYPE, SEGS, NSLOT, ROWS><<<grid, MV_WARPS * 32, smem, ctx().cur>>>((const uint8_t *)W, x, y,
                                                                                           N, K);
    g_mv_last = 2;
    return cudaGetLastError() == cudaSuccess || fail("matvec launch failed");
}

// The deepest ring (4, 3 or 2 slots per warp, each of ROWS row segments)
// whose shared memory fits.
template <int TYPE, int SEGS, int ROWS>
static bool try_matvec_stream(float *y, const void *W, const float *x, int N, int K)
{
    constexpr int BB = KQ<TYPE>::BYTES;
    const int bpr = K / QK;
    if (bpr % SEGS || ((size_t)(bpr / SEGS) * BB) % 16 || ((uintptr_t)W & 15)) return false;
    const size_t base = (size_t)K * 4 + (size_t)((K / 32 + 3) & ~3) * 4;
    const size_t seg = (size_t)MV_WARPS * (bpr / SEGS) * BB * ROWS;
    const size_t cap = 200 * 1024;
    if (base + 4 * seg <= cap) return launch_matvec_stream<TYPE, SEGS, 4, ROWS>(y, W, x, N, K, base + 4 * seg);
    if (base + 3 * seg <= cap) return launch_matvec_stream<TYPE, SEGS, 3, ROWS>(y, W, x, N, K, base + 3 * seg);
    if (base + 2 * seg <= cap) return launch_matvec_stream<TYPE, SEGS, 2, ROWS>(y, W, x, N, K, base + 2 * seg);
    return false;
}

static unsigned grid_for(size_t warps_needed)
{
    const size_t cap = (size_t)ctx().sms * 8;   // 8 CTAs x 8 warps per SM
    const size_t need = (warps_needed + WARPS - 1) / WARPS;
    return (unsigned)(need < cap ? (need ? need : 1) : cap);
}

template <int TYPE, int WPR>
static bool launch_matvec(float *y, const void *W, const float *x, int N, int K)
{
    constexpr int ROWS = WARPS / WPR;
    const size_t ctas = ((size_t)N + ROWS - 1) / ROWS;
    const size_t cap = (size_t)ctx().sms * 8;
    matvec_kq_kernel<TYPE, WPR><<<(unsigned)(ctas < cap ? ctas : cap), WARPS * 32, 0, ctx().cur>>>(
        (const uint8_t *)W, x, y, N, K);
    g_mv_last = 3;
    TCG_LAUNCHED();
    return true;
}

bool launch_matvec_tc_q4k(float *y, const void *W, const float *x, int N, int K, bool *used);   // mv_tc.cu
bool launch_matvec_mma_q4k(float *y, const void *W, const float *x, int N, int K, bool *used);  // mv_mma.cu
bool launch_matvec_mma_q6k(float *y, const void *W, const float *x, int N, int K, bool *used);  // mv_mma.cu

template <int TYPE>
static bool matvec_dispatch(float *y, const void *W, const float *x, int N, int K)
{
    // Q4_K on the tensor cores when enabled (tcg_matvec_set_tc) and the
    // matrix is 16-byte aligned
    if (TYPE == GGML_TYPE_Q4_K) {
        bool used = false;
        if (!launch_matvec_tc_q4k(y, W, x, N, K, &used)) return false;
        if (used) {
            g_mv_last = 4;
            return true;
        }
        // the integer mma.sync kernel (default) wherever it applies
        if (!launch_matvec_mma_q4k(y, W, x, N, K, &used)) return false;
        if (used) {
            g_mv_last = 5;
            return true;
        }
    } else {
        // Q6_K on the integer mma.sync kernel where rows are whole 8-superblock segments
        bool used = false;
        if (!launch_matvec_mma_q6k(y, W, x, N, K, &used)) return false;
        if (used) {
            g_mv_last = 6;
            return true;
        }
    }
    // The streaming kernel whenever its segments tile the rows in 16-byte
    // units and x fits on chip; rows split in 4 when there are few of them.
    const long rows_per_sm = (long)N / (ctx().sms > 0 ? ctx().sms : 148);
    if (rows_per_sm < 64 && try_matvec_stream<TYPE, 4, 1>(y, W, x, N, K)) return true;
    if (try_matvec_stream<TYPE, 1, 1>(y, W, x, N, K)) return true;
    if (try_matvec_stream<TYPE, 2, 1>(y, W, x, N, K)) return true;
    // Rows too long for those rings: Q4_K in row pairs (one x load for both,
    // 2.2 TB/s at 16384 x 14336 where the staged kernel makes 0.73), then
    // shorter segments.
    if constexpr (TYPE == GGML_TYPE_Q4_K) {
        if (try_matvec_stream<TYPE, 1, 2>(y, W, x, N, K) || try_matvec_stream<TYPE, 2, 2>(y, W, x, N, K) ||
            try_matvec_stream<TYPE, 4, 2>(y, W, x, N, K) || try_matvec_stream<TYPE, 8, 2>(y, W, x, N, K))
            return true;
    }
    if (try_matvec_stream<TYPE, 4, 1>(y, W, x, N, K)) return true;
    if (try_matvec_stream<TYPE, 8, 1>(y, W, x, N, K)) return true;
    // Otherwise the staged kernel, with enough warps per row to keep ~48
    // resident per SM streaming weight bytes.
    const long want = (long)ctx().sms * 48;
    if ((long)N >= want) return launch_matvec<TYPE, 1>(y, W, x, N, K);
    if ((long)N * 2 >= want) return launch_matvec<TYPE, 2>(y, W, x, N, K);
    if ((long)N * 4 >= want) return launch_matvec<TYPE, 4>(y, W, x, N, K);
    return launch_matvec<TYPE, 8>(y, W, x, N, K);
}

// Q4_K / Q6_K blocks to their tf32 pairs (hi, lo), 16-byte aligned outputs,
// n a multiple of 256: dequantisation bit-identical to tcg_dequant, then the
// split of tcg_split_tf32.
bool launch_dequant_split(const void *src, float *hi, float *lo, size_t n, ggml_type_t t, cudaStream_t s)
{
    if (n % QK || ((uintptr_t)hi & 15) || ((uintptr_t)lo & 15))
        return fail("dequant split: %zu weights / unaligned outputs", n);
    const size_t nb = n / QK;
    const unsigned grid = grid_for((nb + GROUP - 1) / GROUP);
    if (t == GGML_TYPE_Q4_K)
        dequant_kq_kernel<GGML_TYPE_Q4_K, true><<<grid, WARPS * 32, 0, s>>>((const uint8_t *)src, hi, nb, lo);
    else if (t == GGML_TYPE_Q6_K)
        dequant_kq_kernel<GGML_TYPE_Q6_K, true><<<grid, WARPS * 32, 0, s>>>((const uint8_t *)src, hi, nb, lo);
    else
        return fail("dequant split: type %s", ggml_type_name(t));
    TCG_LAUNCHED();
    return true;
}

}  // namespace tcg

using namespace tcg;

extern "C" {

bool tcg_dequant(float *dst, const void *src, size_t n, ggml_type_t t)
{
    if (!need_ctx()) return false;
    if (n == 0) return true;
    if (!dst || !src) return fail("tcg_dequant: null pointer");
    switch (t) {
    case GGML_TYPE_F32:
        TCG_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, ctx().cur));
        return true;
    case GGML_TYPE_F16: {
        if ((uintptr_t)src & 1) return fail("tcg_dequant: F16 source is not 2-byte aligned");
        size_t blocks = (n + 255) / 256, cap = (size_t)ctx().sms * 16;
        f16_to_f32_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, ctx().cur>>>(
            (const uint16_t *)src, dst, n);
        TCG_LAUNCHED();
        return true;
    }
    case GGML_TYPE_Q4_K:
    case GGML_TYPE_Q6_K: {
        if (n % QK) return fail("tcg_dequant: %zu elements is not a whole number of %d-weight superblocks", n, QK);
        if ((uintptr_t)dst & 15) return fail("tcg_dequant: destination is not 16-byte aligned");
        const size_t nb = n / QK;
        const unsigned grid = grid_for((nb + GROUP - 1) / GROUP);
        if (t == GGML_TYPE_Q4_K)
            dequant_kq_kernel<GGML_TYPE_Q4_K><<<grid, WARPS * 32, 0, ctx().cur>>>((const uint8_t *)src, dst, nb);
        else
            dequant_kq_kernel<GGML_TYPE_Q6_K><<<grid, WARPS * 32, 0, ctx().cur>>>((const uint8_t *)src, dst, nb);
        TCG_LAUNCHED();
        return true;
    }
    default:
        return fail("tcg_dequant: no conversion for type %s", ggml_type_name(t));
    }
}

bool tcg_matvec_q(float *y, const void *W, const float *x, int N, int K, ggml_type_t t)
{
    if (!need_ctx()) return false;
    if (N < 0 || K < 0) return fail("tcg_matvec_q: negative size");
    if (N == 0) return true;
    if (K % QK) return fail("tcg_matvec_q: K=%d is not a multiple of %d", K, QK);
    if ((uintptr_t)x & 15) return fail("tcg_matvec_q: x is not 16-byte aligned");
    if (K == 0) {
        TCG_CUDA(cudaMemsetAsync(y, 0, (size_t)N * sizeof(float), ctx().cur));
        return true;
    }
    if (t == GGML_TYPE_Q4_K) return matvec_dispatch<GGML_TYPE_Q4_K>(y, W, x, N, K);
    if (t == GGML_TYPE_Q6_K) return matvec_dispatch<GGML_TYPE_Q6_K>(y, W, x, N, K);
    return fail("tcg_matvec_q: type %s is not a supported K-quant", ggml_type_name(t));
}

bool tcg_dequant_host(float *dst, const void *src, size_t n, ggml_type_t t)
{
    if (!need_ctx()) return false;
    if (n == 0) return true;
    size_t in_bytes;
    switch (t) {
    case GGML_TYPE_F32: in_bytes = n * 4; break;
    case GGML_TYPE_F16: in_bytes = n * 2; break;
    case GGML_TYPE_Q4_K: in_bytes = n / QK * KQ<GGML_TYPE_Q4_K>::BYTES; break;
    case GGML_TYPE_Q6_K: in_bytes = n / QK * KQ<GGML_TYPE_Q6_K>::BYTES; break;
    default: return fail("tc_dequant: no conversion for type %s", ggml_type_name(t));
    }
    const size_t out_bytes = n * sizeof(float), in_at = (out_bytes + 255) & ~(size_t)255;
    uint8_t *buf = (uint8_t *)scratch(in_at + in_bytes);
    if (!buf) return false;
    cudaStream_t s = ctx().cur;
    TCG_CUDA(cudaMemcpyAsync(buf + in_at, src, in_bytes, cudaMemcpyHostToDevice, s));
    if (!tcg_dequant((float *)buf, buf + in_at, n, t)) return false;
    TCG_CUDA(cudaMemcpyAsync(dst, buf, out_bytes, cudaMemcpyDeviceToHost, s));
    TCG_CUDA(cudaStreamSynchronize(s));
    return true;
}

const void *tcg_tensor_upload(const gguf_tensor_t *t, tcg_arena_t *a)
{
    if (!t || !t->data || t->nbytes == 0) { fail("tensor has no readable payload"); return nullptr; }
    void *d = tcg_arena_alloc(a, (size_t)t->nbytes, 256);
    if (!d) return nullptr;
    if (!tcg_h2d(d, t->data, (size_t)t->nbytes)) return nullptr;
    return d;
}

const float *tcg_dequant_view(const gguf_tensor_t *t, tcg_arena_t *a, bool *converted)
{
    if (!t || !t->data) { fail("tensor has no readable payload"); return nullptr; }
    if (t->type == GGML_TYPE_F32) {
        if (converted) *converted = false;
        return (const float *)tcg_tensor_upload(t, a);
    }
    const size_t mark = tcg_arena_mark(a);
    float *out = (float *)tcg_arena_alloc(a, (size_t)t->n_elem * sizeof(float), 256);
    if (!out) return nullptr;
    const void *raw = tcg_tensor_upload(t, a);
    if (!raw || !tcg_dequant(out, raw, (size_t)t->n_elem, t->type)) {
        tcg_arena_release(a, mark);
        return nullptr;
    }
    // the packed copy sits above `out`; it is dead once the kernel has run
    if (!tcg_sync()) return nullptr;
    tcg_arena_release(a, (size_t)((unsigned char *)out - a->base) + (size_t)t->n_elem * sizeof(float));
    if (converted) *converted = true;
    return out;
}

}  // extern "C"

// Test hook: the kernel of the latest K-quant matvec (2: row segments
// streamed through a cp.async ring, 3: staged groups, 4: Q4_K on tcgen05,
// 5: Q4_K on the integer mma.sync kernel; 0: none yet).
extern "C" int tcg_matvec_last_kernel(void) { return tcg::g_mv_last; }

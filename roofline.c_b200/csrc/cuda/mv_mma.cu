// mv_mma.cu -- the fused Q4_K dequant-matvec y = W x on the warp-level
// integer tensor path (mma.sync m16n8k32, u8 x s8 -> s32).
//
// The Q4_K arm of the dequant seam (roofline.c src/dequant.c:40-63 with
// ggml's Q4_K block: fp16 d and dmin, twelve bytes of 6-bit scales and mins,
// 128 bytes of nibbles) gives weight k of 32-weight sub-block j the value
// (d*sc_j)*q_k - (dmin*m_j), so a row's dot product regroups as
//     y_r = sum_sb d * sum_j sc_j * sum_{k in j} q_k x_k  -  dmin * sum_j m_j * X_j,
// X_j the sum of x over sub-block j. The sums over q run as exact integer
// MMAs; everything per weight is one mask:
//   - A (16 rows x 32 weights of one sub-block): the quant bytes as loaded,
//     masked to the low nibbles (sub-block 2c of 32-byte chunk c) or to the
//     high nibbles kept in place, i.e. 16 q (sub-block 2c+1);
//   - B (32 weights x 8 columns): each superblock of x is scaled by a power
//     of two to |v| < 64 and split into four int8 pieces
//     v = p0 + p1/2^7 + p2/2^14 + p3/2^21 (the rest is below 2^-26 of the
//     superblock's largest |x|), pieces in columns 0-3, zeros in 4-7. The
//     pieces of the superblocks a CTA needs are built in shared memory when
//     it starts;
//   - C: per thread, rows g and g+8 of the tile times columns 2t, 2t+1:
//     lane quad t = 0 holds the p0/p1 sums, t = 1 the p2/p3 sums. They are
//     multiplied by the row's 6-bit sub-block scale and summed over the
//     superblock in 32-bit integers (exact: below 2^28), then converted once
//     per superblock, scaled by d and the power of two, and accumulated in
//     fp32. The min term is spread over the four lanes of a quad (two
//     sub-blocks each) and the quad's partial sums meet by two shuffles.
// Results differ from the dequantise-then-dot order by rounding only.
//
// Work: units of (16-row tile, K segment of spb superblocks), segment-major,
// split into one contiguous range per CTA (one persistent CTA per SM). The
// weights are fed by the tensor memory accelerator: one producer lane copies
// each unit's 16 row segments (spb * 144 contiguous bytes each) into a ring of
// shared-memory slots, as many units ahead as the slots hold, from the
// kernel's first instructions on, so that most of an SM's share of the
// matrix is in flight at once while x is being prepared: one 3-D tensor copy
// per unit (36 words x spb superblocks x 16 rows; rows past N arrive as
// zeros). The slot's rows are spb * 144 bytes apart, and MMA row g reads slot
// row sigma(g), a permutation chosen per spb so that the quant loads of a
// half-warp hit distinct shared-memory banks. Sixteen consumer
// warps take the CTA's units in turn. A tile split into S > 1 segments is
// summed by the last warp to finish one of its segments, in segment order (a
// per-tile arrival counter that this warp resets), so every call gives the
// same bits. Slot waits are bounded; one that gives up raises the device
// error word, and the unit still arrives (with a zero partial sum) so the
// counters stay consistent. No thread waits on another CTA.
#include "tcg_common.cuh"
#include "tc05.cuh"

#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

namespace tcg {

namespace {

constexpr int MM_WARPS = 16;
constexpr int MM_BB = 144;                  // Q4_K bytes per superblock
constexpr int MM_XSB = 1024 + 32 + 16;      // shared bytes per superblock of x: pieces, 8 sums, scale (+pad)
constexpr int MQ_BB = 210;                  // Q6_K bytes per superblock
constexpr int MQ_SPB = 8;                   // Q6_K superblocks per unit: 1680 bytes, a whole number of 16
constexpr int MQ_XSB = 1024 + 256 + 16;     // Q6_K: pieces, -32 x (sum) per (group, half, piece), scale

template <int QT> struct MmType;
template <> struct MmType<4> { static constexpr int BB = MM_BB, XSB = MM_XSB; };
template <> struct MmType<6> { static constexpr int BB = MQ_BB, XSB = MQ_XSB; };

// D = A B over one sub-block: A u8 16 x 32 (a0: row g, k 4t..4t+3; a1: row
// g+8; a2, a3: k 16+4t..), B s8 32 x 8 (b0: k 4t..4t+3 of column g, b1: k
// 16+4t..), D rows g, g+8 x columns 2t, 2t+1.
__device__ __forceinline__ void mma_u8s8(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%10, %10, %10, %10};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D += A B (layouts of mma_u8s8)
__device__ __forceinline__ void mma_u8s8_acc(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int b) { return __byte_perm(w, 0u, 0x4440u | (unsigned)b); }

// four int8 from four integer-valued floats in [-128, 127]
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d)
{
    const uint32_t lo = __byte_perm((uint32_t)__float2int_rn(a), (uint32_t)__float2int_rn(b), 0x0040u);
    const uint32_t hi = __byte_perm((uint32_t)__float2int_rn(c), (uint32_t)__float2int_rn(d), 0x0040u);
    return __byte_perm(lo, hi, 0x5410u);
}

// One superblock of a unit in flight: headers (d, dmin, scales) of rows g and
// g+8, and this lane's 8 quant bytes of each 32-byte chunk of both rows.
struct Sb {
    uint4 h0, h1;
    uint2 q0[4], q1[4];
};

// The 6-bit scales (sc) and mins (mn) of sub-blocks 0-3 and 4-7, one per byte.
__device__ __forceinline__ void scales_of(const uint4 &h, uint32_t &sc_lo, uint32_t &sc_hi, uint32_t &mn_lo,
                                          uint32_t &mn_hi)
{
    sc_lo = h.y & 0x3F3F3F3Fu;
    mn_lo = h.z & 0x3F3F3F3Fu;
    sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
}

__device__ __forceinline__ float f16lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float f16hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
// a small non-negative integer (< 2^23) as a float, exactly
__device__ __forceinline__ float small_int_float(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// Accumulate superblock s (x pieces at xsb) of rows g, g+8 into acc0 / acc1.
// Each 32-byte chunk c holds sub-block 2c in its low nibbles and 2c + 1 in
// its high nibbles. Two chained MMAs give both sub-blocks in one D: B columns
// 0-3 carry the pieces of x's sub-block 2c and meet the low nibbles (zero in
// columns 4-7), then columns 4-7 carry the pieces of sub-block 2c + 1 and
// meet the high nibbles kept in place, 16 q (zero in columns 0-3). Lane (g,
// t) holds columns 2t, 2t + 1: sub-block 2c + t / 2, pieces 2 (t % 2) and
// 2 (t % 2) + 1, multiplied by that sub-block's scale of rows g, g + 8 in
// 32-bit integers (|.| < 2^27 over the superblock). Its share of the min
// terms: sub-blocks 2t, 2t + 1.
__device__ __forceinline__ void sb_dot(const Sb &s, const uint8_t *xsb, int g, int t, float &acc0, float &acc1)
{
    uint32_t sc0l, sc0h, mn0l, mn0h, sc1l, sc1h, mn1l, mn1h;
    scales_of(s.h0, sc0l, sc0h, mn0l, mn0h);
    scales_of(s.h1, sc1l, sc1h, mn1l, mn1h);
    const uint32_t th = (uint32_t)t >> 1;                           // 0: low-nibble sub-block, 1: high
    const bool bhi = g >= 4;                                        // this lane's B column: 2c + 1
    const uint8_t *xb = xsb + (bhi ? 128 : 0) + (g & 3) * 32 + 8 * t;
    int a[4] = { 0, 0, 0, 0 };
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint2 bx = *reinterpret_cast<const uint2 *>(xb + c * 256);
        const uint32_t bl0 = bhi ? 0u : bx.x, bl1 = bhi ? 0u : bx.y;
        const uint32_t bh0 = bhi ? bx.x : 0u, bh1 = bhi ? bx.y : 0u;
        int d[4];
        mma_u8s8(d, s.q0[c].x & 0x0F0F0F0Fu, s.q1[c].x & 0x0F0F0F0Fu, s.q0[c].y & 0x0F0F0F0Fu,
                 s.q1[c].y & 0x0F0F0F0Fu, bl0, bl1);
        mma_u8s8_acc(d, s.q0[c].x & 0xF0F0F0F0u, s.q1[c].x & 0xF0F0F0F0u, s.q0[c].y & 0xF0F0F0F0u,
                     s.q1[c].y & 0xF0F0F0F0u, bh0, bh1);
        // scale of sub-block 2c + th: byte 2 (c % 2) + th of the low (c < 2) or high scale word
        const uint32_t sel = 0x4440u | (2u * (c & 1) + th);
        const int s0 = (int)__byte_perm(c < 2 ? sc0l : sc0h, 0u, sel);
        const int s1 = (int)__byte_perm(c < 2 ? sc1l : sc1h, 0u, sel);
        a[0] += d[0] * s0; a[1] += d[1] * s0; a[2] += d[2] * s1; a[3] += d[3] * s1;
    }
    // pieces (0, 1) for even t, (2, 3) for odd t: x = (p0 + p1/2^7 + p2/2^14
    // + p3/2^21) 2^(e-6), 2^(e-13) stored; the high sub-block's sums are 16x
    const float xe = *reinterpret_cast<const float *>(xsb + 1024 + 32);      // 2^(e - 13)
    const float k = ((t & 1) ? 6.103515625e-05f : 1.0f) * (th ? 0.0625f : 1.0f);
    const float f0 = fmaf((float)a[0], 128.0f, (float)a[1]), f1 = fmaf((float)a[2], 128.0f, (float)a[3]);
    const float d0 = f16lo(s.h0.x), d1 = f16lo(s.h1.x);
    // (f xe) (d k): both factors stay normal floats for every d and exponent
    acc0 = fmaf(f0 * xe, d0 * k, acc0);
    acc1 = fmaf(f1 * xe, d1 * k, acc1);
    // min terms of sub-blocks 2t, 2t+1
    const float2 X = *reinterpret_cast<const float2 *>(xsb + 1024 + 8 * t);
    const uint32_t m0 = t < 2 ? mn0l : mn0h, m1 = t < 2 ? mn1l : mn1h;
    const int bm = (2 * t) & 3;
    const float dm0 = f16hi(s.h0.x), dm1 = f16hi(s.h1.x);
    acc0 = fmaf(-dm0, fmaf(small_int_float(byte_of(m0, bm)), X.x, small_int_float(byte_of(m0, bm + 1)) * X.y), acc0);
    acc1 = fmaf(-dm1, fmaf(small_int_float(byte_of(m1, bm)), X.x, small_int_float(byte_of(m1, bm + 1)) * X.y), acc1);
}

// D = A B + C over one 32-weight group (layouts of mma_u8s8)
__device__ __forceinline__ void mma_u8s8_c(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1, int c0, int c1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%10, %11, %10, %11};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// prmt with selector sel as PTX defines it: bit 3 of a selector nibble
// replicates the sign of the byte chosen by its bits 0-2 (the __byte_perm
// intrinsic reads bits 0-2 only)
__device__ __forceinline__ uint32_t prmt_s(uint32_t a, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(a), "r"(sel));
    return r;
}

// Four bytes of shared memory at p. A Q6_K superblock is 210 bytes, so the
// odd ones of a unit start 2 bytes past a word boundary: two aligned words
// and a byte permute.
template <bool ODD>
__device__ __forceinline__ uint32_t ld_q6(const uint8_t *p)
{
    if constexpr (!ODD) {
        return *reinterpret_cast<const uint32_t *>(p);
    } else {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(p - 2);
        return __byte_perm(w[0], w[1], 0x5432u);
    }
}

// Q6_K superblock (src/dequant.c:40-63 with ggml's block: ql[128] low
// nibbles, qh[64] high bit pairs, 16 int8 scales, fp16 d; weight 128h + 32j
// + l = d * sc[8h + 2j + l/16] * (q - 32), q = nibble of ql[64h + 32(j&1) +
// l] (low for j < 2) | bits 2j, 2j+1 of qh[32h + l] << 4). Group gi = 4h + j
// holds 32 consecutive weights, the x sub-block gi of the pieces. One MMA
// per group: A = q of rows g, g+8 (a0/a1 k 4t.., a2/a3 k 16+4t..); B
// columns 0-3 the pieces of x at k < 16 (zero above), columns 4-7 the pieces
// at k >= 16, so column c sums one 16-weight scale half (c / 4) times piece
// c % 4; C = -32 (sum of that half's piece) makes it the sum of (q - 32) x
// exactly. Lane (g, t) holds columns 2t, 2t+1: half s = t / 2, pieces 2(t%2),
// 2(t%2)+1, multiplied by the rows' scale of (gi, s) in 32-bit integers
// (|.| < 2^27 over the superblock), then converted once.
template <bool ODD>
__device__ __forceinline__ void sb6_dot(const uint8_t *r0, const uint8_t *r1, const uint8_t *xsb, int g, int t,
                                        float &acc0, float &acc1)
{
    const int s = t >> 1;
    uint32_t l0[2][2][2], l1[2][2][2], h0[2][2], h1[2][2];      // ql [h][j&1][k half], qh [h][k half]
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int kh = 0; kh < 2; kh++) {
#pragma unroll
            for (int jl = 0; jl < 2; jl++) {
                l0[h][jl][kh] = ld_q6<ODD>(r0 + 64 * h + 32 * jl + 16 * kh + 4 * t);
                l1[h][jl][kh] = ld_q6<ODD>(r1 + 64 * h + 32 * jl + 16 * kh + 4 * t);
            }
            h0[h][kh] = ld_q6<ODD>(r0 + 128 + 32 * h + 16 * kh + 4 * t);
            h1[h][kh] = ld_q6<ODD>(r1 + 128 + 32 * h + 16 * kh + 4 * t);
        }
    uint32_t w0[4], w1[4];                                      // the 16 scales
#pragma unroll
    for (int w = 0; w < 4; w++) {
        w0[w] = ld_q6<ODD>(r0 + 192 + 4 * w);
        w1[w] = ld_q6<ODD>(r1 + 192 + 4 * w);
    }
    // scale byte 2gi + s: byte s of the word's even half, 2 + s of its odd half, sign-extended
    const uint32_t se = 0x8880u | 0x1110u * (uint32_t)s;
    const uint32_t sel_even = se | (uint32_t)s, sel_odd = (se + 0x2220u) | (uint32_t)(2 + s);
    int acc[4] = { 0, 0, 0, 0 };
#pragma unroll
    for (int gi = 0; gi < 8; gi++) {
        const int h = gi >> 2, j = gi & 3;
        const auto qword = [&](uint32_t wl, uint32_t wh) {
            const uint32_t nib = j < 2 ? wl : wl >> 4;
            const uint32_t hb = (j < 3 ? wh << (4 - 2 * j) : wh >> 2) & 0x30303030u;
            return (nib & 0x0F0F0F0Fu) | hb;
        };
        const uint32_t a0 = qword(l0[h][j & 1][0], h0[h][0]), a1 = qword(l1[h][j & 1][0], h1[h][0]);
        const uint32_t a2 = qword(l0[h][j & 1][1], h0[h][1]), a3 = qword(l1[h][j & 1][1], h1[h][1]);
        const uint32_t bw = *reinterpret_cast<const uint32_t *>(xsb + gi * 128 + (g & 3) * 32 + (g >> 2) * 16 + 4 * t);
        const int2 cx = *reinterpret_cast<const int2 *>(xsb + 1024 + (2 * gi + s) * 16 + 8 * (t & 1));
        int d[4];
        mma_u8s8_c(d, a0, a1, a2, a3, g < 4 ? bw : 0u, g < 4 ? 0u : bw, cx.x, cx.y);
        const uint32_t sel = (gi & 1) ? sel_odd : sel_even;
        const int sc0 = (int)prmt_s(w0[gi >> 1], sel), sc1 = (int)prmt_s(w1[gi >> 1], sel);
        acc[0] += d[0] * sc0;
        acc[1] += d[1] * sc0;
        acc[2] += d[2] * sc1;
        acc[3] += d[3] * sc1;
    }
    // columns 2t, 2t+1 = pieces (0, 1) for even t, (2, 3) for odd t:
    // x = (p0 + p1/2^7 + p2/2^14 + p3/2^21) 2^(e-6), 2^(e-13) stored
    const float xe = *reinterpret_cast<const float *>(xsb + 1280);
    const float k = (t & 1) ? 6.103515625e-05f : 1.0f;                     // 2^-14 : 1
    const float f0 = fmaf((float)acc[0], 128.0f, (float)acc[1]), f1 = fmaf((float)acc[2], 128.0f, (float)acc[3]);
    const float d0 = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(r1 + 208)));
    acc0 = fmaf(f0 * xe, d0 * k, acc0);
    acc1 = fmaf(f1 * xe, d1 * k, acc1);
}

constexpr int MM_THREADS = MM_WARPS * 32 + 32;   // sixteen consumer warps and the producer warp
constexpr int MM_CMB_FLOATS = 2 * MM_WARPS * 16; // the parts' sums: owners x hs <= MM_WARPS, two buffers, 16 rows

// fetch-and-add with release (the warp's partial sums, ordered before it by
// __syncwarp) and acquire (the other segments' sums, for the last to arrive)
__device__ __forceinline__ int atom_add_acq_rel(int *p, int v)
{
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(dst), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(z), "r"(bar) : "memory");
}

// the bytes of a 3-D box into L2 (nothing written to shared memory)
__device__ __forceinline__ void tma_prefetch3(const CUtensorMap *map, int x, int y, int z)
{
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];"
                 ::"l"((unsigned long long)map), "r"(x), "r"(y), "r"(z) : "memory");
}

__device__ __forceinline__ void tma_load2(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar) : "memory");
}

// The same from global memory: rows r0, r1 (null past the matrix: zeros),
// superblock at byte offset o
__device__ __forceinline__ void load_sb_global(Sb &s, const uint8_t *r0, const uint8_t *r1, int o, int t)
{
    const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
    const uint2 z2 = make_uint2(0u, 0u);
    s.h0 = r0 ? __ldg(reinterpret_cast<const uint4 *>(r0 + o)) : z4;
    s.h1 = r1 ? __ldg(reinterpret_cast<const uint4 *>(r1 + o)) : z4;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        s.q0[c] = r0 ? __ldg(reinterpret_cast<const uint2 *>(r0 + o + 16 + 32 * c + 8 * t)) : z2;
        s.q1[c] = r1 ? __ldg(reinterpret_cast<const uint2 *>(r1 + o + 16 + 32 * c + 8 * t)) : z2;
    }
}

__device__ __forceinline__ void load_sb_smem(Sb &s, const uint8_t *r0, const uint8_t *r1, int t)
{
    s.h0 = *reinterpret_cast<const uint4 *>(r0);
    s.h1 = *reinterpret_cast<const uint4 *>(r1);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        s.q0[c] = *reinterpret_cast<const uint2 *>(r0 + 16 + 32 * c + 8 * t);
        s.q1[c] = *reinterpret_cast<const uint2 *>(r1 + 16 + 32 * c + 8 * t);
    }
}

// Shared memory: x pieces (nsl superblocks), nslot unit slots of 16 rows x rs
// bytes, then the slots' full and empty barriers and the abort flag. QT 4:
// Q4_K, a 3-D tensor copy per unit; QT 6: Q6_K, a 2-D one (8-byte elements,
// 210 per 8-superblock row segment).
template <int QT>
__global__ void __launch_bounds__(MM_THREADS, 1)
mv_kq_mma_kernel(const __grid_constant__ CUtensorMap wmap, const float *__restrict__ x, float *__restrict__ y,
                 int N, int nsb, int spb, int S, int tiles, long long U, float *ws, int *cnt, int nslot, int nwork,
                 int hs, int tm, uint32_t sigma, int x_bytes, int early, const void *Wg, int direct, int *err)
{
    constexpr int BB = MmType<QT>::BB, XSB = MmType<QT>::XSB;
    extern __shared__ __align__(128) uint8_t smx[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    // Units: segment-major, one contiguous range of them per CTA (tm 0), or
    // whole tiles per CTA, tile-major (tm 1: a tile's segments meet in
    // shared memory)
    const long long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    const int T0 = (int)((long long)tiles * blockIdx.x / gridDim.x);
    const int T1 = (int)((long long)tiles * (blockIdx.x + 1) / gridDim.x);
    const int nunits = tm ? (T1 - T0) * S : (int)(u1 - u0);
    const int seg_lo = tm ? 0 : (int)(u0 / tiles);
    const int sb0 = seg_lo * spb;                                   // first superblock of x this CTA holds
    const int nsl = tm ? nsb : min((int)((u1 - 1) / tiles + 1) * spb, nsb) - sb0;   // superblocks of x it holds
    const auto unit_of = [&](int k, int &seg, int &tile) {
        if (tm) {
            tile = T0 + k / S;
            seg = k - (k / S) * S;
        } else {
            const long long u = u0 + k;
            seg = (int)(u / tiles);
            tile = (int)(u - (long long)seg * tiles);
        }
    };
    const int rs = spb * BB;                                        // slot row stride
    uint8_t *slots = smx + x_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(slots + (size_t)nslot * 16 * rs);
    const uint32_t full0 = su32(bars), empty0 = su32(bars + nslot);
    volatile int *abort = reinterpret_cast<volatile int *>(bars + 2 * nslot);
    // units read by several warps (hs > 1, or direct units): the parts' sums
    // meet here, two buffers per group of warps (alternate units)
    float *cmb = reinterpret_cast<float *>(bars + 2 * nslot + 2);
    // tm: the partial sums of the CTA's tiles (S x 16 rows each) and their
    // arrival counters
    float *tpart = cmb + (hs > 1 || direct ? MM_CMB_FLOATS : 0);
    int *tcnt = reinterpret_cast<int *>(tpart + (tm ? (size_t)(T1 - T0) * S * 16 : 0));
    // Q6_K slots hold spb / 8 boxes of 16 rows x 1680 bytes one after another
    constexpr int RB = QT == 4 ? 0 : MQ_SPB * MQ_BB;                // bytes of a box row (Q6_K)

    // With early set (a decode pass over static weights) the kernel queued
    // after this one may be scheduled as this one's CTAs retire: a matvec
    // then fetches its weights on the SMs freed first, and waits for this
    // kernel's completion (pdl_wait) before it reads x or writes anything.
    if (early) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < nslot; s++) {
            bar_init(full0 + 8 * s, 1);
            bar_init(empty0 + 8 * s, hs);                           // the hs warps sharing the slot
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tm)
        for (int i = threadIdx.x; i < T1 - T0; i += blockDim.x) tcnt[i] = 0;
    __syncthreads();

    if (warp == MM_WARPS) {
        // producer: unit k of the CTA into slot k % nslot once its previous
        // unit has been consumed
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&wmap) : "memory");
            auto fill = [&](int k) {
                int seg, tile;
                unit_of(k, seg, tile);
                const uint32_t fb = full0 + 8 * (k % nslot);
                bar_expect_tx(fb, (uint32_t)(16 * rs));
                if constexpr (QT == 4) {
                    tma_load3(su32(slots + (size_t)(k % nslot) * 16 * rs), &wmap, fb, 0, seg * spb, tile * 16);
                } else {
                    for (int b = 0; b < spb / MQ_SPB; b++)
                        tma_load2(su32(slots + (size_t)(k % nslot) * 16 * rs + (size_t)b * 16 * RB), &wmap, fb,
                                  (seg * (spb / MQ_SPB) + b) * (RB / 8), tile * 16);
                }
            };
            // direct: units past the slots are read from global memory by
            // the idle consumer warps; L2 gets them first
            const auto prefetch_rest = [&]() {
                if constexpr (QT == 4) {
                    for (int j = nslot; direct && j < nunits; j++) {
                        int seg, tile;
                        unit_of(j, seg, tile);
                        tma_prefetch3(&wmap, 0, seg * spb, tile * 16);
                    }
                }
            };
            const int nfill = direct ? min(nunits, nslot) : nunits;
            int k = 0;
            // With early set, the caller guarantees that no kernel before this
            // one on the stream writes W: the first slots fill while that
            // kernel finishes.
            if (early) {
                for (; k < nslot && k < nfill; k++) fill(k);
                prefetch_rest();
            }
            pdl_wait();
            if (!early) prefetch_rest();
            for (; k < nfill; k++) {
                const int slot = k % nslot;
                if (k >= nslot && !bar_wait(empty0 + 8 * slot, (uint32_t)((k / nslot - 1) & 1), abort, err, 0x4D4D01))
                    break;
                fill(k);
            }
            // the copies in flight land before the CTA exits
            for (int j = k - 1; j >= 0 && j >= k - nslot; j--)
                bar_wait(full0 + 8 * (j % nslot), (uint32_t)((j / nslot) & 1), abort, err, 0x4D4D02, false);
        }
        return;
    }
    pdl_wait();
    if (QT == 4 && direct && warp >= nwork && warp < MM_WARPS) {
        // the spare warps' shares of the direct units into L1 while x is
        // prepared (the producer has asked L2 for them)
        const int nspare = MM_WARPS - nwork, dp = warp - nwork;
        const int sg = (int)((sigma >> (3 * g)) & 7u);
        for (int k = nslot; k < nunits; k++) {
            int seg, tile;
            unit_of(k, seg, tile);
            const int steps = min(spb, nsb - seg * spb);
            const int i0 = dp * steps / nspare, i1 = (dp + 1) * steps / nspare;
            for (int h = 0; h < 2; h++) {
                const int r = tile * 16 + sg + 8 * h;
                if (r >= N) continue;
                const uint8_t *row = static_cast<const uint8_t *>(Wg) + ((size_t)r * nsb + (size_t)seg * spb) * BB;
                // lane t: byte 0, 48, 96 or 143 of each 144-byte superblock,
                // so every 128-byte line it touches is asked for
                for (int i = i0; i < i1; i++)
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(row + (size_t)i * BB + (t < 3 ? 48 * t : BB - 1)));
            }
        }
    }

    // x pieces of the CTA's superblocks: warp per superblock, lane l holds
    // x 8l .. 8l+7 (sub-block l/4, positions 8(l%4) ..)
    for (int i = warp; i < nsl; i += MM_WARPS) {
        const float4 *xv = reinterpret_cast<const float4 *>(x + (size_t)(sb0 + i) * 256 + 8 * lane);
        const float4 va = __ldg(xv), vb = __ldg(xv + 1);
        float v[8] = { va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w };
        float mx = 0.0f, sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            mx = fmaxf(mx, fabsf(v[k]));
            sum += v[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
        int e = 0;
        if (mx > 0.0f) frexpf(mx, &e);                              // max|x| < 2^e
        e = max(e, -110);                                           // keeps 2^(e-13) and 2^(6-e) normal floats
        const float sc = __uint_as_float((uint32_t)(127 + 6 - e) << 23);   // 2^(6-e): |v sc| < 64
        uint8_t *xsb = smx + (size_t)i * XSB;
        uint32_t pw[4][2];
        int psum[4] = { 0, 0, 0, 0 };                               // this lane's sum of each piece
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float r[4], p[4][4];
#pragma unroll
            for (int k = 0; k < 4; k++) r[k] = v[4 * h + k] * sc;   // exact
#pragma unroll
            for (int piece = 0; piece < 4; piece++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    p[piece][k] = rintf(r[k]);
                    r[k] = (r[k] - p[piece][k]) * 128.0f;           // exact; |r| <= 64
                }
#pragma unroll
            for (int piece = 0; piece < 4; piece++) {
                pw[piece][h] = pack4(p[piece][0], p[piece][1], p[piece][2], p[piece][3]);
                if constexpr (QT == 6)
                    psum[piece] += __float2int_rn(p[piece][0]) + __float2int_rn(p[piece][1]) +
                                   __float2int_rn(p[piece][2]) + __float2int_rn(p[piece][3]);
            }
        }
        const int j = lane >> 2, pos = 8 * (lane & 3);
#pragma unroll
        for (int piece = 0; piece < 4; piece++)
            *reinterpret_cast<uint2 *>(xsb + j * 128 + piece * 32 + pos) = make_uint2(pw[piece][0], pw[piece][1]);
        const float xe = __uint_as_float((uint32_t)(127 + e - 13) << 23);
        if constexpr (QT == 4) {
            if ((lane & 3) == 0) reinterpret_cast<float *>(xsb + 1024)[j] = sum;
            if (lane == 0) *reinterpret_cast<float *>(xsb + 1024 + 32) = xe;
        } else {
            // -32 (sum of each piece over a 16-weight half): lanes 2s, 2s+1 of a group's four
#pragma unroll
            for (int piece = 0; piece < 4; piece++) psum[piece] += __shfl_xor_sync(0xFFFFFFFFu, psum[piece], 1);
            if ((lane & 1) == 0)
                *reinterpret_cast<int4 *>(xsb + 1024 + (2 * j + ((lane >> 1) & 1)) * 16) =
                    make_int4(-32 * psum[0], -32 * psum[1], -32 * psum[2], -32 * psum[3]);
            if (lane == 0) *reinterpret_cast<float *>(xsb + 1280) = xe;
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(MM_WARPS * 32) : "memory");    // the consumers only

    // A unit's sums of rows sg, sg + 8 (every lane of the warp holds its
    // quad's): into y, or the K segment's partial sum, the last of a tile's
    // S partial sums to arrive adding them in segment order
    const int SP = S;
    const auto emit = [&](float acc0, float acc1, int seg, int tile, int sg) {
        const int r0 = tile * 16 + sg, r1 = r0 + 8;
        if (SP == 1) {
            if (t == 0) {
                if (r0 < N) y[r0] = acc0;
                if (r1 < N) y[r1] = acc1;
            }
            return;
        }
        const int ps = seg;                                         // this partial sum's index
        if (tm) {
            // the last of the tile's SP parts in this CTA sums them in order
            const int tl = tile - T0;
            float *tp = tpart + ((size_t)tl * SP + ps) * 16;
            if (t == 0) {
                tp[sg] = acc0;
                tp[sg + 8] = acc1;
            }
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(tcnt + tl, 1) == SP - 1;
            }
            last = __shfl_sync(0xFFFFFFFFu, last, 0);
            if (last) {
                __threadfence_block();
                const int r = tile * 16 + lane;
                if (lane < 16 && r < N) {
                    float v = 0.0f;
                    for (int q = 0; q < SP; q++) v += tpart[((size_t)tl * SP + q) * 16 + lane];
                    y[r] = v;
                }
            }
            return;
        }
        if (t == 0) {
            if (r0 < N) ws[(size_t)ps * N + r0] = acc0;
            if (r1 < N) ws[(size_t)ps * N + r1] = acc1;
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atom_add_acq_rel(cnt + tile, 1) == SP - 1;
        last = __shfl_sync(0xFFFFFFFFu, last, 0);
        if (last) {
            __syncwarp();
            const int r = tile * 16 + lane;
            if (lane < 16 && r < N) {
                float v = 0.0f;
                for (int s = 0; s < SP; s++) v += __ldcg(ws + (size_t)s * N + r);
                y[r] = v;
            }
            if (lane == 0) cnt[tile] = 0;                           // ready for the next call
        }
    };
    // the parts' sums of rows sg, sg + 8 (np warps, part p, buffer cb of two
    // alternating ones, named barrier id): part 0's lanes get the totals
    const auto meet = [&](float &acc0, float &acc1, float *cb, int p, int np, int id, int sg) {
        if (t == 0) {
            cb[p * 16 + sg] = acc0;
            cb[p * 16 + sg + 8] = acc1;
        }
        asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(32 * np) : "memory");
        if (p != 0) return false;
        acc0 = acc1 = 0.0f;
        for (int q = 0; q < np; q++) {
            acc0 += cb[q * 16 + sg];
            acc1 += cb[q * 16 + sg + 8];
        }
        return true;
    };
    const int sg = (int)((sigma >> (3 * g)) & 7u);                  // this lane's slot row (and row + 8)

    if (direct && warp >= nwork) {
        // Units past the slots (Q4_K, at most a few per CTA): the nspare
        // warps the slots leave idle read them from global memory (L2 and
        // L1 have been asked for them), a share of each unit's superblocks
        // per warp
        if constexpr (QT == 4) {
            const int nspare = MM_WARPS - nwork, dp = warp - nwork;
            const size_t rowb = (size_t)nsb * BB;
            for (int k = nslot, j = 0; k < nunits; k++, j++) {
                int seg, tile;
                unit_of(k, seg, tile);
                const int steps = min(spb, nsb - seg * spb);
                const int i0 = dp * steps / nspare, i1 = (dp + 1) * steps / nspare;
                const int ra = tile * 16 + sg, rb = ra + 8;
                const uint8_t *w0 = static_cast<const uint8_t *>(Wg);
                const uint8_t *g0 = ra < N ? w0 + (size_t)ra * rowb + (size_t)seg * spb * BB : nullptr;
                const uint8_t *g1 = rb < N ? w0 + (size_t)rb * rowb + (size_t)seg * spb * BB : nullptr;
                const uint8_t *xs = smx + (size_t)(seg * spb - sb0) * XSB;
                float acc0 = 0.0f, acc1 = 0.0f;
                for (int i = i0; i < i1; i++) {
                    Sb sb;
                    load_sb_global(sb, g0, g1, i * BB, t);
                    sb_dot(sb, xs + (size_t)i * XSB, g, t, acc0, acc1);
                }
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 1);
                acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 2);
                acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 2);
                if (nspare > 1 && !meet(acc0, acc1, cmb + (size_t)nwork * 32 + (size_t)(j & 1) * nspare * 16, dp,
                                        nspare, 15, sg))
                    continue;
                emit(acc0, acc1, seg, tile, sg);
            }
        }
        return;
    }

    // Consumers: owners of hs warps each. Unit k lives in slot k % nslot and
    // belongs to the slot's owner, (k % nslot) % owners: every slot is read
    // by one owner only, in unit order, so a warp never tests a slot's
    // barrier while an earlier fill of that slot is still pending (which its
    // parity test would read as complete). The hs warps (parts) of an owner
    // take a share of the unit's superblocks each and add their sums in
    // shared memory, in part order; part 0 emits the unit's sum. With
    // direct set the slots hold units 0 .. nslot - 1 only.
    const int owner = warp / hs, part = warp - owner * hs, owners = nwork / hs;
    const int nslotted = direct ? min(nunits, nslot) : nunits;
    // rounds of nslot units, the owner's slots in each (no division per unit)
    int seq = 0;                                                    // units this owner has taken
    for (int round = 0, kr = 0; warp < nwork && kr < nslotted; round++, kr += nslot)
    for (int slot = owner; slot < nslot && kr + slot < nslotted; slot += owners) {
        const int k = kr + slot;
        int seg, tile;
        unit_of(k, seg, tile);
        const bool ok = bar_wait(full0 + 8 * slot, (uint32_t)(round & 1), abort, err, 0x4D4D03);
        float acc0 = 0.0f, acc1 = 0.0f;
        if (ok) {
            const uint8_t *sl = slots + (size_t)slot * 16 * rs;
            const uint8_t *r0 = sl + (size_t)sg * rs;               // Q4_K rows; Q6_K rows are per box
            const uint8_t *r1 = r0 + (size_t)8 * rs;
            const uint8_t *xs = smx + (size_t)(seg * spb - sb0) * XSB;
            const int steps = min(spb, nsb - seg * spb);            // the last segment of a row may be short
            const int i0 = hs > 1 ? part * steps / hs : 0, i1 = hs > 1 ? (part + 1) * steps / hs : steps;
            if constexpr (QT == 4) {
                for (int i = i0; i < i1; i++) {
                    Sb sb;
                    load_sb_smem(sb, r0 + i * BB, r1 + i * BB, t);
                    sb_dot(sb, xs + (size_t)i * XSB, g, t, acc0, acc1);
                }
            } else {
                // steps = spb (8 or 16), a multiple of 2 hs: this part's share starts even
                for (int i = i0; i < i1; i += 2) {
                    const uint8_t *q0 = sl + (size_t)(i / MQ_SPB) * 16 * RB + (size_t)sg * RB + (i % MQ_SPB) * BB;
                    const uint8_t *q1 = q0 + (size_t)8 * RB;
                    sb6_dot<false>(q0, q1, xs + (size_t)i * XSB, g, t, acc0, acc1);
                    sb6_dot<true>(q0 + BB, q1 + BB, xs + (size_t)(i + 1) * XSB, g, t, acc0, acc1);
                }
            }
        }
        __syncwarp();
        if (lane == 0) bar_arrive(empty0 + 8 * slot);               // the slot's bytes are read
        // the quad's four shares of rows g and g+8
        acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
        acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 1);
        acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 2);
        acc1 += __shfl_xor_sync(0xFFFFFFFFu, acc1, 2);
        // two buffers per owner, so that the next unit's sums never overwrite
        // these before part 0 has read them (it must pass the next barrier first)
        if (hs > 1 && !meet(acc0, acc1, cmb + ((size_t)owner * 2 + (seq++ & 1)) * hs * 16, part, hs, 2 + owner, sg))
            continue;
        emit(acc0, acc1, seg, tile, sg);
    }
}

// Working memory of this host thread's calls on a device: per-tile arrival
// counters (zero between calls) and the segments' partial sums. Grown on
// demand; calls of one thread are stream-ordered, so they never share it.
struct MmBuf {
    uint8_t *p = nullptr;
    size_t bytes = 0;
    int cnt_cap = 0;
};
thread_local MmBuf g_mm[64];

}  // namespace

int g_mv_mma = 1;          // 1 (default): Q4_K matvec on this kernel where it applies
int g_mv_mma_segs = 0;     // tuning hook: K segments per tile (0: chosen per shape)
int g_mv_early = 0;        // 1: the caller's weights are never written by the kernel before a matvec
int g_mv_slots = 0;        // tuning hook: most unit slots per CTA (0: as many as shared memory holds)
int g_mv_split = 1;        // tuning hook: warps per unit (1: by shape, 0: one, 2 or 4)
int g_mv_tiles = -1;       // tuning hook: 1 whole tiles per CTA, 0 segment-major ranges, -1 by shape
int g_mv_direct = 1;       // tuning hook: 0 refills slots instead of reading the units past them directly

// Tiles from which whole tiles go to each CTA (tile-major, no global
// partial sums): six per SM at least, so that shares differ by 1/6 at most
// (measured back to back on B200: Q4_K 14336 x 4096, 896 tiles, 13.4 ->
// 12.1 us; with fewer tiles per SM the imbalance and preparing all of x
// cost more than the global partial sums: 4096 x 14336 13.6 -> 16.5 us,
// 9473 x 14336 23.6 -> 28.4 us, Q6_K 4096 x 14336 16.4 -> 19.8 us).
static int mm_tile_major_min(int sms) { return 6 * sms; }

// Superblocks per unit (the last segment of a row may be shorter): a row of
// at most 8 superblocks is one unit; otherwise 5-8 superblocks, the fewest
// padding columns in the last segment, then closest to 7 (measured, back to
// back on B200: 16 x 7-superblock units give 12.3 us for 4096 x 14336
// against 13.3 us with 8 superblocks and 15.0 us with 4; 14336 x 4096 runs
// 12.8 us with 8 superblocks, 13.6 with 16 and 14.7 with 4; units of one or
// two superblocks are several times slower).
static int mm_unit_superblocks(int nsb)
{
    if (nsb <= 8) return nsb;
    int best = 7, best_pad = 1 << 30;
    for (int spb : { 7, 8, 6, 5 }) {
        const int pad = (nsb + spb - 1) / spb * spb - nsb;
        if (pad < best_pad) {
            best_pad = pad;
            best = spb;
        }
    }
    return best;
}

typedef CUresult (*EncodeFn3)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn3 mm_encode_fn()
{
    static EncodeFn3 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeFn3)p;
        else
            cudaGetLastError();
    }
    return fn;
}

// The order in which MMA rows g = 0..7 read the slot's rows (and rows + 8),
// three bits each: a half-warp's lanes (rows g = 0..3, then 4..7, quad lanes
// t = 0..3) load 8 bytes at word (rs/4) * sigma(g) + 2t (+ a common offset),
// which fall in distinct banks when the four rows' word offsets mod 32 are 8
// apart. The permutation with the fewest bank conflicts, identity first.
static uint32_t mm_sigma_search(int w)
{
    int perm[8] = { 0, 1, 2, 3, 4, 5, 6, 7 }, best[8] = { 0, 1, 2, 3, 4, 5, 6, 7 };
    int best_cost = 1 << 30;
    do {
        int cost = 0;
        for (int h = 0; h < 2; h++) {
            int banks[32] = {};
            for (int gq = 0; gq < 4; gq++)
                for (int tq = 0; tq < 4; tq++)
                    for (int b = 0; b < 2; b++) banks[(w * perm[4 * h + gq] + 2 * tq + b) % 32]++;
            int worst = 0;
            for (int b = 0; b < 32; b++) worst = banks[b] > worst ? banks[b] : worst;
            cost += worst;
        }
        if (cost < best_cost) {
            best_cost = cost;
            for (int i = 0; i < 8; i++) best[i] = perm[i];
        }
    } while (best_cost > 2 && std::next_permutation(perm, perm + 8));
    uint32_t s = 0;
    for (int i = 0; i < 8; i++) s |= (uint32_t)best[i] << (3 * i);
    return s;
}

// mm_sigma_search for the stride rs, computed once per word offset mod 32.
static uint32_t mm_sigma(int rs)
{
    static std::once_flag once[32];
    static uint32_t table[32];
    const int w = (rs / 4) % 32;
    std::call_once(once[w], [w] { table[w] = mm_sigma_search(w); });
    return table[w];
}

// This host thread's tensor map of the latest matrix (and its shape).
struct MmMap {
    const void *w = nullptr;
    int n = 0, k = 0, spb = 0, qt = 0;
    CUtensorMap map;
};
thread_local MmMap g_mm_map[64];

// The identity row order (sigma(g) = g, three bits each): Q6_K slot rows are
// 1680 bytes apart (4 banks), so rows g = 0..7 and quad lanes t = 0..3 read
// 32 distinct banks as they are.
constexpr uint32_t mm_sigma_identity()
{
    uint32_t s = 0;
    for (int i = 0; i < 8; i++) s |= (uint32_t)i << (3 * i);
    return s;
}

template <int QT>
static bool launch_matvec_mma(float *y, const void *W, const float *x, int N, int K, bool *used)
{
    constexpr int BB = MmType<QT>::BB, XSB = MmType<QT>::XSB;
    *used = false;
    if (!g_mv_mma || ((uintptr_t)W & 15) || N <= 0 || K <= 0 || K % 256) return true;
    const int nsb = K / 256, tiles = (N + 15) / 16, sms = ctx().sms > 0 ? ctx().sms : 148;
    // Q6_K: a row is a whole number of 1680-byte (8-superblock) segments, so
    // the rows and the segments start on 16-byte boundaries (TMA's rule)
    if (QT == 6 && nsb % MQ_SPB) return true;
    // spb superblocks per unit, S segments per row (the last one may be short);
    // Q6_K: whole rows of one or two 1680-byte boxes, else 8-superblock segments
    const int spb = QT == 6 ? (nsb <= 2 * MQ_SPB ? nsb : MQ_SPB)
                            : g_mv_mma_segs > 0 ? (nsb + g_mv_mma_segs - 1) / g_mv_mma_segs : mm_unit_superblocks(nsb);
    const int S = (nsb + spb - 1) / spb;
    if (spb > 256) return true;                                  // a box holds at most 256 superblocks
    const long long U = (long long)tiles * S;
    // whole tiles per CTA (their segments summed in shared memory) where a
    // row has several segments and the tiles spread over every SM
    const int tm = S > 1 && (g_mv_tiles == 1 || (g_mv_tiles < 0 && tiles >= mm_tile_major_min(sms))) ? 1 : 0;
    // With the static-weights promise each matvec lets the next be scheduled
    // as its CTAs retire, and the next one's last CTA gets the SM of this
    // one's last CTA only after this grid has completed: it starts ~2 us
    // late and ends last (measured per CTA, Q4_K 4096 x 14336 back to back).
    // One CTA fewer than SMs leaves an SM for that CTA instead.
    const int gmax = sms - (QT == 4 && g_mv_early && sms > 1 ? 1 : 0);
    const int G = tm ? (tiles < gmax ? tiles : gmax) : (int)(U < gmax ? U : gmax);
    // the most superblocks of x, and units, one CTA holds
    int nsl_max = 0, units_max = 0, tiles_max = 0;
    for (int c = 0; c < G; c++) {
        if (tm) {
            const int n = (int)((long long)tiles * (c + 1) / G - (long long)tiles * c / G);
            tiles_max = n > tiles_max ? n : tiles_max;
            continue;
        }
        const long long u0 = U * c / G, u1 = U * (c + 1) / G;
        const int first = (int)(u0 / tiles) * spb, last = (int)((u1 - 1) / tiles + 1) * spb;
        const int n = (last < nsb ? last : nsb) - first;
        nsl_max = n > nsl_max ? n : nsl_max;
        units_max = (int)(u1 - u0) > units_max ? (int)(u1 - u0) : units_max;
    }
    if (tm) {
        nsl_max = nsb;
        units_max = tiles_max * S;
    }
    const int rs = spb * BB;
    const size_t cap = 232448;                                   // the most dynamic shared memory of a CTA
    const size_t x_bytes = ((size_t)nsl_max * XSB + 127) & ~(size_t)127;
    const size_t slot = (size_t)16 * rs;
    // combine buffers: the parts' sums (hs > 1 or direct units); tm: the
    // tiles' partial sums (one per K segment) and counters
    const size_t tm_bytes = tm ? (size_t)tiles_max * (S * 16 + 1) * 4 : 0;
    const auto slots_for = [&](size_t cmb) {
        if (x_bytes + 2 * (slot + 16) + 16 + cmb > cap) return 0;
        int n = (int)((cap - x_bytes - 16 - cmb) / (slot + 16));
        if (g_mv_slots >= 2 && n > g_mv_slots) n = g_mv_slots;
        return n < units_max ? n : units_max;                    // at most every unit its own slot
    };
    int nslot = slots_for(tm_bytes);
    if (!nslot) return true;                                     // not two slots: the CUDA-core kernels
    // hs warps (parts) per unit, a share of its superblocks each, their sums
    // met in shared memory (two buffers per owner). Q6_K units are long and
    // few fit: two or four parts of four superblocks at least, while the
    // warps allow. Q4_K keeps one warp per unit: measured back to back
    // (4096 x 14336), two parts ran 14.6 us and four 17.1 against 12.8; the
    // parts' barriers and uneven shares cost more than they save. Then
    // owners = min(nslot, MM_WARPS / hs) groups of hs warps take the slots.
    int hs = 1;
    if (g_mv_split == 2 || g_mv_split == 4) {
        hs = g_mv_split;
    } else if (g_mv_split && QT == 6) {
        const int o = nslot < MM_WARPS ? nslot : MM_WARPS;
        while (hs < 4 && 2 * hs * o <= MM_WARPS && spb / (2 * hs) >= 4) hs *= 2;
    }
    // direct (Q4_K): the units past the slots, at most three per CTA and
    // three superblocks per idle warp, go to the consumer warps the slots
    // leave idle, read from global memory, so that no slot is refilled: a
    // refill waits for its slot's whole first unit to be consumed, and the
    // CTA's last unit then starts late (measured back to back, 4096 x 14336:
    // 13.0 -> 11.2 us; with 24 superblocks on 5 warps, 14336 x 4096, 13.0 ->
    // 13.8 us)
    const bool direct_try = QT == 4 && g_mv_direct && hs == 1 && units_max > nslot && units_max - nslot <= 3 &&
                            nslot < MM_WARPS && (units_max - nslot) * spb <= 3 * (MM_WARPS - nslot);
    const size_t cmb_bytes = tm_bytes + (hs > 1 || direct_try ? MM_CMB_FLOATS * 4 : 0);
    if (hs > 1 || direct_try) nslot = slots_for(cmb_bytes);
    if (!nslot) return true;
    const int owners = nslot < MM_WARPS / hs ? nslot : MM_WARPS / hs;
    const int nwork = owners * hs;
    const int direct =
        direct_try && nwork < MM_WARPS && units_max - nslot <= 3 && (units_max - nslot) * spb <= 3 * (MM_WARPS - nwork)
            ? 1 : 0;
    const size_t smem = x_bytes + (size_t)nslot * slot + (size_t)nslot * 16 + 16 + cmb_bytes;
    float *ws = nullptr;
    int *cnt = nullptr;
    if (S > 1 && !tm) {
        MmBuf &b = g_mm[ctx().device & 63];
        const int cnt_cap = tiles > b.cnt_cap ? tiles : b.cnt_cap;
        const size_t cnt_bytes = ((size_t)cnt_cap * 4 + 255) & ~(size_t)255;
        const size_t need = cnt_bytes + (size_t)S * N * 4;
        if (need > b.bytes || cnt_cap > b.cnt_cap) {
            if (b.p) {
                TCG_CUDA(cudaStreamSynchronize(ctx().cur));
                cudaFree(b.p);
                b.p = nullptr;
                b.bytes = 0;
            }
            const size_t want = need + need / 4;
            if (cudaMalloc(&b.p, want) != cudaSuccess) {
                cudaGetLastError();
                return fail("matvec working memory of %zu bytes: out of memory", want);
            }
            TCG_CUDA(cudaMemsetAsync(b.p, 0, want, ctx().cur));
            b.bytes = want;
            b.cnt_cap = cnt_cap;
        }
        cnt = (int *)b.p;
        ws = (float *)(b.p + (((size_t)b.cnt_cap * 4 + 255) & ~(size_t)255));
    }
    const int dev = ctx().device & 63;
    MmMap &mp = g_mm_map[dev];
    if (mp.w != W || mp.n != N || mp.k != K || mp.spb != spb || mp.qt != QT) {
        EncodeFn3 fn = mm_encode_fn();
        if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
        CUresult r;
        if constexpr (QT == 4) {
            // 32-bit words: 36 per superblock, nsb superblocks per row, N rows
            cuuint64_t dims[3] = { (cuuint64_t)(BB / 4), (cuuint64_t)nsb, (cuuint64_t)N };
            cuuint64_t strides[2] = { (cuuint64_t)BB, (cuuint64_t)nsb * BB };
            cuuint32_t box[3] = { (cuuint32_t)(BB / 4), (cuuint32_t)spb, 16 };
            cuuint32_t estr[3] = { 1, 1, 1 };
            r = fn(&mp.map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, (void *)W, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        } else {
            // 8-byte elements: nsb * 210 / 8 per row, N rows; a box is 1680 bytes (8 superblocks) of 16 rows
            cuuint64_t dims[2] = { (cuuint64_t)nsb * BB / 8, (cuuint64_t)N };
            cuuint64_t strides[1] = { (cuuint64_t)nsb * BB };
            cuuint32_t box[2] = { (cuuint32_t)(MQ_SPB * BB / 8), 16 };
            cuuint32_t estr[2] = { 1, 1 };
            r = fn(&mp.map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, (void *)W, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        }
        if (r != CUDA_SUCCESS) {
            mp.w = nullptr;
            return fail("cuTensorMapEncodeTiled failed (%d) for the Q%d_K matrix [%d x %d]", (int)r, QT, N, K);
        }
        mp.w = W;
        mp.n = N;
        mp.k = K;
        mp.spb = spb;
        mp.qt = QT;
    }
    static unsigned done[64];
    if (!(done[dev] & (1u << QT))) {
        TCG_CUDA(cudaFuncSetAttribute(mv_kq_mma_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap));
        done[dev] |= 1u << QT;
    }
    const uint32_t sigma = QT == 4 ? mm_sigma(rs) : mm_sigma_identity();
    TCG_CUDA(launch_pdl(mv_kq_mma_kernel<QT>, dim3(G), dim3(MM_THREADS), smem, ctx().cur, mp.map, x, y, N, nsb, spb,
                        S, tiles, U, ws, cnt, nslot, nwork, hs, tm, sigma, (int)x_bytes, g_mv_early, W, direct,
                        ctx().d_err));
    *used = true;
    return true;
}

bool launch_matvec_mma_q4k(float *y, const void *W, const float *x, int N, int K, bool *used)
{
    return launch_matvec_mma<4>(y, W, x, N, K, used);
}

bool launch_matvec_mma_q6k(float *y, const void *W, const float *x, int N, int K, bool *used)
{
    return launch_matvec_mma<6>(y, W, x, N, K, used);
}

}  // namespace tcg

// Tuning and test hook: 1 (default) runs the Q4_K and Q6_K matvecs on the
// integer mma.sync kernel where it applies, 0 on the CUDA-core kernels.
// Returns the previous setting.
extern "C" int tcg_matvec_set_mma(int on)
{
    const int old = tcg::g_mv_mma;
    tcg::g_mv_mma = on ? 1 : 0;
    return old;
}

// Tuning hook: K segments per 16-row tile of the integer mma.sync matvec
// (units of ceil(superblocks per row / segs) superblocks; 0 restores the
// choice per shape). Returns the previous setting.
extern "C" int tcg_matvec_mma_segments(int segs)
{
    const int old = tcg::g_mv_mma_segs;
    tcg::g_mv_mma_segs = segs > 0 ? segs : 0;
    return old;
}

// Matvec promise (default 0): with 1, the caller guarantees that the kernel
// queued just before a matvec on the same stream never writes that matvec's
// weight matrix (true of a decode pass whose weights are uploaded once). The
// integer-MMA matvec then starts fetching its weights while that kernel is
// still finishing (x may still be produced by it), and lets the kernel after
// it be scheduled as its own CTAs retire. Returns the previous value.
extern "C" int tcg_matvec_set_static_weights(int on)
{
    const int old = tcg::g_mv_early;
    tcg::g_mv_early = on ? 1 : 0;
    return old;
}

// Tuning hook: at most this many unit slots (units in flight) per CTA of the
// Q4_K mma.sync matvec; 0 restores as many as shared memory holds. Returns
// the previous setting.
extern "C" int tcg_matvec_mma_slots(int n)
{
    const int old = tcg::g_mv_slots;
    tcg::g_mv_slots = n >= 2 ? n : 0;
    return old;
}

// Tuning hook: warps per unit of the integer-MMA matvec. 1 (default)
// chooses by type and shape, 0 keeps one warp per unit, 2 or 4 sets it.
// Returns the previous setting.
extern "C" int tcg_matvec_mma_split(int mode)
{
    const int old = tcg::g_mv_split;
    tcg::g_mv_split = mode == 2 || mode == 4 ? mode : mode ? 1 : 0;
    return old;
}

// Tuning hook: 1 (default) lets the idle consumer warps of the Q4_K
// integer-MMA matvec read the few units past a CTA's slots from global
// memory; 0 refills the slots instead. Returns the previous setting.
extern "C" int tcg_matvec_mma_direct(int on)
{
    const int old = tcg::g_mv_direct;
    tcg::g_mv_direct = on ? 1 : 0;
    return old;
}

// Tuning hook: 1 gives every CTA of the integer mma.sync matvec whole tiles
// (a tile's K segments summed in shared memory), 0 contiguous ranges of
// segment-major units (split tiles summed through global memory), -1
// (default) chooses by shape. Returns the previous setting.
extern "C" int tcg_matvec_mma_tiles(int mode)
{
    const int old = tcg::g_mv_tiles;
    tcg::g_mv_tiles = mode < 0 ? -1 : (mode ? 1 : 0);
    return old;
}

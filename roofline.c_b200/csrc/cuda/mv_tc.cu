// mv_tc.cu -- the Q4_K matvec y = W x on the tensor cores (tcgen05 kind::i8).
//
// The Q4_K arm of the dequant seam (roofline.c src/dequant.c:40-63 with
// ggml's Q4_K block: d, dmin, twelve bytes of 6-bit scales and mins, 128
// bytes of nibbles) gives weight k of 32-weight sub-block j the value
// (d*sc_j)*q_k - (dmin*m_j), so a row's dot product regroups as
//     y_r = sum_j (d*sc_j) * sum_{k in j} q_k x_k  -  (dmin*m_j) * sum_{k in j} x_k.
// The inner sums over q run on the tensor cores in exact integer arithmetic:
//   - A: the nibbles q (0..15) as int8, 128 rows x 256 weights per tile,
//     unpacked by the CUDA cores from the raw superblocks (one mask per four
//     weights) and stored into TMEM (row r in lane r, four weights per
//     column), so that A costs no shared-memory bandwidth;
//   - B: each sub-block of x, scaled by a power of two to |v| < 64, split into
//     four int8 pieces v = p0 + p1/2^7 + p2/2^14 + p3/2^21 (the rest is below
//     2^-22 of the sub-block's largest |v|), built once per call by
//     mvq_prep_kernel. Piece p of sub-block j sits in B row 4(j%4)+p and is
//     zero outside the sub-block's 32 weights, so one M=128 N=16 K=32 MMA per
//     sub-block leaves its four piece sums in TMEM columns 16(j/4)+4(j%4)+p
//     and four sub-blocks accumulate into one 16-column group;
//   - epilogue: per row and sub-block, (p0 + (p1 + (p2 + p3/2^7)/2^7)/2^7)
//     times 2^(e-5) times d*sc_j, minus dmin*m_j times the sub-block's sum of x.
// Results differ from the dequantise-then-dot order by rounding only.
//
// Work: stages of (128-row tile, two superblock columns), so that every row
// of a TMA box is 288 contiguous bytes, tile-major, split evenly over one
// persistent CTA per SM. A CTA that covers a whole tile writes y; tiles shared
// by several CTAs are summed in CTA order by the last CTA to finish its part
// (a per-tile arrival counter that the summing CTA resets), so every call
// gives the same bits.
//
// Roles (576 threads): warps 0-15 convert (thread = row r, 32-byte quant
// group g of the superblock) and run the epilogue of the previous superblock;
// warp 16 lane 0 loads stages with TMA (raw tile) and bulk copies (B tiles, x
// factors); warp 17 owns TMEM and lane 0 issues the MMAs. Every wait is
// bounded; on a timeout the kernel raises the device error word and still
// completes the tile arrivals so the counters stay consistent.
#include "tcg_common.cuh"
#include "tc05.cuh"

#include <cuda.h>

namespace tcg {

namespace {

constexpr int MQ_BB = 144;                       // Q4_K bytes per superblock
constexpr int MQ_SPS = 2;                        // superblocks per stage (contiguous bytes per row)
constexpr int MQ_ROW = MQ_SPS * MQ_BB;           // raw bytes of one row in a stage
constexpr int MQ_RAW = 128 * MQ_ROW;             // raw tile: 128 rows
constexpr int MQ_BT = 4096;                      // B tile: 16 rows x 256 int8, two 128-byte atoms
constexpr int MQ_F = 64;                         // x factors: 2^(e_j - 5), sum_j x  (8 + 8 floats)
constexpr int MQ_OFF_RAW = MQ_SPS * MQ_BT;       // stage: B tiles, raw tile, factors
constexpr int MQ_OFF_F = MQ_OFF_RAW + MQ_RAW;
constexpr int MQ_STAGE = (MQ_OFF_F + MQ_SPS * MQ_F + 1023) & ~1023;
constexpr int MQ_R = 4;                          // stages in flight
constexpr int MQ_CONV = 512;                     // converter threads: row r, 32-byte quant group g
constexpr int MQ_THREADS = MQ_CONV + 64;
constexpr int MQ_TMEM = 256;                     // accumulators at columns 0 / 32, A tiles at 64 / 128
constexpr uint32_t MQ_ACOL = 64;                 // A tile: 128 lanes x 64 columns (4 int8 per column)
constexpr size_t MQ_SMEM_USED = (size_t)MQ_R * MQ_STAGE + 2048;
constexpr size_t MQ_SMEM = MQ_SMEM_USED + 1024;  // + alignment slack

static_assert(MQ_SMEM <= 232448, "shared memory");

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// 16 columns of this thread's TMEM lane from registers; waits for the store.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
                 " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
                 "tcgen05.wait::st.sync.aligned;"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                   "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
                   "r"(v[15])
                 : "memory");
}

// A from TMEM (row i in lane i, four int8 of K per column), B from shared memory.
__device__ __forceinline__ void mma_i8_ts(uint32_t d, uint32_t a_tmem, unsigned long long b, uint32_t id, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
                 ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}

__device__ __forceinline__ void named_bar(int id, int count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// D s32, A and B signed 8-bit, both K-major, N = 16, M = 128.
constexpr uint32_t MQ_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ float f16_exact(uint32_t h)
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
        const uint32_t shift = 10u - (31u - (uint32_t)__clz(f));
        bits = sign | ((113u - shift) << 23) | (((f << shift) & 0x3FFu) << 13);
    }
    return __uint_as_float(bits);
}

// One CTA per superblock column s, one warp per sub-block j: the B tile of x
// (layout above) and the factors 2^(e_j - 5) and sum_j x. e_j is the exponent
// of the sub-block's largest |x|, kept >= -120 so that 2^(5 - e_j) stays a
// normal float.
__global__ void __launch_bounds__(256)
mvq_prep_kernel(const float *__restrict__ x, uint8_t *__restrict__ Bt, float *__restrict__ F)
{
    __shared__ __align__(16) uint8_t tile[MQ_BT];
    const int s = blockIdx.x, tid = threadIdx.x, j = tid >> 5, k = tid & 31;
    reinterpret_cast<uint4 *>(tile)[tid] = make_uint4(0u, 0u, 0u, 0u);
    const float xv = x[(size_t)s * 256 + tid];
    uint32_t mb = __float_as_uint(xv) & 0x7FFFFFFFu;
#pragma unroll
    for (int o = 16; o; o >>= 1) mb = max(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, o));
    int e = (int)(mb >> 23) - 127;
    e = e < -120 ? -120 : (e > 127 ? 127 : e);
    float rr = __fmul_rn(xv, __uint_as_float((uint32_t)(127 + 5 - e) << 23));   // |rr| < 64, exact
    int p[4];
#pragma unroll
    for (int pp = 0; pp < 4; pp++) {
        const float q = rintf(rr);
        p[pp] = (int)q;
        rr = __fmul_rn(__fsub_rn(rr, q), 128.0f);                               // exact
    }
    float X = xv;
#pragma unroll
    for (int o = 16; o; o >>= 1) X += __shfl_xor_sync(0xFFFFFFFFu, X, o);
    __syncthreads();
    const int jj = j & 3, kk = 32 * jj + k;
#pragma unroll
    for (int pp = 0; pp < 4; pp++) {
        const int n = 4 * jj + pp;
        tile[(j >> 2) * 2048 + n * 128 + ((((kk >> 4) ^ (n & 7)) & 7) << 4) + (kk & 15)] = (uint8_t)(int8_t)p[pp];
    }
    if (k == 0) {
        F[(size_t)s * 16 + j] = __uint_as_float((uint32_t)(127 + e - 5) << 23);
        F[(size_t)s * 16 + 8 + j] = X;
    }
    __syncthreads();
    reinterpret_cast<uint4 *>(Bt + (size_t)s * MQ_BT)[tid] = reinterpret_cast<const uint4 *>(tile)[tid];
}

__device__ __forceinline__ int mq_owner(long long u, int G, long long U)
{
    return (int)(((u + 1) * G - 1) / U);
}
__device__ __forceinline__ long long mq_first(int c, int G, long long U)
{
    return (long long)c * U / G;
}

__global__ void __launch_bounds__(MQ_THREADS, 1)
mvq_tc_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t *__restrict__ Bt, const float *__restrict__ F,
              float *__restrict__ y, float *__restrict__ P, int *__restrict__ cnt, int N, int nb, long long U, int *err)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(sm + (size_t)MQ_R * MQ_STAGE);
    uint64_t *full = bars, *empty = bars + MQ_R, *afull = bars + 2 * MQ_R, *mdone = bars + 2 * MQ_R + 2;
    uint64_t *fin = bars + 2 * MQ_R + 4;
    uint32_t *tmem_slot = (uint32_t *)(fin + 1);
    volatile int *abort = (volatile int *)(tmem_slot + 1);
    volatile int *lastflag = (volatile int *)(tmem_slot + 2);
    float *red = (float *)(tmem_slot + 4);                       // [3][128]

    const int tid = threadIdx.x, warp = tid >> 5, G = (int)gridDim.x, c = (int)blockIdx.x;
    const int nbp = (nb + MQ_SPS - 1) / MQ_SPS;                  // stages per row tile
    const long long u0 = mq_first(c, G, U), u1 = mq_first(c + 1, G, U);
    const int n = (int)(u1 - u0);                                // this CTA's stages
    auto stage_sbs = [&](int i) {                                // superblocks in stage i
        const int sp = (int)((u0 + i) % nbp);
        return min(MQ_SPS, nb - sp * MQ_SPS);
    };

    if (tid == 0) {
        for (int i = 0; i < MQ_R; i++) {
            bar_init(su32(full + i), 1);
            bar_init(su32(empty + i), MQ_CONV + 1);
        }
        for (int i = 0; i < 2; i++) {
            bar_init(su32(afull + i), MQ_CONV);
            bar_init(su32(mdone + i), 1);
        }
        bar_init(su32(fin), 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MQ_CONV / 32 + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(su32(tmem_slot)), "r"(MQ_TMEM) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == MQ_CONV / 32) {
        if ((tid & 31) == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&wmap) : "memory");
            bool waited = false;
            int issued = 0;
            for (int i = 0; i < n; i++) {
                const int st = i % MQ_R;
                if (i >= MQ_R && !bar_wait(su32(empty + st), ((i / MQ_R) + 1) & 1, abort, err, 0x4D5101)) break;
                const long long u = u0 + i;
                const int t = (int)(u / nbp), sp = (int)(u % nbp), nv = stage_sbs(i);
                uint8_t *stg = sm + (size_t)st * MQ_STAGE;
                // the box always moves MQ_RAW bytes (columns past the row end read as zero)
                bar_expect_tx(su32(full + st), MQ_RAW + nv * (MQ_BT + MQ_F));
                tma_load(su32(stg + MQ_OFF_RAW), &wmap, su32(full + st), sp * (MQ_ROW / 4), t * 128);
                if (!waited) {
                    pdl_wait();              // B tiles and factors come from the kernel before
                    waited = true;
                }
                for (int v = 0; v < nv; v++) {
                    const int s = sp * MQ_SPS + v;
                    bulk_load(su32(stg + v * MQ_BT), Bt + (size_t)s * MQ_BT, MQ_BT, su32(full + st));
                    bulk_load(su32(stg + MQ_OFF_F + v * MQ_F), F + (size_t)s * 16, MQ_F, su32(full + st));
                }
                issued = i + 1;
            }
            // no copy may still be landing when the CTA exits
            for (int i = issued > MQ_R ? issued - MQ_R : 0; i < issued; i++)
                bar_wait(su32(full + i % MQ_R), (i / MQ_R) & 1, abort, err, 0x4D5102, false);
        }
    } else if (warp == MQ_CONV / 32 + 1) {
        if ((tid & 31) == 0) {
            int ci = 0;
            for (int i = 0; i < n; i++) {
                const int st = i % MQ_R, nv = stage_sbs(i);
                bool ok = true;
                for (int v = 0; v < nv; v++, ci++) {
                    if (!bar_wait(su32(afull + (ci & 1)), (ci >> 1) & 1, abort, err, 0x4D5103)) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint32_t a0 = tmem + MQ_ACOL * (1u + (uint32_t)(ci & 1));
                    const uint32_t b0 = su32(sm + (size_t)st * MQ_STAGE + v * MQ_BT);
                    const uint32_t d0 = tmem + (uint32_t)(ci & 1) * 32;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const unsigned long long bd = sdesc<128>(b0 + (uint32_t)(j >> 2) * 2048 + (uint32_t)(j & 3) * 32);
                        mma_i8_ts(d0 + (uint32_t)(j >> 2) * 16, a0 + 8u * (uint32_t)j, bd, MQ_IDESC, (j & 3) ? 1u : 0u);
                    }
                    mma_commit(su32(mdone + (ci & 1)));
                }
                if (!ok) break;
                mma_commit(su32(empty + st));
            }
            if (ci) {
                mma_commit(su32(fin));
                bar_wait(su32(fin), 0, abort, err, 0x4D5104, false);
            }
        }
    } else {
        // converters: row r of the tile, quant group g (bytes 32g .. 32g + 31
        // of the superblock's nibbles = sub-blocks 2g (low nibbles) and 2g + 1
        // (high nibbles) = TMEM columns 8g .. 8g + 7 of the accumulator)
        const int r = tid & 127, g = tid >> 7;
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        float acc = 0.0f;
        float pa0 = 0.f, pa1 = 0.f, pc = 0.0f;            // factors of the unit awaiting its epilogue
        int p_tile = 0;                                    // its row tile
        bool p_flush = false;                              // it ends this CTA's part of the tile
        bool ok = true;

        auto epilogue = [&](int ci) {
            bool have = ok && bar_wait(su32(mdone + (ci & 1)), (ci >> 1) & 1, abort, err, 0x4D5105);
            have = __all_sync(0xFFFFFFFFu, have);            // the TMEM load is warp-collective
            if (!have) ok = false;
            fence_after();
            uint32_t v[8];
            if (have) {
                tmem_ld8(tmem + lane_base + (uint32_t)(ci & 1) * 32 + 8u * (uint32_t)g, v);
            } else {
#pragma unroll
                for (int q = 0; q < 8; q++) v[q] = 0u;
            }
            float t0 = fmaf((float)(int)v[3], 0.0078125f, (float)(int)v[2]);
            t0 = fmaf(t0, 0.0078125f, (float)(int)v[1]);
            t0 = fmaf(t0, 0.0078125f, (float)(int)v[0]);
            float t1 = fmaf((float)(int)v[7], 0.0078125f, (float)(int)v[6]);
            t1 = fmaf(t1, 0.0078125f, (float)(int)v[5]);
            t1 = fmaf(t1, 0.0078125f, (float)(int)v[4]);
            acc = fmaf(pa0, t0, acc);
            acc = fmaf(pa1, t1, acc);
            acc -= pc;
            if (!p_flush) return;
            // end of this CTA's part of the tile: combine the four groups, then write or reduce
            const int t = p_tile;
            const long long tb = (long long)t * nbp;
            if (g) red[(g - 1) * 128 + r] = acc;
            named_bar(1, MQ_CONV);
            if (g == 0) {
                const float tot = ((acc + red[r]) + red[128 + r]) + red[256 + r];
                const int row = t * 128 + r;
                const int c_lo = mq_owner(tb, G, U), c_hi = mq_owner(tb + nbp - 1, G, U);
                if (c_lo == c_hi) {
                    if (row < N) y[row] = tot;
                } else {
                    const int slot = (t == (int)(u0 / nbp)) ? 0 : 1;
                    __stcg(P + ((size_t)c * 2 + slot) * 128 + r, tot);
                    __threadfence();
                    named_bar(2, 128);
                    if (r == 0) *lastflag = (atomicAdd(cnt + t, 1) == c_hi - c_lo) ? 1 : 0;
                    named_bar(2, 128);
                    if (*lastflag) {
                        __threadfence();
                        float sum = 0.0f;
                        for (int cc = c_lo; cc <= c_hi; cc++) {
                            const int sl = (t == (int)(mq_first(cc, G, U) / nbp)) ? 0 : 1;
                            sum += __ldcg(P + ((size_t)cc * 2 + sl) * 128 + r);
                        }
                        if (row < N) y[row] = sum;
                        if (r == 0) atomicExch(cnt + t, 0);
                    }
                }
            }
            named_bar(1, MQ_CONV);
            acc = 0.0f;
        };

        int ci = 0;
        for (int i = 0; i < n; i++) {
            const int st = i % MQ_R, nv = stage_sbs(i);
            const long long u = u0 + i;
            const int t = (int)(u / nbp), sp = (int)(u % nbp);
            if (ok && !bar_wait(su32(full + st), (i / MQ_R) & 1, abort, err, 0x4D5106)) ok = false;
            ok = __all_sync(0xFFFFFFFFu, ok);                // the TMEM store is warp-collective
            const uint8_t *stg = sm + (size_t)st * MQ_STAGE;
            for (int v = 0; v < nv; v++, ci++) {
                float na0 = 0.f, na1 = 0.f, nc = 0.0f;
                if (ok) {
                    const uint8_t *rw = stg + MQ_OFF_RAW + r * MQ_ROW + v * MQ_BB;
                    const uint4 head = *reinterpret_cast<const uint4 *>(rw);
                    const uint4 q0 = *reinterpret_cast<const uint4 *>(rw + 16 + 32 * g);
                    const uint4 q1 = *reinterpret_cast<const uint4 *>(rw + 32 + 32 * g);
                    const float *Fs = reinterpret_cast<const float *>(stg + MQ_OFF_F + v * MQ_F);
                    const float2 xsv = *reinterpret_cast<const float2 *>(Fs + 2 * g);
                    const float2 Xv = *reinterpret_cast<const float2 *>(Fs + 8 + 2 * g);
                    if (v == nv - 1) bar_arrive(su32(empty + st));

                    // row r of the A tile in TMEM: low nibbles (sub-block 2g, K 64g .. 64g + 31)
                    // to columns 16g .. 16g + 7, high nibbles (sub-block 2g + 1) to 16g + 8 .. 16g + 15
                    const uint32_t w[16] = {
                        q0.x & 0x0F0F0F0Fu, q0.y & 0x0F0F0F0Fu, q0.z & 0x0F0F0F0Fu, q0.w & 0x0F0F0F0Fu,
                        q1.x & 0x0F0F0F0Fu, q1.y & 0x0F0F0F0Fu, q1.z & 0x0F0F0F0Fu, q1.w & 0x0F0F0F0Fu,
                        (q0.x >> 4) & 0x0F0F0F0Fu, (q0.y >> 4) & 0x0F0F0F0Fu, (q0.z >> 4) & 0x0F0F0F0Fu,
                        (q0.w >> 4) & 0x0F0F0F0Fu, (q1.x >> 4) & 0x0F0F0F0Fu, (q1.y >> 4) & 0x0F0F0F0Fu,
                        (q1.z >> 4) & 0x0F0F0F0Fu, (q1.w >> 4) & 0x0F0F0F0Fu };
                    tmem_st16(tmem + lane_base + MQ_ACOL * (1u + (uint32_t)(ci & 1)) + 16u * (uint32_t)g, w);
                    fence_before();
                    bar_arrive(su32(afull + (ci & 1)));

                    // scales and mins of sub-blocks 2g and 2g + 1 (ggml's 6-bit packing:
                    // j < 4 from bytes j and j + 4, j >= 4 from bytes j + 4, j - 4 and j)
                    const float d = f16_exact(head.x & 0xFFFFu), dmin = f16_exact(head.x >> 16);
                    uint32_t sc[2], mn[2];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int j = 2 * g + e, jj = j & 3;
                        const uint32_t b0 = (head.y >> (8 * jj)) & 0xFFu;        // s[j & 3]
                        const uint32_t b4 = (head.z >> (8 * jj)) & 0xFFu;        // s[(j & 3) + 4]
                        const uint32_t b8 = (head.w >> (8 * jj)) & 0xFFu;        // s[(j & 3) + 8]
                        if (j < 4) {
                            sc[e] = b0 & 63u;
                            mn[e] = b4 & 63u;
                        } else {
                            sc[e] = (b8 & 0x0Fu) | ((b0 >> 6) << 4);
                            mn[e] = (b8 >> 4) | ((b4 >> 6) << 4);
                        }
                    }
                    na0 = __fmul_rn(__fmul_rn(d, (float)sc[0]), xsv.x);
                    na1 = __fmul_rn(__fmul_rn(d, (float)sc[1]), xsv.y);
                    nc = fmaf(__fmul_rn(dmin, (float)mn[1]), Xv.y, __fmul_rn(__fmul_rn(dmin, (float)mn[0]), Xv.x));
                }
                if (ci > 0) epilogue(ci - 1);
                pa0 = na0;
                pa1 = na1;
                pc = nc;
                p_tile = t;
                p_flush = (sp * MQ_SPS + v == nb - 1) || (i == n - 1 && v == nv - 1);
            }
        }
        if (ci > 0) epilogue(ci - 1);
    }

    fence_before();
    __syncthreads();
    if (warp == MQ_CONV / 32 + 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(MQ_TMEM) : "memory");
    }
}

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                             const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn mq_encode_fn()
{
    static EncodeFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeFn)p;
        else
            cudaGetLastError();
    }
    return fn;
}

// Working memory of this host thread's calls on a device (the library
// context is per thread too): tile counters (zero between calls), partial
// sums, B tiles and x factors. Grown (and zeroed) on demand. Calls of one
// thread must be stream-ordered: two in flight at once on different streams
// would share the counters.
struct MqBuf {
    uint8_t *p = nullptr;
    size_t bytes = 0;
    int cnt_cap = 0;
    const void *map_w = nullptr;   // tensor map cache
    int map_n = 0, map_k = 0;
    CUtensorMap map;
};
thread_local MqBuf g_mq[64];

}  // namespace

int g_mv_tc = 0;           // 1: Q4_K matvec on the tensor cores where it applies (opt-in: slower today)

bool launch_matvec_tc_q4k(float *y, const void *W, const float *x, int N, int K, bool *used)
{
    *used = false;
    if (!g_mv_tc || ((uintptr_t)W & 15) || N <= 0 || K <= 0 || K % 256) return true;
    const int nb = K / 256, RT = (N + 127) / 128, nbp = (nb + MQ_SPS - 1) / MQ_SPS;
    const long long U = (long long)RT * nbp;
    const int G = (int)(U < ctx().sms ? U : ctx().sms);
    MqBuf &b = g_mq[ctx().device & 63];
    const int cnt_cap = RT > b.cnt_cap ? RT : b.cnt_cap;
    const size_t cnt_bytes = ((size_t)cnt_cap * 4 + 255) & ~(size_t)255;
    const size_t p_bytes = (size_t)G * 2 * 128 * 4;
    const size_t need = cnt_bytes + p_bytes + (size_t)nb * MQ_BT + (size_t)nb * MQ_F;
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
    const size_t cnt_region = ((size_t)b.cnt_cap * 4 + 255) & ~(size_t)255;
    int *cnt = (int *)b.p;
    float *P = (float *)(b.p + cnt_region);
    uint8_t *Bt = b.p + cnt_region + p_bytes;
    float *F = (float *)(Bt + (size_t)nb * MQ_BT);

    if (b.map_w != W || b.map_n != N || b.map_k != K) {
        EncodeFn fn = mq_encode_fn();
        if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
        // 32-bit elements: a row is nb * 36 of them, a box MQ_SPS superblocks of 128 rows
        cuuint64_t dims[2] = { (cuuint64_t)nb * (MQ_BB / 4), (cuuint64_t)N };
        cuuint64_t strides[1] = { (cuuint64_t)nb * MQ_BB };
        cuuint32_t box[2] = { (cuuint32_t)(MQ_ROW / 4), 128 };
        cuuint32_t estr[2] = { 1, 1 };
        CUresult r = fn(&b.map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, (void *)W, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            b.map_w = nullptr;
            return fail("cuTensorMapEncodeTiled failed (%d) for the Q4_K matrix [%d x %d]", (int)r, N, K);
        }
        b.map_w = W;
        b.map_n = N;
        b.map_k = K;
    }
    static unsigned done[64];
    const int dev = ctx().device & 63;
    if (!done[dev]) {
        TCG_CUDA(cudaFuncSetAttribute(mvq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MQ_SMEM));
        done[dev] = 1;
    }
    cudaStream_t s = ctx().cur;
    mvq_prep_kernel<<<nb, 256, 0, s>>>(x, Bt, F);
    TCG_LAUNCHED();
    TCG_CUDA(launch_pdl(mvq_tc_kernel, dim3(G), dim3(MQ_THREADS), MQ_SMEM, s, b.map, (const uint8_t *)Bt,
                        (const float *)F, y, P, cnt, N, nb, U, ctx().d_err));
    *used = true;
    return true;
}

}  // namespace tcg

// Tuning and test hook: 1 runs the Q4_K matvec on the tensor cores where it
// applies, 0 (the default) on the CUDA-core kernels, which are faster: the
// stages of 128 row pieces arrive at ~2.7 TB/s and each CTA's convert -> MMA
// -> epilogue chain does not hide it. Returns the previous setting.
extern "C" int tcg_matvec_set_tc(int on)
{
    const int old = tcg::g_mv_tc;
    tcg::g_mv_tc = on ? 1 : 0;
    return old;
}

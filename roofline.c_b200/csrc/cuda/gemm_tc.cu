// gemm_tc.cu -- fp32-accurate GEMM on the 5th-generation tensor cores.
//
// C[M,N] = A[M,K] * B[N,K]^T (+ epilogue), the shape of every linear in
// roofline.c's ViT (tc_ref_linear, src/ops.c:28-35). Each fp32 operand comes
// as a tf32 pair (hi = rn(v), lo = rn(v - hi)) and every K-step issues three
// tcgen05.mma.kind::tf32 -- lo*hi, hi*lo, hi*hi -- into one fp32 TMEM
// accumulator ("3xTF32"; the dropped lo*lo term is ~2^-22 relative).
//
// Accuracy. The tensor core's own fp32 accumulation truncates, and that
// error grows linearly with the number of MMAs folded into one accumulator
// (measured: ~1.7e-5 of max|C| at K=1024 when a whole K loop accumulates in
// TMEM). So the large hi*hi term accumulates per K chunk (256 by default,
// tcg_gemm_set_chunk_k) in a fresh TMEM buffer (two, ping-pong), and the
// epilogue warps fold every chunk into fp32 registers with round-to-nearest
// adds while the MMAs of the next chunk run. The two small correction terms
// (lo*hi, hi*lo; ~2^-11 of the result) accumulate over the whole tile in their
// own TMEM buffers, where truncation costs nothing measurable. Per product
// the error is a few fp32 ulps of the result, like a sequential fp32 dot.
//
// Persistent, warp-specialised CTA (one per SM, 320 threads):
//   warp 0     one lane issues the TMA loads of a (A_hi, A_lo, B_hi, B_lo)
//              K-slice into a STAGES-deep shared-memory ring;
//   warp 1     allocates TMEM; one lane issues the MMAs and commits them to
//              the ring's "empty" barriers and to the chunk barriers;
//   warps 2-9  two epilogue warpgroups: the warp's TMEM lane quarter gives its
//              32 rows, its warpgroup one half of the BN columns. They drain
//              each chunk into registers and, after the last chunk of a tile,
//              apply bias / position / GELU / residual, split hi/lo and store.
// Operand tiles are K-major with the TMA swizzle that matches the UMMA
// descriptor (BK*4 bytes: 128B for BK=32, 64B for BK=16).
// With CG = 2 a cluster of two CTAs (tcgen05 cta_group::2) computes one
// 256-row tile; each CTA loads its own A rows and half of the B tile with
// plain (unicast) TMA loads, and only the MMA completion commit signals both
// CTAs.
// Every mbarrier wait is bounded (globaltimer); a wait that gives up sets a
// CTA-wide abort flag and the library's device error word, the roles wind
// down, in-flight copies and MMAs are drained, and TMEM is freed.
#include "gemm.cuh"
#include "numerics.cuh"
#include "tc05.cuh"

#include <cuda_fp16.h>

namespace tcg {
namespace {

constexpr int BM = 128;
// Instruction descriptor of kind::tf32, fp32 accumulator, both operands
// K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_tf32()
{
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ float epi_value(const GemmEpi &e, float x, int src_row, int n)
{
    if (e.bias) x = __fadd_rn(x, e.bias[n]);
    if (e.rowadd) x = __fadd_rn(x, e.rowadd[(size_t)src_row * e.ld_rowadd + n]);
    if (e.act == 1) x = gelu_exact(x);
    else if (e.act == 2) x = gelu_quick(x);
    return x;
}

// Finish and store columns n .. n+3 of GEMM row r (cnt of them in range).
__device__ __forceinline__ void epi_store4(const GemmEpi &e, int src_row, size_t dst_row, int n, int cnt,
                                           float v0, float v1, float v2, float v3)
{
    float v[4] = { v0, v1, v2, v3 };
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (j < cnt) v[j] = epi_value(e, v[j], src_row, n + j);
    const size_t o = dst_row * (size_t)e.out.ld + n;
    const bool vec = cnt == 4 && ((e.out.ld | n) & 3) == 0;
    if (e.residual) {
        const float *res = e.residual + o;
        if (vec && !((uintptr_t)res & 15)) {
            const float4 q = *reinterpret_cast<const float4 *>(res);
            v[0] = __fadd_rn(q.x, v[0]); v[1] = __fadd_rn(q.y, v[1]);
            v[2] = __fadd_rn(q.z, v[2]); v[3] = __fadd_rn(q.w, v[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (j < cnt) v[j] = __fadd_rn(res[j], v[j]);
        }
    }
    if (e.out.plain) {
        float *d = e.out.plain + o;
        if (vec && !((uintptr_t)d & 15)) *reinterpret_cast<float4 *>(d) = make_float4(v[0], v[1], v[2], v[3]);
        else
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (j < cnt) d[j] = v[j];
    }
    if (e.out.hi) {
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) split_tf32(v[j], h[j], l[j]);
        float *dh = e.out.hi + o, *dl = e.out.lo + o;
        if (vec && !(((uintptr_t)dh | (uintptr_t)dl) & 15)) {
            *reinterpret_cast<float4 *>(dh) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4 *>(dl) = make_float4(l[0], l[1], l[2], l[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (j < cnt) { dh[j] = h[j]; dl[j] = l[j]; }
        }
    }
}

// ---------------------------------------------- CTA pairs (cta_group::2)
// With CG = 2 a cluster of two CTAs computes one 256 x BN tile: CTA r owns
// rows 128r..128r+127 and loads its 128 rows of A and half of B (BN/2 rows);
// the MMA reads A from each CTA and B from both halves, so each SM's shared
// memory serves 25% fewer operand bytes per FLOP than with one CTA per tile.
// The leader's producer arms the stage barrier with both CTAs' bytes, both
// CTAs' (unicast) TMA loads complete on it, and one lane of the leader issues
// the M = 256 MMAs and commits them to the barrier at the same offset in both
// CTAs. Each CTA drains its own 128 TMEM lanes and releases chunk buffers on
// the leader's barriers.

__device__ __forceinline__ uint32_t cta_rank_in_cluster()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void bar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory whose bytes complete on the
// leader's barrier (cluster address).
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t d, unsigned long long a, unsigned long long b, uint32_t id, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc));
}
// commit the leader's MMAs to the barrier at this offset in both CTAs
__device__ __forceinline__ void mma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(bar), "h"((unsigned short)3) : "memory");
}
// commit the leader's MMAs to one of its own barriers
__device__ __forceinline__ void mma_commit_pair_local(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// EPI_W epilogue warps (8 or 16): warp w drains TMEM lane quarter w & 3 and
// column group (w - 2) / 4 of the tile. ACC, where the three products of a
// K-step accumulate:
//   ACC_SEP   the small lo*hi + hi*lo terms in their own per-tile TMEM
//             buffers (two chunk and two tile accumulators of BN columns): one
//             truncating tensor-core add per K-step into a chunk, the most
//             accurate;
//   ACC_FOLD  all three into the chunk buffer, as many BN-column chunk buffers
//             as the 512 TMEM columns hold (three truncating adds per K-step);
//   ACC_WIDE  one N = 2*BN MMA of A_hi against B_hi and B_lo stacked (they are
//             adjacent in shared memory) puts hi*hi and hi*lo side by side in
//             a 2*BN-column chunk buffer, and one N = BN MMA adds lo*hi to the
//             first half: two MMA instructions per K-step instead of three,
//             each twice as long on average, and two truncating adds into
//             the hi*hi half. The drain adds the halves.
enum { ACC_SEP = 0, ACC_FOLD = 1, ACC_WIDE = 2 };

// OPF 1: the operands are fp16 pieces (2 bytes per element, BK = 64 fills a
// 128-byte swizzled row, BK = 32 a 64-byte one) for kind::f16 MMAs, scaled
// per 128- or 256-element K-block.
template <int BN, int BK, int STAGES, int EPI_W = 8, int ACC = ACC_SEP, int CG = 1, int QB = 0, int OPF = 0>
struct Shape {
    static constexpr int ES = OPF ? 2 : 4;                      // bytes per operand element
    static constexpr uint32_t A_BYTES = BM * BK * ES;
    static constexpr uint32_t B_BYTES = (BN / CG) * BK * ES;    // this CTA's share of the B tile
    static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int CW = ACC == ACC_WIDE ? 2 * BN : BN;    // columns of a chunk buffer
    static constexpr int NBUF = ACC == ACC_SEP ? 2 : (4 * CW <= 512 ? 4 : 2);   // chunk buffers
    static constexpr int NACC = ACC == ACC_SEP ? 4 : NBUF;
    static constexpr uint32_t TMEM_COLS = NACC * CW <= 256 ? 256 : 512;
    static constexpr int GROUPS = EPI_W / 4;
    static constexpr int HALF = BN / GROUPS;           // columns per epilogue thread
    static constexpr int THREADS = 64 + 32 * EPI_W + (QB ? 64 : 0);    // + two converter warps
    static constexpr int LDW = EPI_W > 8 ? 16 : 64;    // widest TMEM load of the drain
    static constexpr uint32_t EPI_STAGE_BYTES = 32 * 16 * 4;   // per epilogue warp: 32 rows x 16 columns
    static constexpr int NBAR = 2 * STAGES + 2 * NBUF + 4 + 1;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + EPI_W * EPI_STAGE_BYTES + 8 * NBAR + 16;
    static_assert(EPI_W == 8 || EPI_W == 16, "two or four epilogue warps per TMEM lane quarter");
    static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair per tile");
    static_assert(HALF % 16 == 0, "each epilogue warp drains whole 16-column slices");
    static_assert(NACC * CW <= 512, "the accumulators must fit the 512 TMEM columns");
    static_assert(ACC != ACC_WIDE || (2 * BN <= 256 && CG == 1), "a wide MMA is at most 256 columns, one CTA");
    static_assert(SMEM <= 232448, "shared memory per block");
    static_assert(QB == 0 || (BN == 128 && BK == 32 && CG == 1), "packed B: 128 rows x one 32-weight sub-block");
    static_assert(OPF == 0 || (QB == 0 && ((ACC == ACC_WIDE && (BK == 64 || BK == 32)) ||
                                           (ACC == ACC_FOLD && BK == 64))),
                  "fp16 pieces: the wide shape (BK = 64 or 32), or the three products folded (BK = 64)");
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const float (&v)[4])
{
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
                 : "memory");
}

// acc[0..HALF) += (first + second) where first and second are the HALF fp32
// columns at TMEM addresses ta and tb (this warp's lanes), 16 at a time.
template <int HALF>
__device__ __forceinline__ void drain_add2(uint32_t ta, uint32_t tb, float (&acc)[HALF])
{
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        uint32_t x[8], y[8];
        tmem_ld8(ta + (uint32_t)j, x);
        tmem_ld8(tb + (uint32_t)j, y);
#pragma unroll
        for (int i = 0; i < 8; i++)
            acc[j + i] = __fadd_rn(acc[j + i], __fadd_rn(__uint_as_float(x[i]), __uint_as_float(y[i])));
    }
}

// drain_add2 for fp16-piece operands: (first + second) times fa = 2^-ea,
// the row's K-block scale undone (exactly: a power of two), added to acc.
// The column scales are undone once per tile (scale_cols).
template <int HALF>
__device__ __forceinline__ void drain_add2_scaled(uint32_t ta, uint32_t tb, float (&acc)[HALF], float fa)
{
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        uint32_t x[8], y[8];
        tmem_ld8(ta + (uint32_t)j, x);
        tmem_ld8(tb + (uint32_t)j, y);
#pragma unroll
        for (int i = 0; i < 8; i++)
            acc[j + i] = fmaf(__fadd_rn(__uint_as_float(x[i]), __uint_as_float(y[i])), fa, acc[j + i]);
    }
}

// drain_add for fp16-piece operands with one chunk buffer: the HALF columns
// at taddr times fa = 2^-ea (the row's K-block scale undone) added to acc.
template <int HALF>
__device__ __forceinline__ void drain_add_scaled(uint32_t taddr, float (&acc)[HALF], float fa)
{
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        uint32_t x[8];
        tmem_ld8(taddr + (uint32_t)j, x);
#pragma unroll
        for (int i = 0; i < 8; i++) acc[j + i] = fmaf(__uint_as_float(x[i]), fa, acc[j + i]);
    }
}

// acc[j] *= 2^-xb[n0 + j]: B row (output column) n was scaled by 2^xb[n] over
// all of K. |xb| <= 63 and the row factors are at most 2^63, so the partial
// sums stay finite and both multiplications are exact.
// (ea: the row's exponent when A is scaled per row, else 0)
template <int HALF>
__device__ __forceinline__ void scale_cols(float (&acc)[HALF], const int8_t *xb, int n0, int N, int ea)
{
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        uint2 e8 = make_uint2(0u, 0u);
        if (n0 + j + 8 <= N) e8 = *reinterpret_cast<const uint2 *>(xb + n0 + j);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int eb = (int)(int8_t)(((i < 4 ? e8.x : e8.y) >> (8 * (i & 3))) & 0xFFu);
            acc[j + i] = __fmul_rn(acc[j + i], __int_as_float((127 - ea - eb) << 23));
        }
    }
}

// scale_cols with the column exponents already in registers (8 per uint2,
// zero past N)
template <int HALF>
__device__ __forceinline__ void scale_cols_r(float (&acc)[HALF], const uint2 (&xbr)[HALF / 8], int ea)
{
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        const uint2 e8 = xbr[j / 8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int eb = (int)(int8_t)(((i < 4 ? e8.x : e8.y) >> (8 * (i & 3))) & 0xFFu);
            acc[j + i] = __fmul_rn(acc[j + i], __int_as_float((127 - ea - eb) << 23));
        }
    }
}

// fp16-piece output of this lane's row, columns n0 .. n0 + HALF - 1: bias and
// activation as epi_value, then the row's power-of-two scale from the bound
// rnorm[m] * bounds[0] + bounds[1] (with 1/256 to spare for rounding), then
// the two pieces; the exponent is written by the lanes of column 0.
template <int HALF>
__device__ __forceinline__ void epi_store_f16(const GemmEpi &e, const float (&acc)[HALF], int m, int n0, int M, int N)
{
    if (m >= M) return;
    const float bound = __fmul_rn(fmaf(e.rnorm[m], e.bounds[0], e.bounds[1]), 1.00390625f);
    const int ex = f16_scale_exp(bound);
    const float f = __int_as_float((127 + ex) << 23);
    __half *fh = (__half *)e.out.fh, *fl = (__half *)e.out.fl;
#pragma unroll
    for (int j = 0; j < HALF; j += 8) {
        if (n0 + j >= N) break;
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            a[i] = epi_value(e, acc[j + i], m, n0 + j + i);
            b[i] = epi_value(e, acc[j + 4 + i], m, n0 + j + 4 + i);
        }
        uint2 ha, la, hb, lb;
        f16_pieces4(a, f, ha, la);
        f16_pieces4(b, f, hb, lb);
        const size_t at = (size_t)m * e.out.ld + n0 + j;
        *reinterpret_cast<uint4 *>(fh + at) = make_uint4(ha.x, ha.y, hb.x, hb.y);
        *reinterpret_cast<uint4 *>(fl + at) = make_uint4(la.x, la.y, lb.x, lb.y);
    }
    if (n0 == 0) e.out.fe[m] = (int8_t)ex;
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// Stores this warp's 32 tile rows x HALF columns (acc: lane = row) through a
// 32 x 16 shared-memory slice, so that the global stores and the bias,
// position and residual loads are row-contiguous (four lanes per 16 columns
// of a row) instead of one row per lane. The slice's float4 chunks are
// XOR-swizzled by (row >> 1) & 3, which keeps both the row-wise writes and the
// column-wise reads free of bank conflicts. Every load of a slice is issued
// before its first store (the residual may be the output itself, so the
// compiler could not reorder them).
template <int HALF>
__device__ __forceinline__ void epi_store_tile(const GemmEpi &e, const float (&acc)[HALF], float *stage, int row0,
                                               int n0, int M, int N)
{
    constexpr int NS = HALF / 16;
    const int lane = threadIdx.x & 31;
    const int c = lane & 3;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < NS; s++) {
        // row indices are recomputed per slice: holding them across slices
        // costs registers that the accumulators need
        int src_row[4];
        size_t dst_row[4];
        bool row_ok[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = row0 + i * 8 + (lane >> 2);
            row_ok[i] = r < M;
            src_row[i] = r % e.rgroup + e.roff;
            dst_row[i] = (size_t)(r / e.rgroup) * e.rstride + e.roff + r % e.rgroup;
        }
        const int j = 16 * s;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int pc = k ^ ((lane >> 1) & 3);
            *reinterpret_cast<float4 *>(stage + lane * 16 + pc * 4) =
                make_float4(acc[j + 4 * k], acc[j + 4 * k + 1], acc[j + 4 * k + 2], acc[j + 4 * k + 3]);
        }
        __syncwarp();
        float4 v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int rr = i * 8 + (lane >> 2);
            v[i] = *reinterpret_cast<const float4 *>(stage + rr * 16 + (c ^ ((rr >> 1) & 3)) * 4);
        }
        __syncwarp();
        const int n = n0 + j + 4 * c;
        if (n >= N) continue;
        if (!e.vec) {
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (row_ok[i]) epi_store4(e, src_row[i], dst_row[i], n, min(4, N - n), v[i].x, v[i].y, v[i].z, v[i].w);
            continue;
        }
        // the one extra operand of a row: its residual, or else its position row
        const float4 b4 = e.bias ? ld4(e.bias + n) : zero;
        float4 ex[4];
#pragma unroll
        for (int i = 0; i < 4; i++)
            ex[i] = !row_ok[i] ? zero
                  : e.residual ? ld4(e.residual + dst_row[i] * (size_t)e.out.ld + n)
                  : e.rowadd   ? ld4(e.rowadd + (size_t)src_row[i] * e.ld_rowadd + n) : zero;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (!row_ok[i]) continue;
            float x[4] = { v[i].x, v[i].y, v[i].z, v[i].w };
            const float bb[4] = { b4.x, b4.y, b4.z, b4.w };
            const float xx[4] = { ex[i].x, ex[i].y, ex[i].z, ex[i].w };
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (e.bias) x[k] = __fadd_rn(x[k], bb[k]);
                if (e.rowadd) x[k] = __fadd_rn(x[k], xx[k]);
                if (e.act == 1) x[k] = gelu_exact(x[k]);
                else if (e.act == 2) x[k] = gelu_quick(x[k]);
                if (e.residual) x[k] = __fadd_rn(xx[k], x[k]);
            }
            const size_t o = dst_row[i] * (size_t)e.out.ld + n;
            if (e.out.plain) *reinterpret_cast<float4 *>(e.out.plain + o) = make_float4(x[0], x[1], x[2], x[3]);
            if (e.out.hi) {
                float h[4], l[4];
#pragma unroll
                for (int k = 0; k < 4; k++) split_tf32(x[k], h[k], l[k]);
                *reinterpret_cast<float4 *>(e.out.hi + o) = make_float4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<float4 *>(e.out.lo + o) = make_float4(l[0], l[1], l[2], l[3]);
            }
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// One bulk tensor store of a shared-memory box to (x, y) of map, as its own
// bulk group.
__device__ __forceinline__ void tma_store(const CUtensorMap *map, uint32_t src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 ::"l"((unsigned long long)map), "r"(x), "r"(y), "r"(src) : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most PENDING of this thread's bulk groups still read shared memory.
template <int PENDING>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(PENDING) : "memory");
}

// The epilogue of a tile whose rows map one to one onto output rows (no
// rowadd): lane = row, as the accumulators come out of TMEM, so nothing is
// transposed. Units of 8 columns of one output array go through two
// alternating 32 x 8 shared buffers in the 32-byte swizzle (16-byte chunk c of
// row r at c ^ ((r >> 2) & 1): conflict-free for row-per-lane float4 writes),
// each sent by one bulk tensor store that clips rows >= M and columns >= N.
// The bias comes from one register per 32 columns (breg, loaded when the
// tile started) by shuffles; the lane's residual row segment of the next unit
// is loaded while the current unit is finished.
template <int HALF>
__device__ __forceinline__ void epi_store_tile_tma(const GemmEpi &e, const float (&acc)[HALF], float *stage,
                                                   const CUtensorMap *mp, const CUtensorMap *mh,
                                                   const CUtensorMap *ml, int row0, int n0, int M, int N,
                                                   const float (&breg)[(HALF + 31) / 32])
{
    constexpr int NU = HALF / 8;
    static_assert(HALF % 8 == 0, "8-column store units");
    if (row0 >= M) return;                         // all 32 rows below the matrix: nothing to store
    const int lane = threadIdx.x & 31;
    const int r = row0 + lane;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const float *res = e.residual && r < M ? e.residual + (size_t)(e.roff + r) * e.out.ld + n0 : nullptr;
    float4 rc0 = zero, rc1 = zero;
    if (res) {
        if (n0 < N) rc0 = ld4(res);
        if (n0 + 4 < N) rc1 = ld4(res + 4);
    }
    const int sw = (lane >> 2) & 1;
    int buf = 0;
#pragma unroll
    for (int u = 0; u < NU; u++) {
        const int n = n0 + 8 * u;
        if (n >= N) break;
        float4 rn0 = zero, rn1 = zero;
        if (res && u + 1 < NU) {
            if (n + 8 < N) rn0 = ld4(res + 8 * (u + 1));
            if (n + 12 < N) rn1 = ld4(res + 8 * (u + 1) + 4);
        }
        const float rv[8] = { rc0.x, rc0.y, rc0.z, rc0.w, rc1.x, rc1.y, rc1.z, rc1.w };
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = 8 * u + j;
            float v = acc[c];
            if (e.bias) v = __fadd_rn(v, __shfl_sync(0xffffffffu, breg[c / 32], c % 32));
            if (e.act == 1) v = gelu_exact(v);
            else if (e.act == 2) v = gelu_quick(v);
            if (e.residual) v = __fadd_rn(rv[j], v);
            x[j] = v;
        }
#pragma unroll
        for (int o = 0; o < 3; o++) {
            const CUtensorMap *m = o == 0 ? (e.out.plain ? mp : nullptr) : o == 1 ? (e.out.hi ? mh : nullptr)
                                                                                  : (e.out.lo ? ml : nullptr);
            if (!m) continue;
            float y[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (o == 0) {
                    y[j] = x[j];
                } else {
                    float h, l;
                    split_tf32(x[j], h, l);
                    y[j] = o == 1 ? h : l;
                }
            }
            if (lane == 0) bulk_wait_read<1>();     // the store that used this buffer last has read it
            __syncwarp();
            float *b = stage + buf * 256;
            *reinterpret_cast<float4 *>(b + lane * 8 + 4 * sw) = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4 *>(b + lane * 8 + 4 * (sw ^ 1)) = make_float4(y[4], y[5], y[6], y[7]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tma_store(m, su32(b), n, row0);
            buf ^= 1;
        }
        rc0 = rn0;
        rc1 = rn1;
    }
}

// epi_store_f16 through bulk tensor stores: 16-column units (32 bytes of
// each of the warp's 32 rows, the fp32 path's 8-column geometry) of the hi
// pieces, then of the lo pieces, staged in the warp's two 32 x 32-byte
// buffers (32-byte swizzle) and stored by fp16 output maps.
template <int HALF>
__device__ __forceinline__ void epi_store_f16_tma(const GemmEpi &e, const float (&acc)[HALF], float *stage,
                                                  const CUtensorMap *mh, const CUtensorMap *ml, int row0, int n0,
                                                  int M, int N, const float (&breg)[(HALF + 31) / 32])
{
    static_assert(HALF % 16 == 0, "16-column store units");
    if (row0 >= M) return;
    const int lane = threadIdx.x & 31;
    const int r = row0 + lane;
    const float bound = r < M ? __fmul_rn(fmaf(e.rnorm[r], e.bounds[0], e.bounds[1]), 1.00390625f) : 0.0f;
    const int ex = f16_scale_exp(bound);
    const float f = __int_as_float((127 + ex) << 23);
    const int sw = (lane >> 2) & 1;
    int buf = 0;
#pragma unroll
    for (int u = 0; u < HALF / 16; u++) {
        const int n = n0 + 16 * u;
        if (n >= N) break;
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int c = 16 * u + j;
            float v = acc[c];
            if (e.bias) v = __fadd_rn(v, __shfl_sync(0xffffffffu, breg[c / 32], c % 32));
            if (e.act == 1) v = gelu_exact(v);
            else if (e.act == 2) v = gelu_quick(v);
            x[j] = v;
        }
        uint2 h[4], l[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float v4[4] = { x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3] };
            f16_pieces4(v4, f, h[q], l[q]);
        }
#pragma unroll
        for (int o = 0; o < 2; o++) {
            const uint2 *y = o == 0 ? h : l;
            if (lane == 0) bulk_wait_read<1>();     // the store that used this buffer last has read it
            __syncwarp();
            float *b = stage + buf * 256;
            *reinterpret_cast<uint4 *>(b + lane * 8 + 4 * sw) = make_uint4(y[0].x, y[0].y, y[1].x, y[1].y);
            *reinterpret_cast<uint4 *>(b + lane * 8 + 4 * (sw ^ 1)) = make_uint4(y[2].x, y[2].y, y[3].x, y[3].y);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tma_store(o == 0 ? mh : ml, su32(b), n, row0);
            buf ^= 1;
        }
    }
    if (n0 == 0 && r < M) e.out.fe[r] = (int8_t)ex;
}

// acc[0..HALF) += the HALF fp32 columns at TMEM address taddr (this warp's
// lanes), in loads of at most LDW columns.
template <int HALF, int LDW = 64>
__device__ __forceinline__ void drain_add(uint32_t taddr, float (&acc)[HALF])
{
    constexpr int W64 = LDW >= 64 ? HALF / 64 * 64 : 0;
#pragma unroll
    for (int j = 0; j < W64; j += 64) {
        uint32_t r[64];
        tmem_ld64(taddr + (uint32_t)j, r);
#pragma unroll
        for (int i = 0; i < 64; i++) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
    }
    constexpr int W32 = W64 + (HALF - W64) / 32 * 32;
#pragma unroll
    for (int j = W64; j < W32; j += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + (uint32_t)j, r);
#pragma unroll
        for (int i = 0; i < 32; i++) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
    }
#pragma unroll
    for (int j = W32; j < HALF; j += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)j, r);
#pragma unroll
        for (int i = 0; i < 16; i++) acc[j + i] = __fadd_rn(acc[j + i], __uint_as_float(r[i]));
    }
}

// Work order of one CTA (or CTA pair) p of a persistent GEMM launch of P
// CTAs (pairs). Whole tiles: p, p + P, p + 2P, ... With stream-K (sk), only the
// R = num_tiles / P full waves run that way; the L = num_tiles % P tiles of the
// last wave become L * C chunk units (C = K chunks per tile) dealt out in
// contiguous, equal ranges [first(p), first(p + 1)), so no SM idles through a
// partial wave. A tile cut by a range boundary is finished by its owner, the
// CTA holding its chunk 0: the later CTAs (contributors) hand their partial
// sums over through global memory. A contributor segment is always the first
// of its CTA's stream-K range and never waits; an owner segment is always the
// last, and waits only for contributor segments, so no wait can be circular.
struct Seg {
    int tile, c0, c1;    // chunks [c0, c1) of tile
};

struct Sched {
    int C, P, p, num_tiles, R, i = 0;
    long long u = 0, ue = 0, LC = 0;
    __device__ Sched(int num_tiles_, int C_, bool sk, int P_, int p_) : C(C_), P(P_), p(p_), num_tiles(num_tiles_)
    {
        if (sk) {
            R = num_tiles / P;
            LC = (long long)(num_tiles % P) * C;
            u = first(p);
            ue = first(p + 1);
        } else {
            R = (num_tiles + P - 1) / P;
        }
    }
    __device__ long long first(int q) const { return LC * q / P; }
    __device__ bool next(Seg &s)
    {
        while (i < R) {
            const int t = i++ * P + p;
            if (t < num_tiles) {
                s.tile = t; s.c0 = 0; s.c1 = C;
                return true;
            }
        }
        if (u >= ue) return false;
        s.tile = R * P + (int)(u / C);
        s.c0 = (int)(u % C);
        s.c1 = (int)min((long long)C, s.c0 + (ue - u));
        u += s.c1 - s.c0;
        return true;
    }
};

__device__ __forceinline__ void st_release(int *f, int v)
{
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int *f)
{
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    return v;
}

// Test hook (tcg_test_gemm_withhold_flags): the stream-K flag wait's limit,
// and whether contributors raise their flags at all (1: they never do, so
// every owner's wait runs out, which is how the failure path gets tested
// without a fault).
__device__ unsigned long long g_flag_wait_ns = WAIT_NS;
__device__ int g_flag_withhold = 0;

// Wait (bounded, like bar_wait) until a contributor has raised flag f.
__device__ bool flag_wait(const int *f, volatile int *abort, int *err, int code)
{
    const unsigned long long t0 = now_ns(), limit = g_flag_wait_ns;
    for (uint32_t it = 1;; ++it) {
        if (ld_acquire(f) != 0) return true;
        if ((it & 63) == 0) {
            if (*abort) return false;
            if (now_ns() - t0 > limit) {
                *abort = 1;
                atomicExch(err, code);
                return false;
            }
        }
    }
}

// chunk_kb: K-blocks whose hi*hi products share one TMEM chunk buffer before
// it is drained into the fp32 registers.
template <int BN, int BK, int STAGES, int EPI_W, int ACC, int CG, int QB = 0, int OPF = 0>
__global__ void __launch_bounds__(Shape<BN, BK, STAGES, EPI_W, ACC, CG, QB, OPF>::THREADS, 1)
gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                   const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                   const __grid_constant__ CUtensorMap o_plain, const __grid_constant__ CUtensorMap o_hi,
                   const __grid_constant__ CUtensorMap o_lo,
                   int M, int N, int K, int chunk_kb, GemmEpi epi, int *err, float *ws, int *flags, int sk)
{
    using S = Shape<BN, BK, STAGES, EPI_W, ACC, CG, QB, OPF>;
    constexpr bool SEP = ACC == ACC_SEP, WIDE = ACC == ACC_WIDE;
    constexpr uint32_t CW = S::CW;
    constexpr int SWB = BK * S::ES;
    constexpr int KPM = OPF ? 16 : 8;                            // K elements per MMA instruction
    constexpr uint32_t FMT = OPF ? 0u : 2u;                      // A/B format: f16 or tf32
    extern __shared__ uint8_t smem_raw[];
    uint8_t *tiles = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float *epi_stage = (float *)(tiles + (size_t)STAGES * S::STAGE_BYTES);
    uint64_t *bars = (uint64_t *)(tiles + (size_t)STAGES * S::STAGE_BYTES + EPI_W * S::EPI_STAGE_BYTES);
    uint32_t *tmem_slot = (uint32_t *)(bars + S::NBAR);
    volatile int *abort = (volatile int *)(tmem_slot + 1);

    const uint32_t rank = CG == 2 ? cta_rank_in_cluster() : 0;
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = ((M + CG * BM - 1) / (CG * BM)) * n_tiles;
    const int num_kb = (K + BK - 1) / BK;
    const int n_chunks = (num_kb + chunk_kb - 1) / chunk_kb;
    const bool skm = !SEP && sk && ws && flags;    // stream-K needs per-chunk partials: not ACC_SEP
    const uint32_t full0 = su32(bars), empty0 = su32(bars + STAGES);
    constexpr int NBUF = S::NBUF;
    const uint32_t cfull0 = su32(bars + 2 * STAGES), cempty0 = cfull0 + 8 * NBUF;
    const uint32_t sfull0 = cempty0 + 8 * NBUF, sempty0 = sfull0 + 16, drain = sempty0 + 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            bar_init(full0 + 8 * s, QB ? 3 : 1);     // packed B: the TMA bytes and two converter warps
            bar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < NBUF; b++) {
            bar_init(cfull0 + 8 * b, 1);
            bar_init(cempty0 + 8 * b, CG * EPI_W);        // the epilogue warps of every CTA of the group
        }
        for (int b = 0; b < 2; b++) {
            bar_init(sfull0 + 8 * b, 1);
            bar_init(sempty0 + 8 * b, CG * EPI_W);
        }
        bar_init(drain, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (CG == 2) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(su32(tmem_slot)), "r"(S::TMEM_COLS) : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(su32(tmem_slot)), "r"(S::TMEM_COLS) : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    fence_before();
    if constexpr (CG == 2) cluster_sync();      // barriers initialised and TMEM allocated in both CTAs
    else __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const int P = gridDim.x / CG, p = blockIdx.x / CG;   // tile groups (CTA pairs) and this one
    pdl_wait();                  // no global access above this line

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&a_hi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&a_lo) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&b_hi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&b_lo) : "memory");
            if (epi.tma) {
                asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&o_plain) : "memory");
                asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&o_hi) : "memory");
                asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&o_lo) : "memory");
            }
            int stage = 0;
            uint32_t phase = 0;
            long issued = 0;
            bool ok = true;
            Sched sc(num_tiles, n_chunks, skm, P, p);
            Seg sg;
            while (ok && sc.next(sg)) {
                const int m0 = (sg.tile / n_tiles) * CG * BM + (int)rank * BM;
                const int nb = (sg.tile % n_tiles) * BN + (int)rank * (BN / CG);
                const int kb_end = min(sg.c1 * chunk_kb, num_kb);
                for (int kb = sg.c0 * chunk_kb; kb < kb_end; kb++) {
                    if (!bar_wait(empty0 + 8 * stage, phase ^ 1, abort, err, 1)) { ok = false; break; }
                    const uint32_t base = su32(tiles + (size_t)stage * S::STAGE_BYTES);
                    if constexpr (CG == 2) {
                        // both CTAs' copies complete on the leader's barrier
                        const uint32_t fb = peer_addr(full0 + 8 * stage, 0);
                        if (leader) bar_expect_tx(full0 + 8 * stage, 2 * S::STAGE_BYTES);
                        tma_load_pair(base, &a_hi, fb, kb * BK, m0);
                        tma_load_pair(base + S::A_BYTES, &a_lo, fb, kb * BK, m0);
                        tma_load_pair(base + 2 * S::A_BYTES, &b_hi, fb, kb * BK, nb);
                        tma_load_pair(base + 2 * S::A_BYTES + S::B_BYTES, &b_lo, fb, kb * BK, nb);
                    } else if constexpr (QB != 0) {
                        // the converter warps write this stage's B tiles
                        const uint32_t fb = full0 + 8 * stage;
                        bar_expect_tx(fb, 2 * S::A_BYTES);
                        tma_load(base, &a_hi, fb, kb * BK, m0);
                        tma_load(base + S::A_BYTES, &a_lo, fb, kb * BK, m0);
                    } else {
                        const uint32_t fb = full0 + 8 * stage;
                        bar_expect_tx(fb, S::STAGE_BYTES);
                        tma_load(base, &a_hi, fb, kb * BK, m0);
                        tma_load(base + S::A_BYTES, &a_lo, fb, kb * BK, m0);
                        tma_load(base + 2 * S::A_BYTES, &b_hi, fb, kb * BK, nb);
                        tma_load(base + 2 * S::A_BYTES + S::B_BYTES, &b_lo, fb, kb * BK, nb);
                    }
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
            // Let the last fill of every stage land before the CTA exits (in a
            // pair, the follower's copies complete on the leader's barrier).
            if (leader)
                for (int i = 1; i <= STAGES && i <= issued; i++) {
                    int s = stage - i;
                    uint32_t ph = phase;
                    if (s < 0) { s += STAGES; ph ^= 1; }
                    bar_wait(full0 + 8 * s, ph, abort, err, 2, false);
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (leader && lane == 0) {
            const uint32_t id = (1u << 4) | (FMT << 7) | (FMT << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)((CG * BM) >> 4) << 24);
            const uint32_t id_wide = (1u << 4) | (FMT << 7) | (FMT << 10) | ((uint32_t)((2 * BN) >> 3) << 17) |
                                     ((uint32_t)((CG * BM) >> 4) << 24);
            int stage = 0;
            uint32_t phase = 0, chunk = 0;
            bool ok = true;
            Sched sc(num_tiles, n_chunks, skm, P, p);
            Seg sg;
            for (int local = 0; ok && sc.next(sg); local++) {
                const uint32_t ts = local & 1;
                if (SEP && !bar_wait(sempty0 + 8 * ts, ((local >> 1) & 1) ^ 1, abort, err, 3)) break;
                fence_after();
                for (int c = sg.c0; ok && c < sg.c1; c++, chunk++) {
                    const uint32_t b = chunk % NBUF;
                    if (!bar_wait(cempty0 + 8 * b, ((chunk / NBUF) & 1) ^ 1, abort, err, 3)) { ok = false; break; }
                    fence_after();
                    const uint32_t db = tmem + b * CW;
                    const uint32_t ds = SEP ? tmem + (NBUF + ts) * CW : db;
                    const int kb0 = c * chunk_kb, kb1 = min(kb0 + chunk_kb, num_kb);
                    const int ks0 = SEP ? 0 : kb0;          // first K-block of the small-term accumulator
                    for (int kb = kb0; kb < kb1; kb++) {
                        if (!bar_wait(full0 + 8 * stage, phase, abort, err, 4)) { ok = false; break; }
                        fence_after();
                        const uint32_t base = su32(tiles + (size_t)stage * S::STAGE_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / KPM; k++) {
                            const uint32_t off = (uint32_t)k * 32u;
                            const unsigned long long ah = sdesc<SWB>(base + off);
                            const unsigned long long al = sdesc<SWB>(base + S::A_BYTES + off);
                            const unsigned long long bh = sdesc<SWB>(base + 2 * S::A_BYTES + off);
                            const unsigned long long bl = sdesc<SWB>(base + 2 * S::A_BYTES + S::B_BYTES + off);
                            const uint32_t acc0 = (kb > kb0 || k > 0) ? 1u : 0u;
                            const uint32_t acc1 = (!SEP || kb > ks0 || k > 0) ? 1u : 0u;
                            if constexpr (OPF && CG == 2) {
                                mma_f16_pair(db, ah, bh, id, acc0);       // hi*hi, then the small terms
                                mma_f16_pair(db, al, bh, id, 1u);
                                mma_f16_pair(db, ah, bl, id, 1u);
                            } else if constexpr (OPF && !WIDE) {
                                mma_f16(db, ah, bh, id, acc0);            // hi*hi, then the small terms
                                mma_f16(db, al, bh, id, 1u);
                                mma_f16(db, ah, bl, id, 1u);
                            } else if constexpr (OPF) {
                                mma_f16(db, ah, bh, id_wide, acc0);       // [hi*hi | hi*lo]
                                mma_f16(db, al, bh, id, 1u);              // + lo*hi
                            } else if constexpr (WIDE) {
                                mma_tf32(db, ah, bh, id_wide, acc0);      // [hi*hi | hi*lo]
                                mma_tf32(db, al, bh, id, 1u);             // + lo*hi
                            } else if constexpr (CG == 2) {
                                mma_tf32_pair(db, ah, bh, id, acc0);
                                mma_tf32_pair(ds, al, bh, id, acc1);
                                mma_tf32_pair(ds, ah, bl, id, 1u);
                            } else {
                                mma_tf32(db, ah, bh, id, acc0);
                                mma_tf32(ds, al, bh, id, acc1);
                                mma_tf32(ds, ah, bl, id, 1u);
                            }
                        }
                        if constexpr (CG == 2) mma_commit_pair(empty0 + 8 * stage);
                        else mma_commit(empty0 + 8 * stage);
                        if (++stage == STAGES) { stage = 0; phase ^= 1; }
                    }
                    if (ok) {
                        if constexpr (CG == 2) mma_commit_pair(cfull0 + 8 * b);
                        else mma_commit(cfull0 + 8 * b);
                    }
                }
                if (SEP && ok) {
                    if constexpr (CG == 2) mma_commit_pair(sfull0 + 8 * ts);
                    else mma_commit(sfull0 + 8 * ts);
                }
            }
            // Every MMA issued above has retired once this barrier flips.
            if constexpr (CG == 2) mma_commit_pair_local(drain);
            else mma_commit(drain);
            bar_wait(drain, 0, abort, err, 5, false);
        }
        __syncwarp();
    } else if (QB == 0 || warp < 2 + EPI_W) {
        const int q = warp & 3;                    // TMEM lanes 32q .. 32q+31 = tile rows
        const int h = (warp - 2) >> 2;             // column group of the tile
        const uint32_t lane_cols = ((uint32_t)(q * 32) << 16) + (uint32_t)(h * S::HALF);
        const int ew = warp - 2;                   // epilogue warp index: its stream-K flag and slot part
        const int me = blockIdx.x;                 // this CTA's stream-K slot
        // chunk and tile buffers are released on the leader's barriers
        const uint32_t cempty_r = CG == 2 ? peer_addr(cempty0, 0) : cempty0;
        const uint32_t sempty_r = CG == 2 ? peer_addr(sempty0, 0) : sempty0;
        uint32_t chunk = 0;
        bool ok = true;
        Sched sc(num_tiles, n_chunks, skm, P, p);
        Seg sg;
        for (int local = 0; ok && sc.next(sg); local++) {
            float acc[S::HALF];
#pragma unroll
            for (int j = 0; j < S::HALF; j++) acc[j] = 0.0f;
            // bias of this warp's columns for the bulk-store epilogue, loaded
            // now so that its latency hides behind the tile's MMAs
            float breg[(S::HALF + 31) / 32];
#pragma unroll
            for (int i = 0; i < (S::HALF + 31) / 32; i++) {
                const int cc = 32 * i + lane, nn = (sg.tile % n_tiles) * BN + h * S::HALF + cc;
                breg[i] = epi.tma && epi.bias && cc < S::HALF && nn < N ? epi.bias[nn] : 0.0f;
            }
            // fp16 pieces: this warp's column exponents and the first chunk's
            // row exponent now, each next chunk's during the drain before it,
            // so that no load waits in the drain or the column scaling
            uint2 xbr[OPF ? S::HALF / 8 : 1];
            int ea_next = 0;
            const int mrow = (sg.tile / n_tiles) * CG * BM + (int)rank * BM + q * 32 + lane;
            if constexpr (OPF) {
                const int nx = (sg.tile % n_tiles) * BN + h * S::HALF;
#pragma unroll
                for (int j = 0; j < S::HALF / 8; j++)
                    xbr[j] = nx + 8 * j + 8 <= N ? *reinterpret_cast<const uint2 *>(epi.xb + nx + 8 * j)
                                                 : make_uint2(0u, 0u);
                if (epi.xa_blk && mrow < M) ea_next = (int)epi.xa[(size_t)sg.c0 * M + mrow];
            }
            for (int c = sg.c0; c < sg.c1; c++, chunk++) {
                const uint32_t b = chunk % NBUF;
                const int ea = ea_next;                    // this chunk's row exponent (fp16 pieces)
                if (OPF && epi.xa_blk && c + 1 < sg.c1 && mrow < M) ea_next = (int)epi.xa[(size_t)(c + 1) * M + mrow];
                if (!bar_wait(cfull0 + 8 * b, (chunk / NBUF) & 1, abort, err, 6)) { ok = false; break; }
                fence_after();
                if constexpr (OPF && !WIDE) {
                    if (epi.xa_blk) {
                        // this chunk is one K-block of A: undo the row's scale of the block
                        drain_add_scaled<S::HALF>(tmem + lane_cols + b * CW, acc, __int_as_float((127 - ea) << 23));
                    } else {
                        drain_add<S::HALF, S::LDW>(tmem + lane_cols + b * CW, acc);
                    }
                } else if constexpr (OPF) {
                    if (epi.xa_blk) {
                        // this chunk is one K-block of A: undo the row's scale of the block
                        drain_add2_scaled<S::HALF>(tmem + lane_cols + b * CW, tmem + lane_cols + b * CW + BN, acc,
                                                   __int_as_float((127 - ea) << 23));
                    } else {
                        drain_add2<S::HALF>(tmem + lane_cols + b * CW, tmem + lane_cols + b * CW + BN, acc);
                    }
                } else if constexpr (WIDE) drain_add2<S::HALF>(tmem + lane_cols + b * CW, tmem + lane_cols + b * CW + BN, acc);
                else drain_add<S::HALF, S::LDW>(tmem + lane_cols + b * CW, acc);
                fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 2) bar_arrive_cluster(cempty_r + 8 * b);
                    else bar_arrive(cempty_r + 8 * b);
                }
            }
            if (!ok) break;
            if (SEP) {
                const uint32_t ts = local & 1;
                if (!bar_wait(sfull0 + 8 * ts, (local >> 1) & 1, abort, err, 7)) break;
                fence_after();
                drain_add<S::HALF, S::LDW>(tmem + lane_cols + (NBUF + ts) * CW, acc);
                fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 2) bar_arrive_cluster(sempty_r + 8 * ts);
                    else bar_arrive(sempty_r + 8 * ts);
                }
            }
            if (skm && sg.c0 > 0) {
                // contributor: this warp's 32 x HALF partial sums to its part of
                // the CTA's slot (column-major, so each column is one 128-byte
                // line), then the flag the owner's matching warp waits on
                float *slot = ws + ((size_t)me * EPI_W + ew) * 32 * S::HALF;
#pragma unroll
                for (int j = 0; j < S::HALF; j++) slot[j * 32 + lane] = acc[j];
                __threadfence();
                __syncwarp();
                if (lane == 0 && !g_flag_withhold) st_release(flags + me * EPI_W + ew, 1);
                continue;
            }
            if (skm && sg.c1 < n_chunks) {
                // owner: add the contributors' partial sums in chunk order (the
                // same-rank CTA of each contributing group), then clear their
                // flags for the next launch
                const long long end = (long long)(sg.tile - sc.R * sc.P + 1) * n_chunks;
                for (int qq = p + 1; ok && qq < sc.P && sc.first(qq) < end; qq++) {
                    if (sc.first(qq + 1) == sc.first(qq)) continue;          // a group with no units
                    const int other = qq * CG + (int)rank;
                    int *f = flags + other * EPI_W + ew;
                    if (!flag_wait(f, abort, err, 8)) { ok = false; break; }
                    const float *slot = ws + ((size_t)other * EPI_W + ew) * 32 * S::HALF;
#pragma unroll
                    for (int j = 0; j < S::HALF; j++) acc[j] = __fadd_rn(acc[j], slot[j * 32 + lane]);
                    __syncwarp();
                    if (lane == 0) *f = 0;
                }
                if (!ok) break;
            }
            const int m0 = (sg.tile / n_tiles) * CG * BM + (int)rank * BM, n0 = (sg.tile % n_tiles) * BN;
            if constexpr (OPF) {
                const int m = m0 + q * 32 + lane;
                scale_cols_r<S::HALF>(acc, xbr, epi.xa_blk || m >= M ? 0 : (int)epi.xa[m]);
                if (epi.out.fh) {
                    if (epi.tma)
                        epi_store_f16_tma<S::HALF>(epi, acc, epi_stage + ew * (S::EPI_STAGE_BYTES / 4), &o_hi, &o_lo,
                                                   m0 + q * 32, n0 + h * S::HALF, M, N, breg);
                    else
                        epi_store_f16<S::HALF>(epi, acc, m, n0 + h * S::HALF, M, N);
                    continue;
                }
            }
            if (epi.tma)
                epi_store_tile_tma<S::HALF>(epi, acc, epi_stage + ew * (S::EPI_STAGE_BYTES / 4), &o_plain, &o_hi,
                                            &o_lo, m0 + q * 32, n0 + h * S::HALF, M, N, breg);
            else
                epi_store_tile<S::HALF>(epi, acc, epi_stage + ew * (S::EPI_STAGE_BYTES / 4), m0 + q * 32,
                                        n0 + h * S::HALF, M, N);
        }
        if (lane == 0) bulk_wait_read<0>();          // shared memory stays until the stores have read it
    } else {
        if constexpr (QB != 0) {
            // Converter warps: thread cr owns rows cr and cr + 64 of every
            // stage's B tile. Per K-step (32-weight sub-block j of superblock
            // kb / 8) it dequantises them with the dequant seam's rounding
            // sequence, (d*sc)*q - (dmin*m), splits each weight into its tf32
            // pair and writes both tiles in the 128-byte swizzle a TMA load
            // would have produced; then makes the writes visible to the
            // tensor cores and arrives on the stage's barrier. The 48 bytes a
            // row needs per K-step (the superblock header and the 32 quant
            // bytes of the sub-block's pair) are loaded one K-step ahead.
            const int cr = (warp - 2 - EPI_W) * 32 + lane;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            Sched sc(num_tiles, n_chunks, skm, P, p);
            Seg sg;
            while (ok && sc.next(sg)) {
                const uint8_t *rowp[2];
                bool live[2];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int n = (sg.tile % n_tiles) * BN + cr + 64 * h;
                    live[h] = n < N;
                    rowp[h] = epi.bq + (size_t)(live[h] ? n : 0) * epi.bq_row;
                }
                const int kb0 = sg.c0 * chunk_kb, kb_end = min(sg.c1 * chunk_kb, num_kb);
                // [row][0]: header, [1], [2]: the 32 quant bytes
                uint4 cur[2][3], nxt[2][3];
                auto fetch = [&](uint4 (&dst)[2][3], int kb) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint4 *sb = reinterpret_cast<const uint4 *>(rowp[h] + (size_t)(kb >> 3) * 144);
                        const int cc = (kb & 7) >> 1;
                        dst[h][0] = __ldg(sb);
                        dst[h][1] = __ldg(sb + 1 + 2 * cc);
                        dst[h][2] = __ldg(sb + 2 + 2 * cc);
                    }
                };
                fetch(nxt, kb0);
                for (int kb = kb0; kb < kb_end; kb++) {
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int i = 0; i < 3; i++) cur[h][i] = nxt[h][i];
                    if (kb + 1 < kb_end) fetch(nxt, kb + 1);
                    if (!bar_wait(empty0 + 8 * stage, phase ^ 1, abort, err, 9)) { ok = false; break; }
                    const int j = kb & 7, jj = 8 * (j & 3), sh = (j & 1) * 4;
                    const uint32_t base = su32(tiles + (size_t)stage * S::STAGE_BYTES) + 2 * S::A_BYTES;
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint4 hd = cur[h][0];
                        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
                        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
                        const uint32_t b0 = (hd.y >> jj) & 0xFFu, b4 = (hd.z >> jj) & 0xFFu, b8 = (hd.w >> jj) & 0xFFu;
                        const uint32_t scq = j < 4 ? (b0 & 63u) : ((b8 & 15u) | ((b0 >> 6) << 4));
                        const uint32_t mnq = j < 4 ? (b4 & 63u) : ((b8 >> 4) | ((b4 >> 6) << 4));
                        const float a = __fmul_rn(d, (float)scq), c = __fmul_rn(dmin, (float)mnq);
                        const uint32_t qw[8] = { cur[h][1].x, cur[h][1].y, cur[h][1].z, cur[h][1].w,
                                                 cur[h][2].x, cur[h][2].y, cur[h][2].z, cur[h][2].w };
                        const int r = cr + 64 * h;
                        const uint32_t rb = base + (uint32_t)r * 128u;
#pragma unroll
                        for (int c16 = 0; c16 < 8; c16++) {
                            float hv[4], lv[4];
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const uint32_t qv = (qw[c16] >> (8 * e + sh)) & 15u;
                                const float w = live[h] ? __fsub_rn(__fmul_rn(a, __uint_as_float(0x4B000000u | qv) - 8388608.0f), c)
                                                        : 0.0f;
                                split_tf32(w, hv[e], lv[e]);
                            }
                            const uint32_t off = (uint32_t)((c16 ^ (r & 7)) << 4);
                            st_shared_v4(rb + off, hv);
                            st_shared_v4(rb + S::B_BYTES + off, lv);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) bar_arrive(full0 + 8 * stage);
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    }

    fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();      // the leader's MMAs into this CTA's TMEM are done
    if (warp == 1) {
        fence_after();
        if constexpr (CG == 2)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ host

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
        else
            cudaGetLastError();
    }
    return fn;
}

// [rows, K] fp32, row stride K, box = BK x box_rows, swizzle = BK*4 bytes.
bool encode_kmajor(CUtensorMap *m, const float *ptr, int rows, int K, int box_rows, int BK)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
    if (((uintptr_t)ptr & 15) || (K & 3)) return fail("GEMM operand not 16-byte aligned / K=%d not a multiple of 4", K);
    cuuint64_t dims[2] = { (cuuint64_t)K, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)K * 4u };
    cuuint32_t box[2] = { (cuuint32_t)BK, (cuuint32_t)box_rows };
    cuuint32_t estr[2] = { 1, 1 };
    const CUtensorMapSwizzle swz = BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : (BK == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (%d) for [%d x %d]", (int)r, rows, K);
    return true;
}

// fp16-piece operand: rows x K fp16, K-major, boxes of box_k elements (64:
// one 128-byte swizzled row; 32: one 64-byte swizzled row) x box_rows.
bool encode_kmajor_f16(CUtensorMap *m, const void *ptr, int rows, int K, int box_rows, int box_k)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
    if (((uintptr_t)ptr & 15) || (K & 7)) return fail("fp16 GEMM operand not 16-byte aligned / K=%d not a multiple of 8", K);
    cuuint64_t dims[2] = { (cuuint64_t)K, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)K * 2u };
    cuuint32_t box[2] = { (cuuint32_t)box_k, (cuuint32_t)box_rows };
    cuuint32_t estr[2] = { 1, 1 };
    const CUtensorMapSwizzle swz = box_k == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (%d) for fp16 [%d x %d]", (int)r, rows, K);
    return true;
}

// fp16-piece output map: rows x cols fp16, row stride ld elements, boxes of
// 32 rows x 16 columns (32 bytes) in the 32-byte swizzle.
bool encode_out_f16(CUtensorMap *m, const void *ptr, int rows, int cols, int ld)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)ld * 2u };
    cuuint32_t box[2] = { 16, 32 };
    cuuint32_t estr[2] = { 1, 1 };
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Output map for the bulk-store epilogue: rows x cols fp32 with row stride
// ld, boxes of 32 rows x 8 columns in the 32-byte swizzle.
bool encode_out(CUtensorMap *m, const float *ptr, int rows, int cols, int ld)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail("cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    cuuint64_t strides[1] = { (cuuint64_t)ld * 4u };
    cuuint32_t box[2] = { 8, 32 };
    cuuint32_t estr[2] = { 1, 1 };
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)ptr, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct Cfg {
    int bn, bk, stages;
    size_t smem;
    const void *fn;
    int cg;             // CTAs per tile: 2 = a CTA pair (256-row tiles, B boxes of bn/2 rows)
    int threads;
    bool sep;           // separate small-term accumulators (no stream-K)
    int epi_warps;
    int qb;             // B packed in these K-quant blocks (0: tf32 pairs by TMA)
    int opf = 0;        // 1: fp16-piece operands (kind::f16), K-blocks of 128 scaled
};

#define TCG_CFG(BN, BK, ST, EW, ACC, CG)                                                                   \
    { BN, BK, ST, Shape<BN, BK, ST, EW, ACC, CG>::SMEM, (const void *)gemm_tf32x3_kernel<BN, BK, ST, EW, ACC, CG>, \
      CG, Shape<BN, BK, ST, EW, ACC, CG>::THREADS, ACC == ACC_SEP, EW, 0 }
#define TCG_CFG_Q(BN, BK, ST, EW, ACC, QB)                                                                 \
    { BN, BK, ST, Shape<BN, BK, ST, EW, ACC, 1, QB>::SMEM,                                                  \
      (const void *)gemm_tf32x3_kernel<BN, BK, ST, EW, ACC, 1, QB>, 1, Shape<BN, BK, ST, EW, ACC, 1, QB>::THREADS, \
      ACC == ACC_SEP, EW, QB }
#define TCG_CFG_F16P(BN, BK, ST, EW)                                                                        \
    { BN, BK, ST, Shape<BN, BK, ST, EW, ACC_FOLD, 2, 0, 1>::SMEM,                                           \
      (const void *)gemm_tf32x3_kernel<BN, BK, ST, EW, ACC_FOLD, 2, 0, 1>, 2,                               \
      Shape<BN, BK, ST, EW, ACC_FOLD, 2, 0, 1>::THREADS, false, EW, 0, 1 }
#define TCG_CFG_F16F(BN, BK, ST, EW)                                                                        \
    { BN, BK, ST, Shape<BN, BK, ST, EW, ACC_FOLD, 1, 0, 1>::SMEM,                                           \
      (const void *)gemm_tf32x3_kernel<BN, BK, ST, EW, ACC_FOLD, 1, 0, 1>, 1,                               \
      Shape<BN, BK, ST, EW, ACC_FOLD, 1, 0, 1>::THREADS, false, EW, 0, 1 }
#define TCG_CFG_F16(BN, BK, ST, EW)                                                                         \
    { BN, BK, ST, Shape<BN, BK, ST, EW, ACC_WIDE, 1, 0, 1>::SMEM,                                           \
      (const void *)gemm_tf32x3_kernel<BN, BK, ST, EW, ACC_WIDE, 1, 0, 1>, 1,                               \
      Shape<BN, BK, ST, EW, ACC_WIDE, 1, 0, 1>::THREADS, false, EW, 0, 1 }
const Cfg CFGS[] = {
    TCG_CFG(128, 32, 3, 8, ACC_SEP, 1), TCG_CFG(64, 32, 4, 8, ACC_SEP, 1), TCG_CFG(128, 16, 6, 8, ACC_SEP, 1),
    TCG_CFG(64, 16, 8, 8, ACC_SEP, 1), TCG_CFG(96, 32, 3, 8, ACC_SEP, 1), TCG_CFG(96, 16, 7, 8, ACC_SEP, 1),
    TCG_CFG(128, 32, 4, 16, ACC_FOLD, 2),                               // CTA pair, folded
    TCG_CFG(256, 16, 4, 16, ACC_FOLD, 1), TCG_CFG(256, 32, 2, 16, ACC_FOLD, 1),
    TCG_CFG(128, 32, 3, 8, ACC_FOLD, 1), TCG_CFG(128, 32, 3, 16, ACC_SEP, 1), TCG_CFG(128, 32, 3, 16, ACC_FOLD, 1),
    TCG_CFG(128, 32, 4, 16, ACC_SEP, 2),                                // CTA pair, separate small terms
    TCG_CFG(128, 32, 3, 16, ACC_WIDE, 1), TCG_CFG(128, 32, 3, 8, ACC_WIDE, 1),
    TCG_CFG_Q(128, 32, 3, 8, ACC_WIDE, GGML_TYPE_Q4_K),                  // B in Q4_K blocks (15)
    TCG_CFG_F16(128, 64, 3, 16),                                          // fp16 pieces, kind::f16 (16)
    TCG_CFG_F16(128, 32, 6, 16),                                          // the same, six 32-element stages (17)
    TCG_CFG_F16P(256, 64, 3, 16),                                         // fp16 pieces, CTA pair, 256 x 256 (18)
    TCG_CFG_F16P(128, 64, 4, 16),                                         // fp16 pieces, CTA pair, 256 x 128 (19)
    TCG_CFG_F16F(128, 64, 3, 16),                                         // fp16 pieces, products folded (20)
};
#undef TCG_CFG
#undef TCG_CFG_Q
#undef TCG_CFG_F16
#undef TCG_CFG_F16P
#undef TCG_CFG_F16F
constexpr int CFG_Q4K = 15;
constexpr int CFG_F16 = 16;
constexpr int NCFG = sizeof(CFGS) / sizeof(CFGS[0]);

int g_force_cfg = -1;     // tuning hook: a configuration every automatic choice takes

int choose_cfg(int M, int N)
{
    // 128 x 128 tiles with separate small-term accumulators and 16 epilogue
    // warps: the most accurate shape (a few fp32 ulps per product, inside the
    // reference's 1e-5 per-op tolerance) and the fastest of the accurate ones.
    (void)M;
    (void)N;
    if (g_force_cfg >= 0 && g_force_cfg < NCFG) return g_force_cfg;
    return 10;
}

}  // namespace

int gemm_throughput_cfg()
{
    // ACC_WIDE 128 x 128 tiles, 16 epilogue warps: two MMA instructions per
    // K-step (an N = 256 one for hi*hi | hi*lo, an N = 128 one for lo*hi), and
    // stream-K capable. 10-15% faster than the three N = 128 MMAs of the other
    // modes on every ViT GEMM, ~1e-6 of max|C| at K = 3072. BN = 64 or 96
    // tiles, CTA pairs and 128 x 256 tiles measured slower.
    if (g_force_cfg >= 0 && g_force_cfg < NCFG) return g_force_cfg;
    return 13;
}

// K-elements accumulated in TMEM between two drains into fp32 registers.
int g_chunk_k = 256;

// configurations with tf32-pair operands (the packed-B ones need GemmEpi::bq)
int gemm_num_cfgs() { return CFG_Q4K; }

// The configuration of one ViT GEMM: the ACC_WIDE 128 x 128 shape of
// gemm_throughput_cfg(), except where its tiles make exactly one whole wave
// plus a remainder of at most 1/16 of the SMs. There every SM runs one whole
// tile with no successor to overlap its pipeline fill and drain, which
// measured ~100 us per 128 x 128 x 3072 tile against ~63 us per wave when
// several waves follow one another. In that case a long K (at least 6 TMEM
// chunks) takes the 128 x 256 folded shape (7) and a short one the
// separate-accumulator 128 x 128 shape (10). Measured at M = 3200, N = 768
// (the ViT-B/32 shard of 64 images): 94 vs 111 us at K = 3072, 43 vs 49 us at
// K = 768. Both stay within ~1.6e-6 of max|C| of a float64 product.
int gemm_vit_cfg(int M, int N, int K)
{
    const int tp = gemm_throughput_cfg();
    if (g_force_cfg >= 0 && g_force_cfg < NCFG) return tp;
    const int sms = ctx().sms > 0 ? ctx().sms : 148;
    const long tiles = (long)((M + BM - 1) / BM) * ((N + CFGS[tp].bn - 1) / CFGS[tp].bn);
    const long last = tiles - sms;
    if (last <= 0 || last > sms / 16) return tp;
    return (K + g_chunk_k - 1) / g_chunk_k >= 6 ? 7 : 10;
}

int gemm_cfg_bn(int cfg) { return cfg >= 0 && cfg < NCFG ? CFGS[cfg].bn : 0; }

int gemm_q4k_cfg() { return CFG_Q4K; }

// The fp16-piece configuration the ViT and the fp16 entry points plan with
int g_f16_cfg = CFG_F16;
int gemm_f16_cfg() { return g_f16_cfg; }

size_t gemm_work_ws_floats(int ctas) { return (size_t)ctas * BM * 256; }
size_t gemm_work_flag_count(int ctas) { return (size_t)ctas * 16; }

GemmWork *ctx_gemm_work()
{
    Ctx &c = ctx();
    if (c.gemm_work) return (GemmWork *)c.gemm_work;
    const int ctas = c.sms > 0 ? c.sms : 148;
    GemmWork *w = new GemmWork;
    w->ctas = ctas;
    if (cudaMalloc(&w->ws, gemm_work_ws_floats(ctas) * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&w->flags, gemm_work_flag_count(ctas) * sizeof(int)) != cudaSuccess ||
        cudaMemset(w->flags, 0, gemm_work_flag_count(ctas) * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(w->ws);
        cudaFree(w->flags);
        delete w;
        fail("GEMM stream-K workspace: out of memory");
        return nullptr;
    }
    c.gemm_work = w;
    return w;
}

bool gemm_work_reset(const GemmWork &w, cudaStream_t s)
{
    if (!w.flags) return true;
    TCG_CUDA(cudaMemsetAsync(w.flags, 0, gemm_work_flag_count(w.ctas) * sizeof(int), s));
    return true;
}

int g_streamk = 1;        // tuning hook: 0 computes every tile whole
int g_tma_store = 1;      // tuning hook: 0 keeps every epilogue on plain stores
static thread_local int g_last_plan[4];   // grid, stream-K, configuration, bulk-store epilogue of the latest plan

bool gemm_plan(GemmPlan &p, const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
               int M, int N, int K, const GemmEpi &epi, int force_cfg, const GemmWork *work)
{
    if (M <= 0 || N <= 0 || K <= 0) return fail("gemm_plan: empty shape %dx%dx%d", M, N, K);
    const int cfg = force_cfg >= 0 ? force_cfg : choose_cfg(M, N);
    if (cfg >= NCFG) return fail("gemm_plan: no configuration %d", cfg);
    const Cfg &c = CFGS[cfg];
    const int b_rows = c.bn / c.cg;                     // B box: this CTA's share of the tile columns
    if (c.opf) {
        // fp16 pieces and their per-K-block exponents
        if ((epi.xa_blk && K % epi.xa_blk) || N % 8 || !epi.xa || !epi.xb ||
            (epi.xa_blk != 0 && epi.xa_blk != 128 && epi.xa_blk != 256) ||
            (epi.out.fh && (!epi.out.fl || !epi.out.fe || !epi.rnorm || !epi.bounds || epi.out.ld % 8 ||
                            epi.out.plain || epi.out.hi)))
            return fail("gemm_plan: fp16-piece operands need K %% 128 == 0, N %% 8 == 0 and both exponent arrays");
        if (!encode_kmajor_f16(&p.a_hi, a_hi, M, K, BM, c.bk) || !encode_kmajor_f16(&p.a_lo, a_lo, M, K, BM, c.bk) ||
            !encode_kmajor_f16(&p.b_hi, b_hi, N, K, b_rows, c.bk) ||
            !encode_kmajor_f16(&p.b_lo, b_lo, N, K, b_rows, c.bk))
            return false;
    } else if (c.qb) {
        // B comes packed: no B tensor maps (the A ones fill the unused parameters)
        if (!epi.bq || ((uintptr_t)epi.bq & 15) || K % 256 || epi.bq_row != (size_t)(K / 256) * 144)
            return fail("gemm_plan: packed Q4_K B needs 16-byte-aligned rows of K/256 superblocks");
        if (!encode_kmajor(&p.a_hi, a_hi, M, K, BM, c.bk) || !encode_kmajor(&p.a_lo, a_lo, M, K, BM, c.bk))
            return false;
        p.b_hi = p.a_hi;
        p.b_lo = p.a_lo;
    } else if (!encode_kmajor(&p.a_hi, a_hi, M, K, BM, c.bk) || !encode_kmajor(&p.a_lo, a_lo, M, K, BM, c.bk) ||
               !encode_kmajor(&p.b_hi, b_hi, N, K, b_rows, c.bk) || !encode_kmajor(&p.b_lo, b_lo, N, K, b_rows, c.bk)) {
        return false;
    }
    p.M = M;
    p.N = N;
    p.K = K;
    p.cfg = cfg;
    p.epi = epi;
    {
        const auto a16 = [](const void *q) { return ((uintptr_t)q & 15) == 0; };
        p.epi.vec = N % 4 == 0 && epi.out.ld % 4 == 0 && a16(epi.bias) && a16(epi.residual) && a16(epi.out.plain) &&
                    a16(epi.out.hi) && a16(epi.out.lo) && a16(epi.rowadd) && (!epi.rowadd || epi.ld_rowadd % 4 == 0) &&
                    !(epi.rowadd && epi.residual);
        // bulk tensor stores need one output row per GEMM row (no remap)
        p.epi.tma = false;
        if (g_tma_store && epi.out.fh && N % 16 == 0 && epi.out.ld % 8 == 0 && !epi.rowadd && epi.rgroup >= M &&
            epi.roff == 0 && !(((uintptr_t)epi.out.fh | (uintptr_t)epi.out.fl) & 15))
            p.epi.tma = encode_out_f16(&p.o_hi, epi.out.fh, M, N, epi.out.ld) &&
                        encode_out_f16(&p.o_lo, epi.out.fl, M, N, epi.out.ld);
        if (g_tma_store && p.epi.vec && !epi.rowadd && epi.rgroup >= M && epi.roff >= 0 && !epi.out.fh) {
            const size_t off = (size_t)epi.roff * epi.out.ld;
            p.epi.tma = (!epi.out.plain || encode_out(&p.o_plain, epi.out.plain + off, M, N, epi.out.ld)) &&
                        (!epi.out.hi || encode_out(&p.o_hi, epi.out.hi + off, M, N, epi.out.ld)) &&
                        (!epi.out.lo || encode_out(&p.o_lo, epi.out.lo + off, M, N, epi.out.ld));
        }
    }
    const int sms = ctx().sms > 0 ? ctx().sms : 148;
    int groups = sms;        // tile groups resident at once: CTAs, or CTA pairs
    if (c.cg == 2) {
        static int max_clusters[64];
        const int dev = ctx().device & 63;
        if (!max_clusters[dev]) {
            int n = 0;
            cudaLaunchConfig_t lc = {};
            cudaLaunchAttribute at;
            at.id = cudaLaunchAttributeClusterDimension;
            at.val.clusterDim.x = 2; at.val.clusterDim.y = 1; at.val.clusterDim.z = 1;
            lc.gridDim = dim3(2);
            lc.blockDim = dim3(c.threads);
            lc.dynamicSmemBytes = c.smem;
            lc.attrs = &at;
            lc.numAttrs = 1;
            if (cudaFuncSetAttribute(c.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem) != cudaSuccess ||
                cudaOccupancyMaxActiveClusters(&n, c.fn, &lc) != cudaSuccess || n < 1) {
                cudaGetLastError();
                n = sms / 2;
            }
            max_clusters[dev] = n < sms / 2 ? n : sms / 2;
        }
        groups = max_clusters[dev];
    }
    const int tiles = ((M + c.cg * BM - 1) / (c.cg * BM)) * ((N + c.bn - 1) / c.bn);
    p.grid = c.cg * (tiles < groups ? tiles : groups);
    // Stream-K for a partial last wave; the grid then has room for every chunk
    // unit when there is less than one wave of tiles. Worth it when the last
    // wave leaves at least half the SMs idle, or when a tile has many chunks
    // (fine units); with 2-5 chunks and a fuller last wave the partial-sum
    // hand-over costs what it saves.
    const int chunk_k = c.opf && epi.xa_blk ? epi.xa_blk : g_chunk_k;
    const int chunks = (K + chunk_k - 1) / chunk_k;
    const int last = tiles % groups;
    const bool pays = g_streamk == 2 || last <= groups / 2 || chunks >= 6;
    if (g_streamk && work && work->ws && work->flags && !c.sep && last != 0 && chunks > 1 && pays) {
        const long units = (long)tiles * chunks;
        const int g = tiles >= groups ? groups : (int)(units < groups ? units : groups);
        if (c.cg * g <= work->ctas) {
            p.grid = c.cg * g;
            p.sk = 1;
            p.work = *work;
        }
    }
    g_last_plan[0] = p.grid;
    g_last_plan[1] = p.sk;
    g_last_plan[2] = cfg;
    g_last_plan[3] = p.epi.tma ? 1 : 0;
    return true;
}

bool gemm_run(const GemmPlan &p, cudaStream_t s, int *err)
{
    if (p.cfg < 0) return fail("gemm_run: plan not built");
    const Cfg &c = CFGS[p.cfg];
    static unsigned long long attr_done[64];   // per device: bit per configuration
    const int dev = ctx().device & 63;
    if (!(attr_done[dev] >> p.cfg & 1ull)) {
        TCG_CUDA(cudaFuncSetAttribute(c.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem));
        attr_done[dev] |= 1ull << p.cfg;
    }
    // fp16 pieces: one TMEM chunk per K-block of A (its scale)
    int chunk_kb = c.opf && p.epi.xa_blk ? p.epi.xa_blk / c.bk : g_chunk_k / c.bk;
    if (chunk_kb < 1) chunk_kb = 1;
    float *ws = p.work.ws;
    int *flags = p.work.flags;
    int sk = p.sk;
    void *args[] = { (void *)&p.a_hi, (void *)&p.a_lo, (void *)&p.b_hi, (void *)&p.b_lo,
                     (void *)&p.o_plain, (void *)&p.o_hi, (void *)&p.o_lo, (void *)&p.M, (void *)&p.N, (void *)&p.K, (void *)&chunk_kb, (void *)&p.epi, (void *)&err,
                     (void *)&ws, (void *)&flags, (void *)&sk };
    cudaLaunchAttribute at[2];
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(p.grid);
    lc.blockDim = dim3(c.threads);
    lc.dynamicSmemBytes = c.smem;
    lc.stream = s;
    lc.attrs = at;
    lc.numAttrs = pdl_attr(at);
    if (c.cg == 2) {
        cudaLaunchAttribute &cl = at[lc.numAttrs++];
        cl.id = cudaLaunchAttributeClusterDimension;
        cl.val.clusterDim.x = 2; cl.val.clusterDim.y = 1; cl.val.clusterDim.z = 1;
    }
    TCG_CUDA(cudaLaunchKernelExC(&lc, c.fn, args));
    return true;
}

// fp32 rows -> fp16 pieces: one warp per (row, 128-element K-block). The
// block is scaled by 2^e with its largest magnitude in [2^14, 2^15), then v =
// p1 + p2 + r with p1 = v rounded to 11 significant bits (exact in fp16), p2 =
// fp16(v - p1), |r| <= 2^-23 |v|: the precision of a tf32 pair. ex[c * rows +
// row] = e. e is kept in [-63, 63] (0 for an all-zero block) so that a
// product's unscaling 2^-(ea + eb) is one normal float: blocks whose largest
// magnitude lies in [2^-49, 2^77) are represented to that precision; smaller
// ones lose low bits to fp16's subnormals, larger ones overflow fp16.
// mode 0: one exponent per (row, 128-element K-block), ex[c * rows + row];
// mode 2: per (row, 256-element K-block), ex[c * rows + row]; mode 1: one per
// row over all of K (the B operand), ex[row]. A warp takes 128 elements; the
// warps of a 256-element block both compute its maximum.
__global__ void split_f16_kernel(const float *__restrict__ src, int rows, int K, __half *__restrict__ hi,
                                 __half *__restrict__ lo, int8_t *__restrict__ ex, int mode)
{
    const int lane = threadIdx.x & 31;
    const int nkb = K >> 7;
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= (long long)rows * nkb) return;
    const int row = (int)(gw / nkb), c = (int)(gw - (long long)row * nkb);
    const size_t o = (size_t)row * K + (size_t)c * 128 + 4 * lane;
    const float4 v = *reinterpret_cast<const float4 *>(src + o);
    const int per_row = mode == 1;
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    if (mode == 2) {    // the other 128 elements of this 256-element block
        const float4 w = *reinterpret_cast<const float4 *>(src + (o ^ 128));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(w.x), fabsf(w.y)), fmaxf(fabsf(w.z), fabsf(w.w))));
    }
    if (per_row)        // the whole row (a few KB, L1/L2 resident for the row's warps)
        for (int i = lane; i < K / 4; i += 32) {
            const float4 w = *reinterpret_cast<const float4 *>(src + (size_t)row * K + 4 * i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(w.x), fabsf(w.y)), fmaxf(fabsf(w.z), fabsf(w.w))));
        }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
    const int e = f16_scale_exp(m);
    const float f = __int_as_float((127 + e) << 23);
    const float vv[4] = { v.x, v.y, v.z, v.w };
    uint2 h, l;
    f16_pieces4(vv, f, h, l);
    *reinterpret_cast<uint2 *>(hi + o) = h;
    *reinterpret_cast<uint2 *>(lo + o) = l;
    if (lane == 0 && (mode == 0 || (mode == 1 && c == 0) || (mode == 2 && !(c & 1))))
        ex[mode == 1 ? (size_t)row : (size_t)(mode == 2 ? c >> 1 : c) * rows + row] = (int8_t)e;
}

bool launch_split_f16(const float *src, int rows, int K, void *hi, void *lo, int8_t *ex, int mode, cudaStream_t s)
{
    if (rows <= 0) return true;
    if (K % (mode == 2 ? 256 : 128) || ((uintptr_t)src & 15) || ((uintptr_t)hi & 15) || ((uintptr_t)lo & 15))
        return fail("fp16 split: K=%d not a multiple of the block or unaligned buffers", K);
    const long long warps = (long long)rows * (K / 128);
    split_f16_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(src, rows, K, (__half *)hi, (__half *)lo, ex,
                                                                 mode);
    TCG_LAUNCHED();
    return true;
}

}  // namespace tcg

// ------------------------------------------------------------ op-level ABI

using namespace tcg;

static bool linear_impl(float *y, const float *x, const float *W, const float *bias, int M, int N, int K,
                        bool bt, int force_cfg)
{
    if (!need_ctx()) return false;
    if (M < 0 || N < 0 || K < 0) return fail("gemm: negative size");
    if (M == 0 || N == 0) return true;
    cudaStream_t s = ctx().cur;
    const bool tc_ok = bt && K > 0 && (K & 3) == 0 && !((uintptr_t)x & 15) && !((uintptr_t)W & 15);
    if (!tc_ok || force_cfg == -2)
        return launch_gemm_simt(y, N, x, K, W, bt ? K : N, bias, M, N, K, bt, s);
    // tf32 hi/lo copies of both operands, each 16-byte aligned
    const size_t xa = ((size_t)M * K + 3) & ~(size_t)3, wa = ((size_t)N * K + 3) & ~(size_t)3;
    float *buf = (float *)scratch((2 * xa + 2 * wa) * sizeof(float));
    if (!buf) return false;
    float *xh = buf, *xl = xh + xa, *wh = xl + xa, *wl = wh + wa;
    if (!launch_split(x, xh, xl, (size_t)M * K, s) || !launch_split(W, wh, wl, (size_t)N * K, s)) return false;
    GemmEpi e;
    e.bias = bias;
    e.out.plain = y;
    e.out.ld = N;
    GemmPlan p;
    const GemmWork *w = ctx_gemm_work();
    if (!w || !gemm_plan(p, xh, xl, wh, wl, M, N, K, e, force_cfg, w)) return false;
    return gemm_run(p, s, ctx().d_err);
}

extern "C" {

bool tcg_gemm(float *C, const float *A, const float *B, int M, int N, int K, bool b_transposed)
{
    return linear_impl(C, A, B, nullptr, M, N, K, b_transposed, -1);
}

bool tcg_linear(float *y, const float *x, const float *W, const float *bias, int M, int N, int K)
{
    return linear_impl(y, x, W, bias, M, N, K, true, -1);
}

bool tcg_split_tf32(float *hi, float *lo, const float *src, size_t n)
{
    return need_ctx() && launch_split(src, hi, lo, n, ctx().cur);
}

// Test and tuning hook: tcg_linear_split with a forced tile configuration.
bool tcg_linear_split_cfg(float *y, const float *x_hi, const float *x_lo, const float *w_hi, const float *w_lo,
                          const float *bias, int M, int N, int K, int cfg)
{
    if (!need_ctx()) return false;
    if (M < 0 || N < 0 || K <= 0) return fail("tcg_linear_split: bad shape %dx%dx%d", M, N, K);
    if (M == 0 || N == 0) return true;
    GemmEpi e;
    e.bias = bias;
    e.out.plain = y;
    e.out.ld = N;
    GemmPlan p;
    const GemmWork *w = ctx_gemm_work();
    if (!w || !gemm_plan(p, x_hi, x_lo, w_hi, w_lo, M, N, K, e, cfg, w)) return false;
    return gemm_run(p, ctx().cur, ctx().d_err);
}

bool tcg_linear_split(float *y, const float *x_hi, const float *x_lo, const float *w_hi, const float *w_lo,
                      const float *bias, int M, int N, int K)
{
    return tcg_linear_split_cfg(y, x_hi, x_lo, w_hi, w_lo, bias, M, N, K, -1);
}

// Test hook: force a GEMM configuration (cfg >= 0 a tcgen05 tile shape, -2
// the CUDA-core kernel). Not part of the public header.
bool tcg_linear_cfg(float *y, const float *x, const float *W, const float *bias, int M, int N, int K, int cfg)
{
    return linear_impl(y, x, W, bias, M, N, K, true, cfg);
}

int tcg_gemm_num_cfgs(void) { return gemm_num_cfgs(); }

// fp32 rows to fp16 pieces (split_f16_kernel): hi, lo [rows, K] fp16; ex
// int8 exponents, [K / 128, rows] per (row, 128-element K-block) (mode 0),
// [K / 256, rows] per 256-element block (mode 2), or [rows], one per row over
// all of K (mode 1: the B operand).
bool tcg_split_f16(void *hi, void *lo, int8_t *ex, const float *src, int rows, int K, int mode)
{
    if (!need_ctx()) return false;
    return launch_split_f16(src, rows, K, hi, lo, ex, mode, ctx().cur);
}

// y = x W^T + bias on fp16-piece operands (tcg_split_f16 of x [M, K] per
// K-block and of W [N, K] per row): kind::f16 MMAs, hi*hi + hi*lo + lo*hi per
// product; each 128-element K-block's row scale is undone in the drain, the
// column scales once per tile.
bool tcg_linear_f16_split(float *y, const void *x_hi, const void *x_lo, const int8_t *x_ex, const void *w_hi,
                          const void *w_lo, const int8_t *w_ex, const float *bias, int M, int N, int K, int x_blk)
{
    if (!need_ctx()) return false;
    if (M < 0 || N < 0 || K <= 0) return fail("tcg_linear_f16_split: bad shape %dx%dx%d", M, N, K);
    if (M == 0 || N == 0) return true;
    GemmEpi e;
    e.bias = bias;
    e.out.plain = y;
    e.out.ld = N;
    e.xa = x_ex;
    e.xb = w_ex;
    e.xa_blk = x_blk;
    GemmPlan p;
    const GemmWork *w = ctx_gemm_work();
    if (!w || !gemm_plan(p, (const float *)x_hi, (const float *)x_lo, (const float *)w_hi, (const float *)w_lo, M, N,
                         K, e, gemm_f16_cfg(), w))
        return false;
    return gemm_run(p, ctx().cur, ctx().d_err);
}

// Tuning hook: the fp16-piece GEMM configuration that ViT plans and
// tcg_linear_f16_split use afterwards: 16 (default) three stages of 64
// K-elements, 17 six stages of 32, 18 and 19 a CTA pair on 256 x 256 and
// 256 x 128 tiles (the three products folded into one accumulator), 20 one
// CTA with the three products folded (four chunk buffers). Other values only
// read the setting.
// Returns the previous one.
extern "C" int tcg_gemm_set_f16_cfg(int cfg)
{
    const int old = tcg::g_f16_cfg;
    if (cfg >= 16 && cfg <= 20) tcg::g_f16_cfg = cfg;
    return old;
}

// Tuning and test hook: 0 keeps every GEMM epilogue on plain stores, 1
// (default) uses bulk tensor stores where the output rows allow. Applies to
// GEMMs planned afterwards. Returns the previous setting.
int tcg_gemm_set_tma_store(int on)
{
    const int old = g_tma_store;
    g_tma_store = on ? 1 : 0;
    return old;
}

// y[M,N] = x[M,K] W^T + bias with W [N,K] held packed in Q4_K blocks on the
// device: the tensor-core GEMM dequantises W tile by tile in shared memory
// (the fused form of tc_dequant then tc_ref_linear, src/dequant.c:40-63,
// src/ops.c:28-35); only x is split, into the op scratch.
bool tcg_linear_q(float *y, const float *x, const void *Wq, const float *bias, int M, int N, int K, ggml_type_t t)
{
    if (!need_ctx()) return false;
    if (M < 0 || N < 0 || K < 0) return fail("tcg_linear_q: negative size");
    if (M == 0 || N == 0) return true;
    if (t != GGML_TYPE_Q4_K) return fail("tcg_linear_q: type %s has no packed GEMM (Q4_K only)", ggml_type_name(t));
    if (K == 0 || K % 256) return fail("tcg_linear_q: K=%d is not a positive multiple of 256", K);
    if (((uintptr_t)x & 15) || ((uintptr_t)Wq & 15))
        return fail("tcg_linear_q: x and the Q4_K matrix must be 16-byte aligned");
    cudaStream_t s = ctx().cur;
    const size_t xa = ((size_t)M * K + 3) & ~(size_t)3;
    float *buf = (float *)scratch(2 * xa * sizeof(float));
    if (!buf) return false;
    if (!launch_split(x, buf, buf + xa, (size_t)M * K, s)) return false;
    GemmEpi e;
    e.bias = bias;
    e.out.plain = y;
    e.out.ld = N;
    e.bq = (const uint8_t *)Wq;
    e.bq_row = (size_t)(K / 256) * 144;
    GemmPlan p;
    const GemmWork *w = ctx_gemm_work();
    if (!w || !gemm_plan(p, buf, buf + xa, nullptr, nullptr, M, N, K, e, CFG_Q4K, w)) return false;
    return gemm_run(p, s, ctx().d_err);
}

// Test hook: the grid size, stream-K flag, configuration and bulk-store
// epilogue flag of the latest GEMM plan made on this thread.
void tcg_gemm_last_plan(int out[4])
{
    for (int i = 0; i < 4; i++) out[i] = g_last_plan[i];
}

// Tuning and test hook: 0 turns the stream-K split of a GEMM's last, partial
// wave off (every tile computed whole, results independent of M), 1 splits it
// where the heuristic expects a gain, 2 whenever there is a partial wave.
// Applies to GEMMs planned afterwards. Returns the previous setting.
int tcg_gemm_set_streamk(int mode)
{
    const int old = g_streamk;
    g_streamk = mode < 0 ? 0 : (mode > 2 ? 2 : mode);
    return old;
}

// Tuning hook: make every automatic configuration choice (tcg_linear, the
// ViT's plans, built at upload) take configuration cfg; -1 restores the
// automatic choice. Returns the previous setting.
int tcg_gemm_force_cfg(int cfg)
{
    const int old = g_force_cfg;
    g_force_cfg = cfg >= 0 && cfg < gemm_num_cfgs() ? cfg : -1;
    return old;
}

// Test hook for the failure path of the stream-K hand-over: with on != 0,
// contributors stop raising their flags and an owner gives up waiting after
// wait_ms (then the kernel winds down, the device error word reads 8 and
// tcg_clear_device_error() makes the GEMMs usable again); on = 0 restores
// normal operation and the 4 s limit. Synchronous. The stream-K flags of a
// plan are only used by the throughput configuration (tcg_gemm_throughput_cfg).
bool tcg_test_gemm_withhold_flags(int on, double wait_ms)
{
    if (!need_ctx()) return false;
    const int w = on ? 1 : 0;
    const unsigned long long ns = on && wait_ms > 0 ? (unsigned long long)(wait_ms * 1e6) : WAIT_NS;
    TCG_CUDA(cudaStreamSynchronize(ctx().cur));
    TCG_CUDA(cudaMemcpyToSymbol(g_flag_withhold, &w, sizeof w));
    TCG_CUDA(cudaMemcpyToSymbol(g_flag_wait_ns, &ns, sizeof ns));
    return true;
}

int tcg_gemm_throughput_cfg(void) { return gemm_throughput_cfg(); }

// Test hook: bytes the op API has allocated on this thread's device for its
// grow-on-demand operand scratch and its stream-K workspace (0 until a call
// needs them).
size_t tcg_op_scratch_bytes(void)
{
    if (!ctx().ready) return 0;
    size_t b = ctx().scratch_bytes;
    if (ctx().gemm_work) {
        const GemmWork *w = (const GemmWork *)ctx().gemm_work;
        b += gemm_work_ws_floats(w->ctas) * sizeof(float) + gemm_work_flag_count(w->ctas) * sizeof(int);
    }
    return b;
}

// Test hook: K-elements per TMEM chunk (a multiple of 32; larger is faster
// and less accurate). Returns the previous value.
int tcg_gemm_set_chunk_k(int k)
{
    const int old = g_chunk_k;
    if (k >= 32 && k % 32 == 0) g_chunk_k = k;
    return old;
}

}  // extern "C"

// attn_tc.cu -- softmax attention (tc_ref_mha, src/ops.c:112-151) for
// head_dim 64 and long sequences (ViT-L/14: T = 257) on the 5th-generation
// tensor cores, fp32-accurate through 3xTF32.
//
// One CTA of 256 threads takes 128 consecutive queries of one (image, head);
// threads r and r + 128 share query row r = TMEM lane r, each with 32 of a
// block's keys and 32 of the output dims. Keys go in blocks of 64, each
// block's K and V loaded into registers while the previous block computes:
//   S = Q K^T    128 x 64 in TMEM columns 0-63: 8 K-steps of 8 dims x 3 tf32
//                products (lo*hi, hi*lo, hi*hi), 24 kind::tf32 MMAs;
//   softmax      the row's two threads scale their scores and exchange their
//                block maxima through shared memory; each keeps the running
//                maximum m, rescales by a = expf(m_old - m), takes p =
//                expf(s - m) and adds its p to its half of a double row sum;
//   O += P V     P goes back to shared memory as tf32 pairs and 24 MMAs give
//                P V (128 x 64) in TMEM columns 64-127; each thread folds its
//                32 dims into fp32 registers: o = o * a + pv.
// At the end o / (sum of the two halves) is written. The result is the reference's softmax up to
// the rounding of the running maximum's rescaling (a few ulp).
// Operands live in shared memory in the K-major, 128-byte-swizzled layout the
// UMMA descriptor reads: a [R x 32 fp32] tile has row r at r * 128 bytes and
// 16-byte chunk c at chunk c ^ (r & 7). Threads write them as tf32 pairs
// (hi = rn(v), lo = rn(v - hi)); V is written transposed ([dim][key], K-major
// in keys for the second product). Every wait is bounded; a wait that gives up
// raises the device error word, and the CTA runs its remaining steps without
// issuing MMAs, waits (bounded) for the last commit it issued and frees TMEM.
//
// Query rows past the last whole block of 128 (one row at T = 257) take the
// CTA-per-row kernel below, the reference's two passes on the CUDA cores.
#include "ops.cuh"
#include "numerics.cuh"
#include "tc05.cuh"

namespace tcg {
namespace {

constexpr int AL_THREADS = 256;
constexpr int AL_KB = 64;                                 // keys per block
constexpr uint32_t T128 = 128 * 128;                      // [128 x 32] fp32 tile, 16 KB
constexpr uint32_t T64 = 64 * 128;                        // [64 x 32] fp32 tile, 8 KB
// byte offsets in the 1024-aligned tile area (two 32-column tiles per operand)
constexpr uint32_t OFF_QH = 0, OFF_QL = 2 * T128;                     // Q [128 q x 64 d]
constexpr uint32_t OFF_KH = 4 * T128, OFF_KL = OFF_KH + 2 * T64;      // K block [64 keys x 64 d]
constexpr uint32_t OFF_VH = OFF_KL + 2 * T64, OFF_VL = OFF_VH + 2 * T64;   // V^T block [64 d x 64 keys]
constexpr uint32_t OFF_PH = OFF_VL + 2 * T64, OFF_PL = OFF_PH + 2 * T128;  // P block [128 q x 64 keys]
constexpr uint32_t AL_TILES = OFF_PL + 2 * T128;          // 192 KB
constexpr size_t AL_SMEM = 1024 + AL_TILES + 32 + 256 * 4 + 256 * 8;
constexpr uint32_t AL_TMEM_COLS = 256;                    // S: two buffers at 0 and 64, P V: at 128 and 192
constexpr unsigned long long AL_WAIT_NS = 4000000000ull;

// byte offset of element (r, c) of a [R x 32] swizzled fp32 tile
__device__ __forceinline__ uint32_t swz(int r, int c)
{
    return (uint32_t)(r * 128 + ((((c >> 2) ^ (r & 7)) & 7) << 4) + (c & 3) * 4);
}

__device__ __forceinline__ uint32_t idesc_f32(int M, int N)
{
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void fence_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_pair4(uint8_t *tiles, uint32_t off_hi, uint32_t off_lo, uint32_t o, float4 v)
{
    float h[4], l[4];
    split_tf32(v.x, h[0], l[0]);
    split_tf32(v.y, h[1], l[1]);
    split_tf32(v.z, h[2], l[2]);
    split_tf32(v.w, h[3], l[3]);
    *reinterpret_cast<float4 *>(tiles + off_hi + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4 *>(tiles + off_lo + o) = make_float4(l[0], l[1], l[2], l[3]);
}

// 24 MMAs: D (128 x 64) = A (128 x 64, two tiles of T128) * B^T (64 x 64, two
// tiles of T64), A and B as hi/lo pairs.
__device__ __forceinline__ void mma_3x(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo)
{
    const uint32_t id = idesc_f32(128, 64);
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
        const uint32_t ao = (uint32_t)(ks >> 2) * T128 + (uint32_t)(ks & 3) * 32;
        const uint32_t bo = (uint32_t)(ks >> 2) * T64 + (uint32_t)(ks & 3) * 32;
        const unsigned long long ah = sdesc<128>(a_hi + ao), al = sdesc<128>(a_lo + ao);
        const unsigned long long bh = sdesc<128>(b_hi + bo), bl = sdesc<128>(b_lo + bo);
        mma_tf32(d, al, bh, id, ks > 0 ? 1u : 0u);
        mma_tf32(d, ah, bl, id, 1u);
        mma_tf32(d, ah, bh, id, 1u);
    }
}

__global__ void __launch_bounds__(AL_THREADS, 1)
mha64_tc_long_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
                     int T, OutSpec out, int *err)
{
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *tiles = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(tiles + AL_TILES);
    uint32_t *tmem_slot = (uint32_t *)(bars + 2);
    volatile int *abort = (volatile int *)(tmem_slot + 1);
    float *xmax = (float *)(tiles + AL_TILES + 32);              // [256] block maxima of the two halves
    double *xsum = (double *)(tiles + AL_TILES + 32 + 256 * 4);  // [256] row sums of the two halves
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & 127, h = tid >> 7;                       // query row, half (keys / dims 32h .. 32h + 31)
    const uint32_t bar_s = su32(bars), bar_o = su32(bars + 1);
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    const int q0 = blockIdx.z * 128;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);

    if (tid == 0) {
        bar_init(bar_s, 1);
        bar_init(bar_o, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(su32(tmem_slot)), "r"(AL_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Q: 128 rows x 16 float4; consecutive threads take consecutive float4 of a row
    for (int i = tid; i < 128 * 16; i += AL_THREADS) {
        const int qr = i >> 4, d4 = i & 15;
        const float4 x = __ldg(reinterpret_cast<const float4 *>(q + (base + q0 + qr) * (size_t)ldi + col + 4 * d4));
        st_pair4(tiles, OFF_QH, OFF_QL, (uint32_t)(d4 >> 3) * T128 + swz(qr, 4 * (d4 & 7)), x);
    }
    // A block's K and V in registers: K element i = tid + 256 u -> key i >> 4, float4 i & 15;
    // V: thread -> key tid & 63, dims 16 (tid >> 6) .. + 15
    float4 kreg[4], vreg[4];
    auto load_k = [&](int t0, int nk) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = tid + AL_THREADS * u, key = i >> 4, d4 = i & 15;
            kreg[u] = key < nk ? __ldg(reinterpret_cast<const float4 *>(k + (base + t0 + key) * (size_t)ldi + col + 4 * d4))
                               : zero;
        }
    };
    auto load_v = [&](int t0, int nk) {
        const int key = tid & 63, dq = tid >> 6;
#pragma unroll
        for (int u = 0; u < 4; u++)
            vreg[u] = key < nk ? __ldg(reinterpret_cast<const float4 *>(v + (base + t0 + key) * (size_t)ldi + col + 16 * dq + 4 * u))
                               : zero;
    };
    auto load_kv = [&](int t0, int nk) {
        load_k(t0, nk);
        load_v(t0, nk);
    };
    auto store_k = [&]() {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = tid + AL_THREADS * u, key = i >> 4, d4 = i & 15;
            st_pair4(tiles, OFF_KH, OFF_KL, (uint32_t)(d4 >> 3) * T64 + swz(key, 4 * (d4 & 7)), kreg[u]);
        }
    };
    auto store_v = [&]() {
        const int key = tid & 63, dq = tid >> 6;
        const uint32_t kt = (uint32_t)(key >> 5) * T64;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float xv[4] = { vreg[u].x, vreg[u].y, vreg[u].z, vreg[u].w };
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float hi, lo;
                split_tf32(xv[j], hi, lo);
                const uint32_t off = kt + swz(16 * dq + 4 * u + j, key & 31);
                *reinterpret_cast<float *>(tiles + OFF_VH + off) = hi;
                *reinterpret_cast<float *>(tiles + OFF_VL + off) = lo;
            }
        }
    };
    const int nblk = (T + AL_KB - 1) / AL_KB;
    load_kv(0, min(AL_KB, T));
    store_k();                                                   // K of block 0; its V stays in registers
    fence_async_smem();
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tbase = su32(tiles);
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    bool ok = true;
    int last_s = -1, last_o = -1;    // blocks of thread 0's latest S and P V commits
    if (tid == 0) {
        mma_3x(tmem, tbase + OFF_QH, tbase + OFF_QL, tbase + OFF_KH, tbase + OFF_KL);
        mma_commit(bar_s);
        last_s = 0;
    }
    __syncwarp();
    if (nblk > 1) load_k(AL_KB, min(AL_KB, T - AL_KB));         // K of block 1

    const float scale = 1.0f / sqrtf(64.0f);
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; j++) o[j] = 0.0f;
    float m = -INFINITY, a_prev = 0.0f;
    double sum = 0.0;                                            // this half's share of the row sum
    // Block kb: S(kb) was issued a block earlier into S buffer kb & 1; after it
    // lands, K(kb + 1) replaces K(kb) and S(kb + 1) goes to the other buffer
    // while this block's softmax runs; P V(kb - 1), issued a block earlier, is
    // folded late (with its rescale factor a_prev); then P(kb) and V(kb)
    // replace P(kb - 1) and V(kb - 1) and P V(kb) goes to P V buffer kb & 1.
    for (int kb = 0; kb < nblk; kb++) {
        const int t0 = kb * AL_KB, nk = min(AL_KB, T - t0);
        if (ok) ok = bar_wait(bar_s, (uint32_t)(kb & 1), abort, err, 13);
        fence_after();
        float p[32];
        {
            uint32_t sv[32];
            tmem_ld32(lane_base + 64 * (kb & 1) + 32 * h, sv);
            float mb = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                p[j] = __fmul_rn(__uint_as_float(sv[j]), scale);
                if (32 * h + j < nk) mb = fmaxf(mb, p[j]);
            }
            xmax[tid] = mb;
        }
        if (kb + 1 < nblk) store_k();                            // S(kb) is done with K(kb)
        fence_async_smem();
        fence_before();
        __syncthreads();                 // both halves' maxima posted; K(kb + 1) in place
        fence_after();
        if (tid == 0 && ok && kb + 1 < nblk) {
            mma_3x(tmem + 64 * ((kb + 1) & 1), tbase + OFF_QH, tbase + OFF_QL, tbase + OFF_KH, tbase + OFF_KL);
            mma_commit(bar_s);
            last_s = kb + 1;
        }
        __syncwarp();
        if (kb + 2 < nblk) load_k(t0 + 2 * AL_KB, min(AL_KB, T - t0 - 2 * AL_KB));
        const float mn = fmaxf(m, fmaxf(xmax[r], xmax[r + 128]));
        const float a = expf(__fsub_rn(m, mn));                  // 0 on the first block (m = -inf)
        {
            double bs = 0.0;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                p[j] = 32 * h + j < nk ? expf(__fsub_rn(p[j], mn)) : 0.0f;
                bs += (double)p[j];
            }
            sum = sum * (double)a + bs;
            m = mn;
        }
        if (kb > 0) {                                            // fold P V(kb - 1)
            if (ok) ok = bar_wait(bar_o, (uint32_t)((kb - 1) & 1), abort, err, 14);
            fence_after();
            uint32_t pv[32];
            tmem_ld32(lane_base + 128 + 64 * ((kb - 1) & 1) + 32 * h, pv);
#pragma unroll
            for (int j = 0; j < 32; j++) o[j] = fmaf(o[j], a_prev, __uint_as_float(pv[j]));
        }
#pragma unroll
        for (int c4 = 0; c4 < 8; c4++)
            st_pair4(tiles, OFF_PH, OFF_PL, (uint32_t)h * T128 + swz(r, 4 * c4),
                     make_float4(p[4 * c4], p[4 * c4 + 1], p[4 * c4 + 2], p[4 * c4 + 3]));
        store_v();                                               // V(kb), loaded a block earlier
        fence_async_smem();
        fence_before();
        __syncthreads();                 // P(kb), V(kb) in place; P V(kb - 1) and the maxima read
        fence_after();
        if (tid == 0 && ok) {
            mma_3x(tmem + 128 + 64 * (kb & 1), tbase + OFF_PH, tbase + OFF_PL, tbase + OFF_VH, tbase + OFF_VL);
            mma_commit(bar_o);
            last_o = kb;
        }
        __syncwarp();
        if (kb + 1 < nblk) load_v(t0 + AL_KB, min(AL_KB, T - t0 - AL_KB));
        a_prev = a;
    }
    if (ok) ok = bar_wait(bar_o, (uint32_t)((nblk - 1) & 1), abort, err, 14);
    fence_after();
    {
        uint32_t pv[32];
        tmem_ld32(lane_base + 128 + 64 * ((nblk - 1) & 1) + 32 * h, pv);
#pragma unroll
        for (int j = 0; j < 32; j++) o[j] = fmaf(o[j], a_prev, __uint_as_float(pv[j]));
    }
    xsum[tid] = sum;
    __syncthreads();
    if (ok) {
        const float inv = (float)(1.0 / (xsum[r] + xsum[r + 128]));
        const size_t row = base + q0 + r;
#pragma unroll
        for (int d = 0; d < 32; d += 4) {
            const float o4[4] = { __fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                                  __fmul_rn(o[d + 3], inv) };
            const size_t i = row * (size_t)out.ld + col + 32 * h + d;
            if (out.plain) *reinterpret_cast<float4 *>(out.plain + i) = make_float4(o4[0], o4[1], o4[2], o4[3]);
            if (out.hi) {
                float hi4[4], lo4[4];
#pragma unroll
                for (int u = 0; u < 4; u++) split_tf32(o4[u], hi4[u], lo4[u]);
                *reinterpret_cast<float4 *>(out.hi + i) = make_float4(hi4[0], hi4[1], hi4[2], hi4[3]);
                *reinterpret_cast<float4 *>(out.lo + i) = make_float4(lo4[0], lo4[1], lo4[2], lo4[3]);
            }
        }
    }
    // MMAs that may still run (a wait gave up) must finish before TMEM is freed:
    // thread 0 waits, bounded, for the last commit it issued.
    if (!ok && tid == 0) {
        const unsigned long long t0 = now_ns();
        if (last_s >= 0)
            while (!bar_test(bar_s, (uint32_t)(last_s & 1)) && now_ns() - t0 < AL_WAIT_NS) {}
        if (last_o >= 0)
            while (!bar_test(bar_o, (uint32_t)(last_o & 1)) && now_ns() - t0 < AL_WAIT_NS) {}
    }
    fence_before();
    __syncthreads();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AL_TMEM_COLS) : "memory");
    }
}

// One CTA of 256 threads per query row (rows row0 .. T - 1): the reference's
// two passes (src/ops.c:129-139). Thread t scores keys t, t + 256, ... against
// the row (dims in order); the block's maximum, expf of the differences, a
// double sum over the warps in order and its reciprocal; then thread t sums
// dim t & 63 over one quarter of the keys (in order, V rows read coalesced,
// eight in flight), and the quarters are added in order.
__global__ void __launch_bounds__(256)
mha64_row_cta_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
                     int T, int row0, OutSpec out)
{
    pdl_wait();
    __shared__ __align__(16) float qs[64];
    __shared__ float ps[1024];
    __shared__ float wmax[8];
    __shared__ double wsum[8];
    __shared__ float part[4][64];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = row0 + blockIdx.z;
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    if (tid < 16)
        reinterpret_cast<float4 *>(qs)[tid] =
            __ldg(reinterpret_cast<const float4 *>(q + (base + row) * (size_t)ldi + col + 4 * tid));
    __syncthreads();
    const float scale = 1.0f / sqrtf(64.0f);
    float mx = -INFINITY;
    for (int s = tid; s < T; s += 256) {
        const float4 *kr = reinterpret_cast<const float4 *>(k + (base + s) * (size_t)ldi + col);
        float4 x[16];
#pragma unroll
        for (int d4 = 0; d4 < 16; d4++) x[d4] = __ldg(kr + d4);
        float acc = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < 16; d4++) {
            acc = fmaf(qs[4 * d4], x[d4].x, acc);
            acc = fmaf(qs[4 * d4 + 1], x[d4].y, acc);
            acc = fmaf(qs[4 * d4 + 2], x[d4].z, acc);
            acc = fmaf(qs[4 * d4 + 3], x[d4].w, acc);
        }
        ps[s] = __fmul_rn(acc, scale);
        mx = fmaxf(mx, ps[s]);
    }
    mx = warp_max(mx);
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    mx = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, wmax[w]);
    double sum = 0.0;
    for (int s = tid; s < T; s += 256) {
        const float e = expf(__fsub_rn(ps[s], mx));
        ps[s] = e;
        sum += (double)e;
    }
    sum = warp_sum(sum);
    if (lane == 0) wsum[warp] = sum;
    __syncthreads();
    double tot = wsum[0];
#pragma unroll
    for (int w = 1; w < 8; w++) tot += wsum[w];
    const float inv = (float)(1.0 / tot);
    const int d = tid & 63, qq = tid >> 6, per = (T + 3) / 4;
    const int s0 = qq * per, s1 = min(T, s0 + per);
    float o = 0.0f;
    for (int s = s0; s < s1; s += 8) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) x[u] = s + u < s1 ? __ldg(v + (base + s + u) * (size_t)ldi + col + d) : 0.0f;
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (s + u < s1) o = fmaf(__fmul_rn(ps[s + u], inv), x[u], o);
    }
    part[qq][d] = o;
    __syncthreads();
    if (tid < 64) {
        const float r = __fadd_rn(__fadd_rn(__fadd_rn(part[0][tid], part[1][tid]), part[2][tid]), part[3][tid]);
        const size_t i = (base + row) * (size_t)out.ld + col + tid;
        if (out.plain) out.plain[i] = r;
        if (out.hi) {
            float hi, lo;
            split_tf32(r, hi, lo);
            out.hi[i] = hi;
            out.lo[i] = lo;
        }
    }
}

}  // namespace

// head_dim 64, 128 <= T <= 1024: whole blocks of 128 queries on the tensor
// cores, the rest one CTA per row. False (nothing launched) when the shape
// does not fit; the caller then takes a CUDA-core kernel.
bool launch_mha64_tc_long(const float *q, const float *k, const float *v, int ldi, int T, int n_head, int n_img,
                          const OutSpec &out, cudaStream_t s)
{
    if (T < 128 || T > 1024) return false;
    static unsigned done[64];
    const int dev = ctx().device & 63;
    if (!done[dev]) {
        TCG_CUDA(cudaFuncSetAttribute(mha64_tc_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AL_SMEM));
        done[dev] = 1;
    }
    const int nfull = T / 128, rest = T - 128 * nfull;
    TCG_CUDA(launch_pdl(mha64_tc_long_kernel, dim3(n_head, n_img, nfull), dim3(AL_THREADS), AL_SMEM, s, q, k, v, ldi, T,
                        out, ctx().d_err));
    if (rest > 0)
        TCG_CUDA(launch_pdl(mha64_row_cta_kernel, dim3(n_head, n_img, rest), dim3(256), 0, s, q, k, v, ldi, T,
                            128 * nfull, out));
    TCG_LAUNCHED();
    return true;
}

}  // namespace tcg

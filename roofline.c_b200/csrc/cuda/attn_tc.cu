// attn_tc.cu -- softmax attention (tc_ref_mha, src/ops.c:112-151) for
// head_dim 64 and long sequences (ViT-L/14: T = 257) on the 5th-generation
// tensor cores, fp32-accurate through 3xTF32.
//
// One CTA of 128 threads takes 128 consecutive queries of one (image, head);
// thread r owns query row r = TMEM lane r. Keys go in blocks of 64:
//   S = Q K^T    128 x 64 in TMEM columns 0-63: 8 K-steps of 8 dims x 3 tf32
//                products (lo*hi, hi*lo, hi*hi), 24 kind::tf32 MMAs;
//   softmax      thread r scales its row, keeps a running maximum m, rescales
//                by a = expf(m_old - m), takes p = expf(s - m), and adds the
//                p to a double row sum;
//   O += P V     P goes back to shared memory as tf32 pairs and 24 MMAs give
//                P V (128 x 64) in TMEM columns 64-127; thread r folds its
//                row into 64 fp32 registers: o = o * a + pv.
// At the end o / sum is written. The result is the reference's softmax up to
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
// warp-per-row kernel below, the reference's two passes on the CUDA cores.
#include "ops.cuh"
#include "numerics.cuh"
#include "tc05.cuh"

namespace tcg {
namespace {

constexpr int AL_THREADS = 128;
constexpr int AL_KB = 64;                                 // keys per block
constexpr uint32_t T128 = 128 * 128;                      // [128 x 32] fp32 tile, 16 KB
constexpr uint32_t T64 = 64 * 128;                        // [64 x 32] fp32 tile, 8 KB
// byte offsets in the 1024-aligned tile area (two 32-column tiles per operand)
constexpr uint32_t OFF_QH = 0, OFF_QL = 2 * T128;                     // Q [128 q x 64 d]
constexpr uint32_t OFF_KH = 4 * T128, OFF_KL = OFF_KH + 2 * T64;      // K block [64 keys x 64 d]
constexpr uint32_t OFF_VH = OFF_KL + 2 * T64, OFF_VL = OFF_VH + 2 * T64;   // V^T block [64 d x 64 keys]
constexpr uint32_t OFF_PH = OFF_VL + 2 * T64, OFF_PL = OFF_PH + 2 * T128;  // P block [128 q x 64 keys]
constexpr uint32_t AL_TILES = OFF_PL + 2 * T128;          // 192 KB
constexpr size_t AL_SMEM = 1024 + AL_TILES + 64;
constexpr uint32_t AL_TMEM_COLS = 128;                    // S: 0-63, P V: 64-127
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
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
        const int r = i >> 4, d4 = i & 15;
        const float4 x = __ldg(reinterpret_cast<const float4 *>(q + (base + q0 + r) * (size_t)ldi + col + 4 * d4));
        st_pair4(tiles, OFF_QH, OFF_QL, (uint32_t)(d4 >> 3) * T128 + swz(r, 4 * (d4 & 7)), x);
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tbase = su32(tiles);
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);

    const float scale = 1.0f / sqrtf(64.0f);
    float o[64];
#pragma unroll
    for (int j = 0; j < 64; j++) o[j] = 0.0f;
    float m = -INFINITY;
    double sum = 0.0;
    bool ok = true;
    int issued = 0;                  // thread 0's last commit: 1 S, 2 P V (of block last_kb)
    int last_kb = 0;
    const int nblk = (T + AL_KB - 1) / AL_KB;
    for (int kb = 0; kb < nblk; kb++) {
        const int t0 = kb * AL_KB, nk = min(AL_KB, T - t0);
        // K block: 64 keys x 16 float4 (keys past T zero)
        for (int i = tid; i < AL_KB * 16; i += AL_THREADS) {
            const int r = i >> 4, d4 = i & 15;
            const float4 x = r < nk ? __ldg(reinterpret_cast<const float4 *>(k + (base + t0 + r) * (size_t)ldi + col + 4 * d4))
                                    : zero;
            st_pair4(tiles, OFF_KH, OFF_KL, (uint32_t)(d4 >> 3) * T64 + swz(r, 4 * (d4 & 7)), x);
        }
        // V block transposed: thread -> key tid & 63, dims 32 (tid >> 6) .. + 31
        {
            const int key = tid & 63, dh = tid >> 6;
            const bool in = key < nk;
            const float *src = v + (base + t0 + key) * (size_t)ldi + col + 32 * dh;
            const uint32_t kt = (uint32_t)(key >> 5) * T64;
#pragma unroll 2
            for (int d4 = 0; d4 < 8; d4++) {
                const float4 x = in ? __ldg(reinterpret_cast<const float4 *>(src + 4 * d4)) : zero;
                const float xv[4] = { x.x, x.y, x.z, x.w };
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float h, l;
                    split_tf32(xv[j], h, l);
                    const uint32_t off = kt + swz(32 * dh + 4 * d4 + j, key & 31);
                    *reinterpret_cast<float *>(tiles + OFF_VH + off) = h;
                    *reinterpret_cast<float *>(tiles + OFF_VL + off) = l;
                }
            }
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        fence_after();
        if (tid == 0 && ok) {
            mma_3x(tmem, tbase + OFF_QH, tbase + OFF_QL, tbase + OFF_KH, tbase + OFF_KL);
            mma_commit(bar_s);
            issued = 1;
            last_kb = kb;
        }
        __syncwarp();
        if (ok) ok = bar_wait(bar_s, (uint32_t)(kb & 1), abort, err, 13);
        fence_after();
        // softmax step of row tid over this block's nk keys
        float p[64];
        float a;
        {
            uint32_t sv[64];
            tmem_ld64(lane_base, sv);
            float mb = -INFINITY;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                p[j] = __fmul_rn(__uint_as_float(sv[j]), scale);
                if (j < nk) mb = fmaxf(mb, p[j]);
            }
            const float mn = fmaxf(m, mb);
            a = expf(__fsub_rn(m, mn));              // 0 on the first block (m = -inf)
            double bs = 0.0;
#pragma unroll
            for (int j = 0; j < 64; j++) {
                p[j] = j < nk ? expf(__fsub_rn(p[j], mn)) : 0.0f;
                bs += (double)p[j];
            }
            sum = sum * (double)a + bs;
            m = mn;
        }
        fence_before();
        __syncthreads();                         // every row's S is read; the last P V is folded
#pragma unroll
        for (int c4 = 0; c4 < 16; c4++) {
            const int key = 4 * c4;
            st_pair4(tiles, OFF_PH, OFF_PL, (uint32_t)(key >> 5) * T128 + swz(tid, key & 31),
                     make_float4(p[key], p[key + 1], p[key + 2], p[key + 3]));
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        fence_after();
        if (tid == 0 && ok) {
            mma_3x(tmem + 64, tbase + OFF_PH, tbase + OFF_PL, tbase + OFF_VH, tbase + OFF_VL);
            mma_commit(bar_o);
            issued = 2;
            last_kb = kb;
        }
        __syncwarp();
        if (ok) ok = bar_wait(bar_o, (uint32_t)(kb & 1), abort, err, 14);
        fence_after();
        {
            uint32_t pv[64];
            tmem_ld64(lane_base + 64, pv);
#pragma unroll
            for (int j = 0; j < 64; j++) o[j] = fmaf(o[j], a, __uint_as_float(pv[j]));
        }
        fence_before();
        __syncthreads();                         // P V is read; the next block may overwrite K, V, P
        fence_after();
    }
    if (ok) {
        const float inv = (float)(1.0 / sum);
        const size_t row = base + q0 + tid;
#pragma unroll
        for (int d = 0; d < 64; d += 4) {
            const float o4[4] = { __fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv), __fmul_rn(o[d + 2], inv),
                                  __fmul_rn(o[d + 3], inv) };
            const size_t i = row * (size_t)out.ld + col + d;
            if (out.plain) *reinterpret_cast<float4 *>(out.plain + i) = make_float4(o4[0], o4[1], o4[2], o4[3]);
            if (out.hi) {
                float h[4], l[4];
#pragma unroll
                for (int u = 0; u < 4; u++) split_tf32(o4[u], h[u], l[u]);
                *reinterpret_cast<float4 *>(out.hi + i) = make_float4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<float4 *>(out.lo + i) = make_float4(l[0], l[1], l[2], l[3]);
            }
        }
    }
    // MMAs that may still run (a wait gave up) must finish before TMEM is freed:
    // thread 0 waits, bounded, for the last commit it issued.
    if (!ok && tid == 0 && issued) {
        const uint32_t last = issued == 2 ? bar_o : bar_s;
        const uint32_t parity = (uint32_t)(last_kb & 1);
        const unsigned long long t0 = now_ns();
        while (!bar_test(last, parity) && now_ns() - t0 < AL_WAIT_NS) {}
    }
    fence_before();
    __syncthreads();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AL_TMEM_COLS) : "memory");
    }
}

// One warp per query row (rows row0 .. T - 1): the reference's two passes.
// Lane l scores keys l, l + 32, ... against the whole query row; the maximum,
// expf of the differences, the double sum and its reciprocal as in
// src/ops.c:129-139; lane l then accumulates output dims 2l, 2l + 1 over the
// keys in order, taking each probability from its lane by a shuffle.
constexpr int AR_KEYS = 32;                               // keys per lane (T <= 1024)

__global__ void __launch_bounds__(128)
mha64_rows_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
                  int T, int row0, OutSpec out)
{
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = row0 + blockIdx.z * 4 + (threadIdx.x >> 5);
    if (row >= T) return;
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    float qr[64];
#pragma unroll
    for (int d4 = 0; d4 < 16; d4++) {
        const float4 x = __ldg(reinterpret_cast<const float4 *>(q + (base + row) * (size_t)ldi + col + 4 * d4));
        qr[4 * d4] = x.x; qr[4 * d4 + 1] = x.y; qr[4 * d4 + 2] = x.z; qr[4 * d4 + 3] = x.w;
    }
    const float scale = 1.0f / sqrtf(64.0f);
    float e[AR_KEYS];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < AR_KEYS; i++) {
        const int s = lane + 32 * i;
        e[i] = -INFINITY;
        if (s < T) {
            const float *kr = k + (base + s) * (size_t)ldi + col;
            float acc = 0.0f;
#pragma unroll
            for (int d4 = 0; d4 < 16; d4++) {
                const float4 x = __ldg(reinterpret_cast<const float4 *>(kr + 4 * d4));
                acc = fmaf(qr[4 * d4], x.x, acc);
                acc = fmaf(qr[4 * d4 + 1], x.y, acc);
                acc = fmaf(qr[4 * d4 + 2], x.z, acc);
                acc = fmaf(qr[4 * d4 + 3], x.w, acc);
            }
            e[i] = __fmul_rn(acc, scale);
            mx = fmaxf(mx, e[i]);
        }
    }
    mx = warp_max(mx);
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < AR_KEYS; i++) {
        const int s = lane + 32 * i;
        e[i] = s < T ? expf(__fsub_rn(e[i], mx)) : 0.0f;
        sum += (double)e[i];
    }
    const float inv = (float)(1.0 / warp_sum(sum));
    float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
    for (int i = 0; i < AR_KEYS; i++) {
        if (32 * i >= T) break;
        const float ps = __fmul_rn(e[i], inv);
        for (int s8 = 0; s8 < 32; s8 += 8) {                // eight V rows in flight, then their sums in order
            if (32 * i + s8 >= T) break;
            float2 x[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int s = 32 * i + s8 + u;
                x[u] = s < T ? __ldg(reinterpret_cast<const float2 *>(v + (base + s) * (size_t)ldi + col + 2 * lane))
                             : make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float p = __shfl_sync(0xffffffffu, ps, s8 + u);
                if (32 * i + s8 + u < T) {
                    o0 = fmaf(p, x[u].x, o0);
                    o1 = fmaf(p, x[u].y, o1);
                }
            }
        }
    }
    const size_t i = (base + row) * (size_t)out.ld + col + 2 * lane;
    if (out.plain) {
        out.plain[i] = o0;
        out.plain[i + 1] = o1;
    }
    if (out.hi) {
        float h, l;
        split_tf32(o0, h, l);
        out.hi[i] = h;
        out.lo[i] = l;
        split_tf32(o1, h, l);
        out.hi[i + 1] = h;
        out.lo[i + 1] = l;
    }
}

}  // namespace

// head_dim 64, 128 <= T <= 1024: whole blocks of 128 queries on the tensor
// cores, the rest one warp per row. False (nothing launched) when the shape
// does not fit; the caller then takes a CUDA-core kernel.
bool launch_mha64_tc_long(const float *q, const float *k, const float *v, int ldi, int T, int n_head, int n_img,
                          const OutSpec &out, cudaStream_t s)
{
    if (T < 128 || T > 32 * AR_KEYS) return false;
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
        TCG_CUDA(launch_pdl(mha64_rows_kernel, dim3(n_head, n_img, (rest + 3) / 4), dim3(128), 0, s, q, k, v, ldi, T,
                            128 * nfull, out));
    TCG_LAUNCHED();
    return true;
}

}  // namespace tcg

// ops.cu -- CUDA-core kernels for the O(T*D) ops of roofline.c src/ops.c and
// the op-level C ABI (tcg_layernorm, tcg_gelu, ..., tcg_mha).
#include "ops.cuh"
#include "numerics.cuh"
#include "gemm.cuh"

#include <cuda_fp16.h>
#include <type_traits>

namespace tcg {

__device__ __forceinline__ void put(const OutSpec &o, size_t row, int col, float v)
{
    const size_t i = row * (size_t)o.ld + col;
    if (o.plain) o.plain[i] = v;
    if (o.hi) {
        float h, l;
        split_tf32(v, h, l);
        o.hi[i] = h;
        o.lo[i] = l;
    }
}

__device__ __forceinline__ void put4(const OutSpec &o, size_t row, int col, const float (&v)[4])
{
    const size_t i = row * (size_t)o.ld + col;
    if (o.plain) *reinterpret_cast<float4 *>(o.plain + i) = make_float4(v[0], v[1], v[2], v[3]);
    if (o.hi) {
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) split_tf32(v[j], h[j], l[j]);
        *reinterpret_cast<float4 *>(o.hi + i) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(o.lo + i) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row. Pass 1: double sum -> mean. Pass 2: double sum of
// squared deviations -> biased variance. inv = (float)(1/sqrt(var+eps)) in
// double. Output (float)(x - mean) * inv, * gamma, + beta, each in float.
__global__ void layernorm_kernel(const float *x, int ld_in, const float *__restrict__ g,
                                 const float *__restrict__ b, int rows, int cols, float eps, OutSpec out)
{
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *in = x + (size_t)row * ld_in;
    double s = 0.0;
    for (int c = lane; c < cols; c += 32) s += (double)in[c];
    const double mean = warp_sum(s) / (double)cols;
    double ss = 0.0;
    for (int c = lane; c < cols; c += 32) {
        const double dv = __dsub_rn((double)in[c], mean);
        ss = __dadd_rn(ss, __dmul_rn(dv, dv));
    }
    const double var = warp_sum(ss) / (double)cols;
    const float inv = (float)(1.0 / sqrt(var + (double)eps));
    for (int c = lane; c < cols; c += 32) {
        float v = __fmul_rn((float)((double)in[c] - mean), inv);
        if (g) v = __fmul_rn(v, g[c]);
        if (b) v = __fadd_rn(v, b[c]);
        put(out, row, c, v);
    }
}

// The same LayerNorm with the row held in registers: lane l owns the float4s
// l, l + 32, ... (VPL of them, cols = 128 * VPL), read once and written once
// as float4 (plain or tf32 hi/lo). Same arithmetic as layernorm_kernel; the
// double sums run in another order. (Staging gamma/beta in shared memory
// needed 111 registers, two CTAs per SM, and ran 15% slower.)
template <int VPL>
__global__ void __launch_bounds__(256, 3)
layernorm_vec_kernel(const float *x, int ld_in, const float *__restrict__ g, const float *__restrict__ b, int rows,
                     float eps, OutSpec out)
{
    pdl_wait();
    constexpr int cols = 128 * VPL;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float4 *in = reinterpret_cast<const float4 *>(x + (size_t)row * ld_in);
    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = in[lane + 32 * i];
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < VPL; i++) s += ((double)v[i].x + (double)v[i].y) + ((double)v[i].z + (double)v[i].w);
    const double mean = warp_sum(s) / (double)cols;
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const double a = __dsub_rn((double)v[i].x, mean), bb = __dsub_rn((double)v[i].y, mean);
        const double c = __dsub_rn((double)v[i].z, mean), d = __dsub_rn((double)v[i].w, mean);
        ss = __dadd_rn(ss, __dadd_rn(__dadd_rn(__dmul_rn(a, a), __dmul_rn(bb, bb)),
                                     __dadd_rn(__dmul_rn(c, c), __dmul_rn(d, d))));
    }
    const double var = warp_sum(ss) / (double)cols;
    const float inv = (float)(1.0 / sqrt(var + (double)eps));
    if (out.fh) {
        // fp16 pieces: the whole row first, then one exponent per 256-column
        // block (float4s 2b and 2b+1 of every lane)
        float o[VPL][4];
#pragma unroll
        for (int i = 0; i < VPL; i++) {
            const int c = 4 * (lane + 32 * i);
            const float4 gg = g ? *reinterpret_cast<const float4 *>(g + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 bv = b ? *reinterpret_cast<const float4 *>(b + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float gv[4] = { gg.x, gg.y, gg.z, gg.w }, bb4[4] = { bv.x, bv.y, bv.z, bv.w };
            const float xv[4] = { v[i].x, v[i].y, v[i].z, v[i].w };
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float t = __fmul_rn((float)((double)xv[k] - mean), inv);
                if (g) t = __fmul_rn(t, gv[k]);
                if (b) t = __fadd_rn(t, bb4[k]);
                o[i][k] = t;
            }
        }
        if (out.rnorm) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < VPL; i++)
#pragma unroll
                for (int k = 0; k < 4; k++) ss = fmaf(o[i][k], o[i][k], ss);
#pragma unroll
            for (int d = 16; d >= 1; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
            if (lane == 0) out.rnorm[row] = sqrtf(ss);
        }
#pragma unroll
        for (int bk = 0; bk < VPL / 2; bk++) {
            float m = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; k++) m = fmaxf(m, fmaxf(fabsf(o[2 * bk][k]), fabsf(o[2 * bk + 1][k])));
#pragma unroll
            for (int d = 16; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
            const int e = f16_scale_exp(m);
            const float f = __int_as_float((127 + e) << 23);
#pragma unroll
            for (int i = 2 * bk; i < 2 * bk + 2; i++) {
                uint2 h, l;
                f16_pieces4(o[i], f, h, l);
                const size_t at = (size_t)row * out.ld + 4 * (lane + 32 * i);
                *reinterpret_cast<uint2 *>((__half *)out.fh + at) = h;
                *reinterpret_cast<uint2 *>((__half *)out.fl + at) = l;
            }
            if (lane == 0) out.fe[(size_t)bk * out.fe_rows + row] = (int8_t)e;
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int c = 4 * (lane + 32 * i);
        float o[4] = { __fmul_rn((float)((double)v[i].x - mean), inv), __fmul_rn((float)((double)v[i].y - mean), inv),
                       __fmul_rn((float)((double)v[i].z - mean), inv), __fmul_rn((float)((double)v[i].w - mean), inv) };
        if (g) {
            const float4 gg = *reinterpret_cast<const float4 *>(g + c);
            o[0] = __fmul_rn(o[0], gg.x); o[1] = __fmul_rn(o[1], gg.y);
            o[2] = __fmul_rn(o[2], gg.z); o[3] = __fmul_rn(o[3], gg.w);
        }
        if (b) {
            const float4 bv = *reinterpret_cast<const float4 *>(b + c);
            o[0] = __fadd_rn(o[0], bv.x); o[1] = __fadd_rn(o[1], bv.y);
            o[2] = __fadd_rn(o[2], bv.z); o[3] = __fadd_rn(o[3], bv.w);
        }
        put4(out, row, c, o);
    }
}

bool launch_layernorm(const float *x, int ld_in, const float *g, const float *b, int rows, int cols,
                      float eps, const OutSpec &out, cudaStream_t s)
{
    if (rows <= 0) return true;
    const auto a16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
    const bool vec = cols % 128 == 0 && cols <= 1024 && !(ld_in & 3) && !(out.ld & 3) && a16(x) && a16(g) &&
                     a16(b) && a16(out.plain) && a16(out.hi) && a16(out.lo);
    if (out.fh && (!vec || cols % 256 || !out.fl || !out.fe || out.plain || out.hi || ((uintptr_t)out.fh & 7) ||
                   ((uintptr_t)out.fl & 7)))
        return fail("layernorm: fp16-piece output needs whole 256-column blocks (cols %d) and no other output", cols);
    const unsigned grid = ceil_div(rows, 8);
    if (vec) {
        switch (cols / 128) {
        case 1: TCG_CUDA(launch_pdl(layernorm_vec_kernel<1>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 2: TCG_CUDA(launch_pdl(layernorm_vec_kernel<2>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 3: TCG_CUDA(launch_pdl(layernorm_vec_kernel<3>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 4: TCG_CUDA(launch_pdl(layernorm_vec_kernel<4>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 5: TCG_CUDA(launch_pdl(layernorm_vec_kernel<5>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 6: TCG_CUDA(launch_pdl(layernorm_vec_kernel<6>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        case 7: TCG_CUDA(launch_pdl(layernorm_vec_kernel<7>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        default: TCG_CUDA(launch_pdl(layernorm_vec_kernel<8>, grid, 256, 0, s, x, ld_in, g, b, rows, eps, out)); break;
        }
    } else {
        TCG_CUDA(launch_pdl(layernorm_kernel, grid, 256, 0, s, x, ld_in, g, b, rows, cols, eps, out));
    }
    TCG_LAUNCHED();
    return true;
}

// ---------------------------------------------------------------- attention
// One CTA per (head, image); K with a padded row (hd+1 floats) so that lanes
// walking different keys hit different banks; V unpadded (lanes walk d).
// One warp per query row: lane j scores keys j, j+32, ...; the softmax is
// max-subtracted with a double sum (src/ops.c:129-139); then lane d
// accumulates o[d] over keys in order.
template <int DPL>   // head dims per lane: hd <= 32*DPL
__global__ void mha_kernel(const float *__restrict__ q, const float *__restrict__ k,
                           const float *__restrict__ v, int ldi, int T, int hd, OutSpec out)
{
    pdl_wait();
    extern __shared__ float sm[];
    const int h = blockIdx.x, img = blockIdx.y;
    const int nw = blockDim.x >> 5, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int kst = hd + 1;
    float *Ks = sm;                           // [T][hd+1]
    float *Vs = Ks + (size_t)T * kst;         // [T][hd]
    float *Ps = Vs + (size_t)T * hd;          // [nw][T]
    float *Qs = Ps + (size_t)nw * T;          // [nw][hd]
    const size_t base = (size_t)img * T;
    const int col = h * hd;

    for (int i = threadIdx.x; i < T * hd; i += blockDim.x) {
        const int t = i / hd, d = i - t * hd;
        const size_t gi = (base + t) * (size_t)ldi + col + d;
        Ks[t * kst + d] = k[gi];
        Vs[t * hd + d] = v[gi];
    }
    __syncthreads();

    const float scale = 1.0f / sqrtf((float)hd);
    float *P = Ps + (size_t)wid * T, *Qr = Qs + (size_t)wid * hd;
    for (int t = wid; t < T; t += nw) {
        const float *qg = q + (base + t) * (size_t)ldi + col;
        for (int d = lane; d < hd; d += 32) Qr[d] = qg[d];
        __syncwarp();
        float mx = -INFINITY;
        for (int s = lane; s < T; s += 32) {
            const float *kr = Ks + s * kst;
            float acc = 0.0f;
            for (int d = 0; d < hd; d++) acc = fmaf(Qr[d], kr[d], acc);
            acc = __fmul_rn(acc, scale);
            P[s] = acc;
            mx = fmaxf(mx, acc);
        }
        mx = warp_max(mx);
        double sum = 0.0;
        for (int s = lane; s < T; s += 32) {
            const float e = expf(__fsub_rn(P[s], mx));
            P[s] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / warp_sum(sum));
        __syncwarp();
        float o[DPL];
#pragma unroll
        for (int j = 0; j < DPL; j++) o[j] = 0.0f;
        for (int s = 0; s < T; s++) {
            const float w = __fmul_rn(P[s], inv);
            const float *vr = Vs + s * hd;
#pragma unroll
            for (int j = 0; j < DPL; j++) {
                const int d = lane + 32 * j;
                if (d < hd) o[j] = fmaf(w, vr[d], o[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < DPL; j++) {
            const int d = lane + 32 * j;
            if (d < hd) put(out, base + t, col + d, o[j]);
        }
        __syncwarp();
    }
}

// head_dim 64 (every ViT here): one CTA per (head, image, block of 64
// queries), 16 x 16 threads, each owning a 4 x 4 register tile of the scores
// and then of the output. Keys are held transposed (d-major) so a thread's 4
// key columns are one 128-bit shared load; query and probability rows are
// read as per-row scalars that the 16 threads of a row share (broadcast).
// Softmax is exact two-pass per row as in src/ops.c:129-139 (max, expf, double
// sum, one reciprocal); the weighted sum runs over keys in order.
constexpr int MHA_BQ = 64;

__global__ void __launch_bounds__(256)
mha64_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
             int ldi, int T, OutSpec out)
{
    pdl_wait();
    extern __shared__ float4 sm4[];
    float *sm = reinterpret_cast<float *>(sm4);
    const int T4 = (T + 3) & ~3;
    float *Qs = sm;                      // [64][64]
    float *Kt = Qs + MHA_BQ * 64;        // [64][T4]
    float *Vs = Kt + 64 * T4;            // [T4][64]
    float *Ss = Vs + (size_t)T4 * 64;    // [64][T4]
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    const int q0 = blockIdx.z * MHA_BQ, nq = min(MHA_BQ, T - q0);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int i = threadIdx.x; i < T4 * 16; i += 256) {
        const int t = i >> 4, d = (i & 15) * 4;
        float4 kv = zero, vv = zero;
        if (t < T) {
            const size_t g = (base + t) * (size_t)ldi + col + d;
            kv = __ldg(reinterpret_cast<const float4 *>(k + g));
            vv = __ldg(reinterpret_cast<const float4 *>(v + g));
        }
        Kt[(d + 0) * T4 + t] = kv.x;
        Kt[(d + 1) * T4 + t] = kv.y;
        Kt[(d + 2) * T4 + t] = kv.z;
        Kt[(d + 3) * T4 + t] = kv.w;
        *reinterpret_cast<float4 *>(Vs + t * 64 + d) = vv;
    }
    for (int i = threadIdx.x; i < MHA_BQ * 16; i += 256) {
        const int t = i >> 4, d = (i & 15) * 4;
        float4 qv = zero;
        if (t < nq) qv = __ldg(reinterpret_cast<const float4 *>(q + (base + q0 + t) * (size_t)ldi + col + d));
        *reinterpret_cast<float4 *>(Qs + t * 64 + d) = qv;
    }
    __syncthreads();

    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const float scale = 1.0f / sqrtf(64.0f);
    for (int c0 = 0; c0 < T4; c0 += 64) {
        const int cc = c0 + 4 * tx;
        if (cc >= T4) continue;
        float acc[4][4] = {};
#pragma unroll 8
        for (int d = 0; d < 64; d++) {
            const float4 kk = *reinterpret_cast<const float4 *>(Kt + d * T4 + cc);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float a = Qs[(4 * ty + i) * 64 + d];
                acc[i][0] = fmaf(a, kk.x, acc[i][0]);
                acc[i][1] = fmaf(a, kk.y, acc[i][1]);
                acc[i][2] = fmaf(a, kk.z, acc[i][2]);
                acc[i][3] = fmaf(a, kk.w, acc[i][3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
            *reinterpret_cast<float4 *>(Ss + (4 * ty + i) * T4 + cc) =
                make_float4(__fmul_rn(acc[i][0], scale), __fmul_rn(acc[i][1], scale),
                            __fmul_rn(acc[i][2], scale), __fmul_rn(acc[i][3], scale));
    }
    __syncthreads();

    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int r = wid; r < nq; r += 8) {
        float *row = Ss + r * T4;
        float mx = -INFINITY;
        for (int s = lane; s < T; s += 32) mx = fmaxf(mx, row[s]);
        mx = warp_max(mx);
        double sum = 0.0;
        for (int s = lane; s < T; s += 32) {
            const float e = expf(__fsub_rn(row[s], mx));
            row[s] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / warp_sum(sum));
        for (int s = lane; s < T; s += 32) row[s] = __fmul_rn(row[s], inv);
    }
    __syncthreads();

    float o[4][4] = {};
    for (int s = 0; s < T; s++) {
        const float4 vv = *reinterpret_cast<const float4 *>(Vs + s * 64 + 4 * tx);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float p = Ss[(4 * ty + i) * T4 + s];
            o[i][0] = fmaf(p, vv.x, o[i][0]);
            o[i][1] = fmaf(p, vv.y, o[i][1]);
            o[i][2] = fmaf(p, vv.z, o[i][2]);
            o[i][3] = fmaf(p, vv.w, o[i][3]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (4 * ty + i < nq) put4(out, base + q0 + 4 * ty + i, col + 4 * tx, o[i]);
}

// head_dim 64, any T whose scores fit (ViT-L/14: 257 tokens): one CTA per
// (head, image, block of BQ queries), BQ/4 x 16 threads. The block's scores
// against all T keys stay in shared memory (the two-pass softmax of
// src/ops.c:129-139), while K and V stream through a double-buffered window
// of 64 keys, copied by cp.async in their row-major layout.
//   scores: thread (ty, tx) takes keys 4ty.., queries 4tx.. of the window; per
//           four dims, four float4 of K rows and four float4 of Q^T (Q stored
//           d-major once per CTA); sums run over d in order.
//   output: thread (qy, dx) takes queries 4qy.., dims 4dx..; per four keys,
//           four float4 of P and four of V; sums run over keys in order.
// The arithmetic is that of mha64_kernel, operation for operation.
constexpr int MHB_W = 64;            // keys per K/V window

__device__ __forceinline__ void mhb_cp16(float *dst, const float *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src) : "memory");
}

__host__ __device__ __forceinline__ int mhb_stride(int T)
{
    const int T4 = (T + 3) & ~3;
    return (T4 / 4) & 1 ? T4 : T4 + 4;        // an odd number of float4 per score row
}

template <int BQ>
static size_t mhb_smem(int T)
{
    return ((size_t)64 * BQ + (size_t)BQ * mhb_stride(T) + 2 * MHB_W * 64) * sizeof(float);
}

template <int BQ>
__global__ void __launch_bounds__(BQ * 4)
mha64b_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
              int T, OutSpec out)
{
    constexpr int NT = BQ * 4, QG = BQ / 4;
    pdl_wait();
    extern __shared__ float4 sm4[];
    const int TS = mhb_stride(T);
    float *Qt = reinterpret_cast<float *>(sm4);            // [64 d][BQ]
    float *Ss = Qt + 64 * BQ;                              // [BQ][TS]
    float *KV = Ss + (size_t)BQ * TS;                      // [2][MHB_W keys][64 d]
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    const int q0 = blockIdx.z * BQ, nq = min(BQ, T - q0);
    const int tid = threadIdx.x;
    const int nwin = (T + MHB_W - 1) / MHB_W;

    // rows t0 .. t0 + 63 of K or V into window buffer w (rows past T left as they are)
    auto fetch = [&](const float *src, int win) {
        float *dst = KV + (win & 1) * MHB_W * 64;
        const int t0 = win * MHB_W;
        for (int i = tid; i < MHB_W * 16; i += NT) {
            const int r = i >> 4, c = (i & 15) * 4;
            if (t0 + r < T) mhb_cp16(dst + r * 64 + c, src + (base + t0 + r) * (size_t)ldi + col + c);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(k, 0);
    // Q^T, d-major: a warp's lanes take consecutive queries of one float4 of dims
    for (int i = tid; i < BQ * 16; i += NT) {
        const int qq = i % BQ, d4 = i / BQ;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qq < nq) x = __ldg(reinterpret_cast<const float4 *>(q + (base + q0 + qq) * (size_t)ldi + col + 4 * d4));
        Qt[(4 * d4 + 0) * BQ + qq] = x.x;
        Qt[(4 * d4 + 1) * BQ + qq] = x.y;
        Qt[(4 * d4 + 2) * BQ + qq] = x.z;
        Qt[(4 * d4 + 3) * BQ + qq] = x.w;
    }

    const float scale = 1.0f / sqrtf(64.0f);
    {
        const int ty = tid / QG, tx = tid % QG;            // keys 4ty.., queries 4tx..
        for (int w = 0; w < nwin; w++) {
            if (w + 1 < nwin) fetch(k, w + 1);
            else asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncthreads();
            const float *Kb = KV + (w & 1) * MHB_W * 64;
            const int kc = w * MHB_W + 4 * ty;
            if (kc < T) {
                float acc[4][4] = {};                      // [key j][query i]
#pragma unroll 4
                for (int d = 0; d < 64; d += 4) {
                    float4 kr[4], qc[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) kr[j] = *reinterpret_cast<const float4 *>(Kb + (4 * ty + j) * 64 + d);
#pragma unroll
                    for (int c = 0; c < 4; c++) qc[c] = *reinterpret_cast<const float4 *>(Qt + (d + c) * BQ + 4 * tx);
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const float qv[4] = { qc[c].x, qc[c].y, qc[c].z, qc[c].w };
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float kv = c == 0 ? kr[j].x : c == 1 ? kr[j].y : c == 2 ? kr[j].z : kr[j].w;
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[j][i] = fmaf(qv[i], kv, acc[j][i]);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
                    *reinterpret_cast<float4 *>(Ss + (4 * tx + i) * TS + kc) =
                        make_float4(__fmul_rn(acc[0][i], scale), __fmul_rn(acc[1][i], scale),
                                    __fmul_rn(acc[2][i], scale), __fmul_rn(acc[3][i], scale));
            }
            __syncthreads();                               // window w is read; w + 2 may overwrite it
        }
    }
    fetch(v, 0);                                           // V's first window loads during the softmax

    const int lane = tid & 31, wid = tid >> 5;
    for (int r = wid; r < nq; r += NT / 32) {
        float *row = Ss + r * TS;
        float mx = -INFINITY;
        for (int s = lane; s < T; s += 32) mx = fmaxf(mx, row[s]);
        mx = warp_max(mx);
        double sum = 0.0;
        for (int s = lane; s < T; s += 32) {
            const float e = expf(__fsub_rn(row[s], mx));
            row[s] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / warp_sum(sum));
        for (int s = lane; s < T; s += 32) row[s] = __fmul_rn(row[s], inv);
    }

    const int qy = tid >> 4, dx = tid & 15;                // queries 4qy.., dims 4dx..
    float o[4][4] = {};
    for (int w = 0; w < nwin; w++) {
        if (w + 1 < nwin) fetch(v, w + 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();                                   // also: the softmax is done (first window)
        const float *Vb = KV + (w & 1) * MHB_W * 64;
        const int t0 = w * MHB_W, n = min(MHB_W, T - t0);
        if (4 * qy < nq) {
            for (int s0 = 0; s0 < n; s0 += 4) {
                float4 pr[4];
#pragma unroll
                for (int i = 0; i < 4; i++) pr[i] = *reinterpret_cast<const float4 *>(Ss + (4 * qy + i) * TS + t0 + s0);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (s0 + u >= n) break;
                    const float4 vv = *reinterpret_cast<const float4 *>(Vb + (s0 + u) * 64 + 4 * dx);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float pv = u == 0 ? pr[i].x : u == 1 ? pr[i].y : u == 2 ? pr[i].z : pr[i].w;
                        o[i][0] = fmaf(pv, vv.x, o[i][0]);
                        o[i][1] = fmaf(pv, vv.y, o[i][1]);
                        o[i][2] = fmaf(pv, vv.z, o[i][2]);
                        o[i][3] = fmaf(pv, vv.w, o[i][3]);
                    }
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (4 * qy + i < nq) put4(out, base + q0 + 4 * qy + i, col + 4 * dx, o[i]);
}

// head_dim 64 and T <= 64 (ViT-B/32: 50 tokens): one CTA of 16 x 16 threads
// per (head, image). Q and K are stored d-major (t contiguous), so the 4 x 4
// score tile of thread (ty, tx) -- rows 4ty.., keys 4tx.. -- costs two float4
// shared loads per d (the Q one a broadcast within the half-warp). The
// softmax runs on those registers: a row's 64 scores live in the 16 lanes of
// one half-warp, reduced by shuffles, with the steps of src/ops.c:129-139
// (max, expf of the difference, double sum, one reciprocal, multiply). P then
// overwrites Q's shared array row-major and the thread's 4 x 4 output tile --
// rows 4ty.., dims 4tx.. -- accumulates p * v over keys in order, with float4
// loads of P (broadcast) and V. 48 KB per CTA.
constexpr int MHAS_T = 64;

__global__ void __launch_bounds__(256, 4)
mha64s_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
              int T, OutSpec out)
{
    pdl_wait();
    __shared__ __align__(16) float Qt[64 * MHAS_T];    // [d][t], then P [t][s]
    __shared__ __align__(16) float Kt[64 * MHAS_T];    // [d][t]
    __shared__ __align__(16) float Vs[MHAS_T * 64];    // [t][d]
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);

    // Q, K transposed: a warp task is (matrix, 4 dims, 32 rows); lane = row,
    // so the shared stores are consecutive; the neighbouring tasks of a warp
    // read the other half of each 32-byte sector. All twelve loads of a thread
    // (eight Q/K tasks, four V float4s) are issued before the first store: one
    // memory round trip instead of twelve.
    float4 xqk[8], xv[4];
#pragma unroll
    for (int it = 0; it < 8; it++) {
        const int task = wid + 8 * it;
        const int mat = task >> 5, d4 = (task >> 1) & 15, t = (task & 1) * 32 + lane;
        const float *src = mat ? k : q;
        xqk[it] = t < T ? __ldg(reinterpret_cast<const float4 *>(src + (base + t) * (size_t)ldi + col + 4 * d4)) : zero;
    }
#pragma unroll
    for (int it = 0; it < 4; it++) {
        const int i = threadIdx.x + 256 * it;
        const int t = i >> 4, d = (i & 15) * 4;
        xv[it] = t < T ? __ldg(reinterpret_cast<const float4 *>(v + (base + t) * (size_t)ldi + col + d)) : zero;
    }
#pragma unroll
    for (int it = 0; it < 8; it++) {
        const int task = wid + 8 * it;
        const int mat = task >> 5, d4 = (task >> 1) & 15, t = (task & 1) * 32 + lane;
        float *dst = (mat ? Kt : Qt) + 4 * d4 * MHAS_T + t;
        dst[0] = xqk[it].x;
        dst[MHAS_T] = xqk[it].y;
        dst[2 * MHAS_T] = xqk[it].z;
        dst[3 * MHAS_T] = xqk[it].w;
    }
#pragma unroll
    for (int it = 0; it < 4; it++) {
        const int i = threadIdx.x + 256 * it;
        *reinterpret_cast<float4 *>(Vs + (i >> 4) * 64 + (i & 15) * 4) = xv[it];
    }
    __syncthreads();

    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const bool active = 4 * ty < T && 4 * tx < T;       // a half-warp shares ty: uniform per row group
    float sc[4][4] = {};
    if (4 * ty < T) {
#pragma unroll 8
        for (int d = 0; d < 64; d++) {
            const float4 a = *reinterpret_cast<const float4 *>(Qt + d * MHAS_T + 4 * ty);
            const float4 kk = *reinterpret_cast<const float4 *>(Kt + d * MHAS_T + 4 * tx);
            const float av[4] = { a.x, a.y, a.z, a.w };
#pragma unroll
            for (int i = 0; i < 4; i++) {
                sc[i][0] = fmaf(av[i], kk.x, sc[i][0]);
                sc[i][1] = fmaf(av[i], kk.y, sc[i][1]);
                sc[i][2] = fmaf(av[i], kk.z, sc[i][2]);
                sc[i][3] = fmaf(av[i], kk.w, sc[i][3]);
            }
        }
    }
    (void)active;
    const float scale = 1.0f / sqrtf(64.0f);
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            sc[i][j] = __fmul_rn(sc[i][j], scale);
            if (4 * tx + j < T) mx = fmaxf(mx, sc[i][j]);
        }
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        double sum = 0.0;
        float e[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            e[j] = 4 * tx + j < T ? expf(__fsub_rn(sc[i][j], mx)) : 0.0f;
            sum += (double)e[j];
        }
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = (float)(1.0 / sum);
#pragma unroll
        for (int j = 0; j < 4; j++) p[i][j] = __fmul_rn(e[j], inv);
    }
    __syncthreads();                                    // every thread is done with Qt
    float *Ps = Qt;                                     // [t][s]
#pragma unroll
    for (int i = 0; i < 4; i++)
        *reinterpret_cast<float4 *>(Ps + (4 * ty + i) * MHAS_T + 4 * tx) = make_float4(p[i][0], p[i][1], p[i][2], p[i][3]);
    __syncthreads();

    if (4 * ty >= T) return;
    float o[4][4] = {};
    const int T4 = (T + 3) & ~3;
    for (int s0 = 0; s0 < T4; s0 += 4) {
        float4 pr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) pr[i] = *reinterpret_cast<const float4 *>(Ps + (4 * ty + i) * MHAS_T + s0);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (s0 + u >= T) break;
            const float4 vv = *reinterpret_cast<const float4 *>(Vs + (s0 + u) * 64 + 4 * tx);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float pv = u == 0 ? pr[i].x : u == 1 ? pr[i].y : u == 2 ? pr[i].z : pr[i].w;
                o[i][0] = fmaf(pv, vv.x, o[i][0]);
                o[i][1] = fmaf(pv, vv.y, o[i][1]);
                o[i][2] = fmaf(pv, vv.z, o[i][2]);
                o[i][3] = fmaf(pv, vv.w, o[i][3]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (4 * ty + i < T) put4(out, base + 4 * ty + i, col + 4 * tx, o[i]);
}

// ------------------------------------------------ attention, T <= 64, mma.sync
// head_dim 64 and T <= 64 (ViT-B/32's 50 tokens) on the m16n8k16 tensor-core
// instruction with fp16 operands that carry an fp32 value in two pieces. A
// block is first scaled by a power of two that puts its largest magnitude in
// [2^14, 2^15), inside fp16's normal range (one scale per query row, one for
// the (image, head)'s K, one for its V; P, in [0, 1], is scaled by 2^14);
// scaling by a power of two is exact and is undone on the fp32 accumulators.
// Pieces: x = p1 + p2 + r, p1 = x rounded to 11 bits (exact in fp16), p2 =
// fp16(x - p1); |r| <= 2^-23 |x|, the precision of a tf32 pair. Q K^T takes the
// three products p1k1, p1k2, p2k1 and P V the three p1v1, p1v2, p2v1 (the
// fourth, p2 p2, is below 2^-24 of the product: under fp32's own rounding).
// The fp32 accumulation of an MMA truncates relative to its largest addend,
// so each accumulator sums every cross product (2^-11 of the result and
// less) over all keys or dims first and the four p1 p1 steps last: four
// truncations at the result's magnitude. Against the oracle this measures as
// close as the fp32 FMA kernel, peaked softmax rows included. The softmax
// follows src/ops.c:129-139 on the score accumulators (a row's keys sit in
// the four lanes of a quad): scale, max, expf of the difference, sum, one
// reciprocal (in double), multiply; a lane adds its 16 terms of a row in fp32
// (relative error below 2^-20) and the quad's four partial sums are added in
// double. The accumulator layout of S is the A-operand layout of P, so P
// stays in registers. One CTA of four warps per (head, image), warp w owning
// query rows 16w..16w+15; K and V are staged once per CTA as fp16 [key][dim]
// planes (two pieces each) with the 16-byte chunks of a key row
// XOR-swizzled by the key (conflict-free ldmatrix), 32 KB: five CTAs per SM.
// Keys T..63 are zero rows, masked out of the softmax.
constexpr int MHAM_T = 64;

// two floats -> one register of fp16 halves, a in the low 16 bits
__device__ __forceinline__ uint32_t mham_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// (x0, x1) -> NP packed fp16 pieces, x0 in the low 16 bits of each. Every
// piece but the last is x rounded to 11 significant bits (to_tf32's integer
// rounding: 11 bits are fp16's precision, so the conversion is exact) and the
// residual x - piece is an exact fp32 subtraction; the last piece is the
// residual rounded to fp16. Pieces below fp16's normal range (2^-14, 2^-28 of
// a block's largest magnitude) take fp16's subnormal rounding, an error of at
// most 2^-25.
template <int NP>
__device__ __forceinline__ void mham_split(float x0, float x1, uint32_t (&pc)[NP])
{
#pragma unroll
    for (int i = 0; i + 1 < NP; i++) {
        const float h0 = to_tf32(x0), h1 = to_tf32(x1);
        pc[i] = mham_h2(h0, h1);
        x0 = __fsub_rn(x0, h0);
        x1 = __fsub_rn(x1, h1);
    }
    pc[NP - 1] = mham_h2(x0, x1);
}

// e with m * 2^e in [2^14, 2^15) for a finite m > 0, at most 100; 0 when m is
// 0 or not finite.
__device__ __forceinline__ int mham_exp(float m)
{
    const int E = (__float_as_int(m) >> 23) & 0xff;
    if (m == 0.0f || E == 0xff) return 0;
    return min(141 - E, 100);
}

__device__ __forceinline__ float mham_pow2(int e) { return __int_as_float((127 + e) << 23); }   // |e| <= 126

__device__ __forceinline__ void mham_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mham_ldsm(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

__device__ __forceinline__ void mham_ldsm_t(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

__device__ __forceinline__ void put2(const OutSpec &o, size_t row, int col, float a, float b)
{
    const size_t i = row * (size_t)o.ld + col;
    if (o.plain) *reinterpret_cast<float2 *>(o.plain + i) = make_float2(a, b);
    if (o.hi) {
        float ha, la, hb, lb;
        split_tf32(a, ha, la);
        split_tf32(b, hb, lb);
        *reinterpret_cast<float2 *>(o.hi + i) = make_float2(ha, hb);
        *reinterpret_cast<float2 *>(o.lo + i) = make_float2(la, lb);
    }
}

// byte offset of (key, 16-byte chunk) in a swizzled [64][64] fp16 plane
__device__ __forceinline__ uint32_t mham_off(int key, int chunk)
{
    return (uint32_t)(key * 128 + ((chunk ^ (key & 7)) << 4));
}

__global__ void __launch_bounds__(128, 5)
mha64m_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int ldi,
              int T, OutSpec out)
{
    pdl_wait();
    constexpr int NQK = 2;                              // pieces of Q and K
    constexpr uint32_t PLANE = MHAM_T * 64 * 2;
    __shared__ __align__(128) __half kv[NQK + 2][MHAM_T * 64];    // K's NQK pieces, V's two
    __shared__ float red[2][4];
    const int col = blockIdx.x * 64;
    const size_t base = (size_t)blockIdx.y * T;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int t4 = lane & 3;
    const float2 z2 = make_float2(0.f, 0.f);
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);

    // K and V: step it covers element i = thread + 128 it, key i >> 4, dims 4 (i & 15)..
    float4 xk[8], xv[8];
#pragma unroll
    for (int it = 0; it < 8; it++) {
        const int i = threadIdx.x + 128 * it, key = i >> 4, d = col + 4 * (i & 15);
        xk[it] = key < T ? __ldg(reinterpret_cast<const float4 *>(k + (base + key) * (size_t)ldi + d)) : z4;
        xv[it] = key < T ? __ldg(reinterpret_cast<const float4 *>(v + (base + key) * (size_t)ldi + d)) : z4;
    }
    float mk = 0.f, mv = 0.f;
#pragma unroll
    for (int it = 0; it < 8; it++) {
        mk = fmaxf(mk, fmaxf(fmaxf(fabsf(xk[it].x), fabsf(xk[it].y)), fmaxf(fabsf(xk[it].z), fabsf(xk[it].w))));
        mv = fmaxf(mv, fmaxf(fmaxf(fabsf(xv[it].x), fabsf(xv[it].y)), fmaxf(fabsf(xv[it].z), fabsf(xv[it].w))));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
        mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
    }
    if (lane == 0) {
        red[0][wid] = mk;
        red[1][wid] = mv;
    }
    __syncthreads();
    mk = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
    mv = fmaxf(fmaxf(red[1][0], red[1][1]), fmaxf(red[1][2], red[1][3]));
    const int ek = mham_exp(mk), ev = mham_exp(mv);
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(&kv[0][0]);
    // K's pieces first; then this warp's query rows are requested (their
    // latency overlaps V's pieces) straight into A-operand order: xq[kk][0]
    // row r0, dims 16kk + 2t4 + {0,1}; [1] row r1, same dims; [2] and [3]
    // the dims 8 further on.
    {
        const float fk = mham_pow2(ek);
#pragma unroll
        for (int it = 0; it < 8; it++) {
            const int i = threadIdx.x + 128 * it, key = i >> 4, c4 = i & 15;
            const uint32_t off = mham_off(key, c4 >> 1) + 8 * (c4 & 1);
            uint32_t a[NQK], b[NQK];
            mham_split<NQK>(__fmul_rn(xk[it].x, fk), __fmul_rn(xk[it].y, fk), a);
            mham_split<NQK>(__fmul_rn(xk[it].z, fk), __fmul_rn(xk[it].w, fk), b);
#pragma unroll
            for (int pc = 0; pc < NQK; pc++)
                asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(s0 + pc * PLANE + off), "r"(a[pc]), "r"(b[pc]));
        }
    }
    const int r0 = 16 * wid + (lane >> 2), r1 = r0 + 8;
    float2 xq[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const int d = col + 16 * kk + 2 * t4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = (i & 1) ? r1 : r0;
            xq[kk][i] = r < T ? __ldg(reinterpret_cast<const float2 *>(q + (base + r) * (size_t)ldi + d + 4 * (i & 2)))
                              : z2;
        }
    }
    {
        const float fv = mham_pow2(ev);
#pragma unroll
        for (int it = 0; it < 8; it++) {
            const int i = threadIdx.x + 128 * it, key = i >> 4, c4 = i & 15;
            const uint32_t off = mham_off(key, c4 >> 1) + 8 * (c4 & 1);
            uint32_t c[2], e[2];
            mham_split<2>(__fmul_rn(xv[it].x, fv), __fmul_rn(xv[it].y, fv), c);
            mham_split<2>(__fmul_rn(xv[it].z, fv), __fmul_rn(xv[it].w, fv), e);
#pragma unroll
            for (int pc = 0; pc < 2; pc++)
                asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(s0 + (NQK + pc) * PLANE + off), "r"(c[pc]), "r"(e[pc]));
        }
    }
    __syncthreads();
    if (16 * wid >= T) return;                          // no later barrier

    // Q: one scale per row (a row's 64 dims sit in the four lanes of a quad)
    float m0 = 0.f, m1 = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        m0 = fmaxf(m0, fmaxf(fmaxf(fabsf(xq[kk][0].x), fabsf(xq[kk][0].y)), fmaxf(fabsf(xq[kk][2].x), fabsf(xq[kk][2].y))));
        m1 = fmaxf(m1, fmaxf(fmaxf(fabsf(xq[kk][1].x), fabsf(xq[kk][1].y)), fmaxf(fabsf(xq[kk][3].x), fabsf(xq[kk][3].y))));
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    const int eq0 = mham_exp(m0), eq1 = mham_exp(m1);
    uint32_t qa[NQK][4][4];                             // [piece][kk][A register]
    {
        const float f0 = mham_pow2(eq0), f1 = mham_pow2(eq1);
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float f = (i & 1) ? f1 : f0;
                uint32_t pc[NQK];
                mham_split<NQK>(__fmul_rn(xq[kk][i].x, f), __fmul_rn(xq[kk][i].y, f), pc);
#pragma unroll
                for (int x = 0; x < NQK; x++) qa[x][kk][i] = pc[x];
            }
    }

    // S = Q K^T: key block j (8 keys), dims 32p..32p+31 per ldmatrix; the
    // blocks are independent accumulators, the j loop inside keeps eight
    // (seven for T <= 56) of them in flight. Pass 0: the cross products over
    // all 64 dims; pass 1: the four p1 k1 steps.
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const bool blk7 = T > 56;
#pragma unroll
    for (int pass = 0; pass < 2; pass++)
#pragma unroll
        for (int p = 0; p < 2; p++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j == 7 && !blk7) break;
                const uint32_t off = mham_off(8 * j + (lane & 7), 4 * p + (lane >> 3));
                uint32_t bk[NQK][4];
                if (pass == 0) {
#pragma unroll
                    for (int x = 0; x < NQK; x++) mham_ldsm(s0 + x * PLANE + off, bk[x]);
                } else {
                    mham_ldsm(s0 + off, bk[0]);
                }
#pragma unroll
                for (int h = 0; h < 2; h++) {           // kk = 2p + h: B registers 2h, 2h + 1
                    const int kk = 2 * p + h, x = 2 * h, y = 2 * h + 1;
                    if (pass == 0) {
                        mham_mma(s[j], qa[0][kk], bk[1][x], bk[1][y]);
                        mham_mma(s[j], qa[1][kk], bk[0][x], bk[0][y]);
                    } else {
                        mham_mma(s[j], qa[0][kk], bk[0][x], bk[0][y]);
                    }
                }
            }

    // softmax of rows r0 (s[j][0..1]) and r1 (s[j][2..3]); key 8j + 2t4 + c.
    // Undoing the scales and multiplying by 1/sqrt(64) = 2^-3 are exact, so
    // one multiply by 2^-(eq + ek + 3) gives the same bits as the three
    // whenever that power of two is a normal float.
    const int E0 = eq0 + ek + 3, E1 = eq1 + ek + 3;
    if (abs(E0) <= 126 && abs(E1) <= 126) {
        const float g0 = mham_pow2(-E0), g1 = mham_pow2(-E1);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            s[j][0] = __fmul_rn(s[j][0], g0);
            s[j][1] = __fmul_rn(s[j][1], g0);
            s[j][2] = __fmul_rn(s[j][2], g1);
            s[j][3] = __fmul_rn(s[j][3], g1);
        }
    } else {
        const float scale = 1.0f / sqrtf(64.0f);
        const float uk = mham_pow2(-ek), u0 = mham_pow2(-eq0), u1 = mham_pow2(-eq1);
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                s[j][c] = __fmul_rn(__fmul_rn(__fmul_rn(s[j][c], u0), uk), scale);
                s[j][2 + c] = __fmul_rn(__fmul_rn(__fmul_rn(s[j][2 + c], u1), uk), scale);
            }
    }
    const int jfull = T >> 3;                           // key blocks 0..jfull-1 hold no key past T
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (j < jfull || 8 * j + 2 * t4 + c < T) {
                mx0 = fmaxf(mx0, s[j][c]);
                mx1 = fmaxf(mx1, s[j][2 + c]);
            }
        }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const bool in = j < jfull || 8 * j + 2 * t4 + c < T;
            s[j][c] = in ? expf(__fsub_rn(s[j][c], mx0)) : 0.0f;
            s[j][2 + c] = in ? expf(__fsub_rn(s[j][2 + c], mx1)) : 0.0f;
            ps0 = __fadd_rn(ps0, s[j][c]);
            ps1 = __fadd_rn(ps1, s[j][2 + c]);
        }
    double sum0 = ps0, sum1 = ps1;
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, o);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, o);
    }
    const float inv0 = (float)(1.0 / sum0), inv1 = (float)(1.0 / sum1);
    // e * inv * 2^14 == e * (inv * 2^14): scaling by a power of two is exact
    const float w0 = __fmul_rn(inv0, 16384.0f), w1 = __fmul_rn(inv1, 16384.0f);

    // P (times 2^14) as two pieces in A order: k-step kk covers key blocks 2kk, 2kk+1
    uint32_t pa[2][4][4];
#pragma unroll
    for (int kk = 0; kk < 4; kk++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float(&sj)[4] = s[2 * kk + (i >> 1)];
            const float w = (i & 1) ? w1 : w0;
            const int c = 2 * (i & 1);
            uint32_t pc[2];
            mham_split<2>(__fmul_rn(sj[c], w), __fmul_rn(sj[c + 1], w), pc);
            pa[0][kk][i] = pc[0];
            pa[1][kk][i] = pc[1];
        }

    // O = P V: n-blocks 2np, 2np+1 from one transposed ldmatrix per piece;
    // pass 0: the cross products p1 v2 and p2 v1 over all keys; pass 1: the
    // p1 v1 steps.
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    const int nk = (T + 15) >> 4;
#pragma unroll
    for (int pass = 0; pass < 2; pass++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            if (kk >= nk) break;
            const int m = lane >> 3, key = 16 * kk + 8 * (m & 1) + (lane & 7);
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t v1[4], v2[4];
                const uint32_t off = mham_off(key, 2 * np + (m >> 1));
                mham_ldsm_t(s0 + NQK * PLANE + off, v1);
                if (pass == 0) {
                    mham_ldsm_t(s0 + (NQK + 1) * PLANE + off, v2);
                    mham_mma(o[2 * np], pa[0][kk], v2[0], v2[1]);
                    mham_mma(o[2 * np], pa[1][kk], v1[0], v1[1]);
                    mham_mma(o[2 * np + 1], pa[0][kk], v2[2], v2[3]);
                    mham_mma(o[2 * np + 1], pa[1][kk], v1[2], v1[3]);
                } else {
                    mham_mma(o[2 * np], pa[0][kk], v1[0], v1[1]);
                    mham_mma(o[2 * np + 1], pa[0][kk], v1[2], v1[3]);
                }
            }
        }
    const float uo = mham_pow2(-(14 + ev));
#pragma unroll
    for (int n = 0; n < 8; n++) {
        const int c = col + 8 * n + 2 * t4;
        if (r0 < T) put2(out, base + r0, c, __fmul_rn(o[n][0], uo), __fmul_rn(o[n][1], uo));
        if (r1 < T) put2(out, base + r1, c, __fmul_rn(o[n][2], uo), __fmul_rn(o[n][3], uo));
    }
}

static size_t mha64_smem(int T)
{
    const size_t T4 = (size_t)((T + 3) & ~3);
    return (MHA_BQ * 64 + 3 * 64 * T4) * sizeof(float);
}

// T > 64: 1 (default) tensor cores where 128 <= T <= 1024, else the streaming kernel with 64-query blocks;
// 0 whole-K/V kernel; 2 streaming kernel with 48-query blocks; 3 tensor cores where they apply
int g_mha_variant = 1;
// head_dim 64, T <= 64: 1 (default) fp16-split tensor cores (mha64m_kernel); 0 fp32 FMA (mha64s_kernel)
int g_mha_short = 1;

bool launch_mha(const float *q, const float *k, const float *v, int ldi, int T, int n_head, int hd,
                int n_img, const OutSpec &out, cudaStream_t s)
{
    if (T <= 0 || n_img <= 0 || n_head <= 0) return true;
    if (hd <= 0 || hd > 128) return fail("attention: head_dim %d outside 1..128", hd);
    const bool aligned = !(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) && !(ldi & 3) &&
                         !(out.ld & 3) && !(((uintptr_t)out.plain | (uintptr_t)out.hi | (uintptr_t)out.lo) & 15);
    if (hd == 64 && aligned && T <= MHAS_T) {
        dim3 grid(n_head, n_img);
        if (g_mha_short == 1) TCG_CUDA(launch_pdl(mha64m_kernel, grid, 128, 0, s, q, k, v, ldi, T, out));
        else TCG_CUDA(launch_pdl(mha64s_kernel, grid, 256, 0, s, q, k, v, ldi, T, out));
        TCG_LAUNCHED();
        return true;
    }
    if (hd == 64 && aligned && (g_mha_variant == 3 || g_mha_variant == 1) &&
        launch_mha64_tc_long(q, k, v, ldi, T, n_head, n_img, out, s))
        return true;
    if (hd == 64 && aligned && g_mha_variant != 0) {
        const bool q48 = g_mha_variant == 2;
        // variant 1 here: T < 128 or T > 1024; variant 3 here: the tensor-core kernel did not apply
        const size_t sm = q48 ? mhb_smem<48>(T) : mhb_smem<64>(T);
        if (sm <= 227 * 1024) {
            static unsigned doneb[64];
            const int dev = ctx().device & 63, bit = q48 ? 2 : 1;
            if (!(doneb[dev] & bit)) {
                TCG_CUDA(cudaFuncSetAttribute(q48 ? mha64b_kernel<48> : mha64b_kernel<64>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
                doneb[dev] |= bit;
            }
            const int bq = q48 ? 48 : 64;
            dim3 grid(n_head, n_img, (T + bq - 1) / bq);
            if (q48) TCG_CUDA(launch_pdl(mha64b_kernel<48>, grid, 192, sm, s, q, k, v, ldi, T, out));
            else TCG_CUDA(launch_pdl(mha64b_kernel<64>, grid, 256, sm, s, q, k, v, ldi, T, out));
            TCG_LAUNCHED();
            return true;
        }
    }
    if (hd == 64 && aligned && mha64_smem(T) <= 227 * 1024) {
        static unsigned done64[64];
        const int dev = ctx().device & 63;
        if (!done64[dev]) {
            TCG_CUDA(cudaFuncSetAttribute(mha64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
            done64[dev] = 1;
        }
        dim3 grid(n_head, n_img, (T + MHA_BQ - 1) / MHA_BQ);
        TCG_CUDA(launch_pdl(mha64_kernel, grid, 256, mha64_smem(T), s, q, k, v, ldi, T, out));
        TCG_LAUNCHED();
        return true;
    }
    const int nw = 8;
    const size_t smem = ((size_t)T * (2 * hd + 1) + (size_t)nw * (T + hd)) * sizeof(float);
    if (smem > 227 * 1024) return fail("attention: T=%d head_dim=%d needs %zu B of shared memory", T, hd, smem);
    dim3 grid(n_head, n_img);
    // Opt every variant in to the full shared-memory window once per device.
    static unsigned attr_done[64];
    const int dev = ctx().device & 63;
    if (!attr_done[dev]) {
        const int maxsm = 227 * 1024;
        TCG_CUDA(cudaFuncSetAttribute(mha_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxsm));
        TCG_CUDA(cudaFuncSetAttribute(mha_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxsm));
        TCG_CUDA(cudaFuncSetAttribute(mha_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxsm));
        attr_done[dev] = 1;
    }
    if (hd <= 32) TCG_CUDA(launch_pdl(mha_kernel<1>, grid, nw * 32, smem, s, q, k, v, ldi, T, hd, out));
    else if (hd <= 64) TCG_CUDA(launch_pdl(mha_kernel<2>, grid, nw * 32, smem, s, q, k, v, ldi, T, hd, out));
    else TCG_CUDA(launch_pdl(mha_kernel<4>, grid, nw * 32, smem, s, q, k, v, ldi, T, hd, out));
    TCG_LAUNCHED();
    return true;
}

// ------------------------------------------------------------ SIMT GEMM
// 64x64 tile, 16-deep K slices in shared memory, 4x4 outputs per thread,
// fp32 FMA accumulation in increasing k.
constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

__global__ void __launch_bounds__(256)
gemm_simt_kernel(float *__restrict__ C, int ldc, const float *__restrict__ A, int lda,
                 const float *__restrict__ B, int ldb, const float *__restrict__ bias,
                 int M, int N, int K, bool bt)
{
    __shared__ float As[SG_BK][SG_BM + 4];
    __shared__ float Bs[SG_BK][SG_BN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += SG_BK) {
        for (int i = threadIdx.x; i < SG_BM * SG_BK; i += 256) {
            const int r = i / SG_BK, kk = i % SG_BK;
            const int m = m0 + r, kg = k0 + kk;
            As[kk][r] = (m < M && kg < K) ? A[(size_t)m * lda + kg] : 0.0f;
        }
        for (int i = threadIdx.x; i < SG_BN * SG_BK; i += 256) {
            int r, kk;
            if (bt) { r = i / SG_BK; kk = i % SG_BK; } else { kk = i / SG_BN; r = i % SG_BN; }
            const int n = n0 + r, kg = k0 + kk;
            float val = 0.0f;
            if (n < N && kg < K) val = bt ? B[(size_t)n * ldb + kg] : B[(size_t)kg * ldb + n];
            Bs[kk][r] = val;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < SG_BK; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx * 4 + j;
            if (n < N) C[(size_t)m * ldc + n] = bias ? __fadd_rn(acc[i][j], bias[n]) : acc[i][j];
        }
    }
}

bool launch_gemm_simt(float *C, int ldc, const float *A, int lda, const float *B, int ldb,
                      const float *bias, int M, int N, int K, bool bt, cudaStream_t s)
{
    if (M <= 0 || N <= 0) return true;
    dim3 grid(ceil_div(N, SG_BN), ceil_div(M, SG_BM));
    gemm_simt_kernel<<<grid, 256, 0, s>>>(C, ldc, A, lda, B, ldb, bias, M, N, K, bt);
    TCG_LAUNCHED();
    return true;
}

// ------------------------------------------------------------ elementwise

__global__ void split_kernel(const float *__restrict__ src, float *__restrict__ hi, float *__restrict__ lo, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float h, l;
        split_tf32(src[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

static unsigned grid1d(size_t n)
{
    const size_t need = (n + 255) / 256, cap = (size_t)ctx().sms * 16;
    return (unsigned)(need < cap ? (need ? need : 1) : cap);
}

bool launch_split(const float *src, float *hi, float *lo, size_t n, cudaStream_t s)
{
    if (n == 0) return true;
    split_kernel<<<grid1d(n), 256, 0, s>>>(src, hi, lo, n);
    TCG_LAUNCHED();
    return true;
}

// Patch row r = i*G*G + gy*G + gx, column c = ch*P*P + ky*P + kx holds
// pixel [i, ch, gy*P + ky, gx*P + kx]. A patch row's kx run is contiguous in
// the image, so each thread moves VEC consecutive floats (VEC | P).
template <int VEC>
__global__ void patches_kernel(const float *__restrict__ px, int n_img, int S, int P,
                               float *__restrict__ hi, float *__restrict__ lo)
{
    pdl_wait();
    typedef typename std::conditional<VEC == 4, float4, typename std::conditional<VEC == 2, float2, float>::type>::type V;
    const int G = S / P, PV = P / VEC, KPV = 3 * P * PV;          // vectors per patch row
    const size_t total = (size_t)n_img * G * G * KPV;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / KPV;
        const int c = (int)(i - r * KPV);                  // vector index within the row
        const int img = (int)(r / (G * G)), t = (int)(r % (G * G));
        const int gy = t / G, gx = t % G;
        const int ch = c / (P * PV), rem = c % (P * PV), ky = rem / PV, kv = rem % PV;
        const V v = *reinterpret_cast<const V *>(px + (((size_t)img * 3 + ch) * S + gy * P + ky) * S + gx * P + kv * VEC);
        const float *f = reinterpret_cast<const float *>(&v);
        if (!lo) {                                          // plain fp32 rows
            reinterpret_cast<V *>(hi)[i] = v;
            continue;
        }
        V h, l;
        float *hf = reinterpret_cast<float *>(&h), *lf = reinterpret_cast<float *>(&l);
#pragma unroll
        for (int j = 0; j < VEC; j++) split_tf32(f[j], hf[j], lf[j]);
        reinterpret_cast<V *>(hi)[i] = h;
        reinterpret_cast<V *>(lo)[i] = l;
    }
}

// One warp per row of W: its 2-norm (and |b| of the row) into bounds by an
// integer max on the bit patterns (non-negative floats order as integers).
__global__ void weight_bounds_kernel(const float *__restrict__ W, int rows, int K, const float *__restrict__ b,
                                     float *bounds)
{
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    float ss = 0.0f;
    for (int k = lane; k < K; k += 32) ss = fmaf(W[(size_t)row * K + k], W[(size_t)row * K + k], ss);
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    if (lane == 0) {
        atomicMax(reinterpret_cast<int *>(bounds), __float_as_int(sqrtf(ss)));
        if (b) atomicMax(reinterpret_cast<int *>(bounds) + 1, __float_as_int(fabsf(b[row])));
    }
}

bool launch_weight_bounds(const float *W, int rows, int K, const float *b, float *bounds, cudaStream_t s)
{
    if (rows <= 0) return true;
    weight_bounds_kernel<<<ceil_div(rows, 8), 256, 0, s>>>(W, rows, K, b, bounds);
    TCG_LAUNCHED();
    return true;
}

bool launch_patches(const float *px, int n_img, int S, int P, float *hi, float *lo, cudaStream_t s)
{
    const size_t total = (size_t)n_img * (S / P) * (S / P) * 3 * P * P;
    if (total == 0) return true;
    const bool a16 = !(((uintptr_t)px | (uintptr_t)hi | (uintptr_t)lo) & 15) && !(S & 3);
    const bool a8 = !(((uintptr_t)px | (uintptr_t)hi | (uintptr_t)lo) & 7) && !(S & 1);
    if (P % 4 == 0 && a16) TCG_CUDA(launch_pdl(patches_kernel<4>, grid1d(total / 4), 256, 0, s, px, n_img, S, P, hi, lo));
    else if (P % 2 == 0 && a8) TCG_CUDA(launch_pdl(patches_kernel<2>, grid1d(total / 2), 256, 0, s, px, n_img, S, P, hi, lo));
    else TCG_CUDA(launch_pdl(patches_kernel<1>, grid1d(total), 256, 0, s, px, n_img, S, P, hi, lo));
    TCG_LAUNCHED();
    return true;
}

// dst_hi/lo [C, R] = tf32 pair of src [R, C] transposed.
__global__ void transpose_split_kernel(const float *__restrict__ src, int R, int C,
                                       float *__restrict__ hi, float *__restrict__ lo)
{
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < C) tile[i][threadIdx.x] = src[(size_t)r * C + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < C) {
            float h, l;
            split_tf32(tile[threadIdx.x][i], h, l);
            hi[(size_t)c * R + r] = h;
            lo[(size_t)c * R + r] = l;
        }
    }
}

bool launch_transpose_split(const float *src, int R, int C, float *hi, float *lo, cudaStream_t s)
{
    if (R <= 0 || C <= 0) return true;
    transpose_split_kernel<<<dim3(ceil_div(C, 32), ceil_div(R, 32)), dim3(32, 8), 0, s>>>(src, R, C, hi, lo);
    TCG_LAUNCHED();
    return true;
}

__global__ void cls_rows_kernel(float *__restrict__ x, const float *__restrict__ cls,
                                const float *__restrict__ pos, int n_img, int T, int D)
{
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_img * D; i += gridDim.x * blockDim.x) {
        const int img = i / D, d = i % D;
        x[(size_t)img * T * D + d] = __fadd_rn(cls[d], pos[d]);
    }
}

bool launch_cls_rows(float *x, const float *cls, const float *pos, int n_img, int T, int D, cudaStream_t s)
{
    if (n_img <= 0) return true;
    TCG_CUDA(launch_pdl(cls_rows_kernel, grid1d((size_t)n_img * D), 256, 0, s, x, cls, pos, n_img, T, D));
    TCG_LAUNCHED();
    return true;
}

__global__ void gelu_kernel(float *__restrict__ out, const float *__restrict__ x, size_t n, bool quick)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = quick ? gelu_quick(x[i]) : gelu_exact(x[i]);
}

bool launch_gelu(float *out, const float *x, size_t n, bool quick, cudaStream_t s)
{
    if (n == 0) return true;
    gelu_kernel<<<grid1d(n), 256, 0, s>>>(out, x, n, quick);
    TCG_LAUNCHED();
    return true;
}

__global__ void softmax_kernel(float *__restrict__ out, const float *__restrict__ x, int rows, int cols)
{
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *in = x + (size_t)row * cols;
    float *o = out + (size_t)row * cols;
    float mx = -INFINITY;
    for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, in[c]);
    mx = warp_max(mx);
    double sum = 0.0;
    for (int c = lane; c < cols; c += 32) {
        const float e = expf(__fsub_rn(in[c], mx));
        o[c] = e;
        sum += (double)e;
    }
    const float inv = (float)(1.0 / warp_sum(sum));
    for (int c = lane; c < cols; c += 32) o[c] = __fmul_rn(o[c], inv);
}

__global__ void add_kernel(float *__restrict__ out, const float *a, const float *b, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

__global__ void scale_kernel(float *__restrict__ out, const float *x, float s, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(x[i], s);
}

}  // namespace tcg

using namespace tcg;

extern "C" {

bool tcg_layernorm(float *out, const float *x, const float *gamma, const float *beta, int rows, int cols, float eps)
{
    if (!need_ctx()) return false;
    if (rows < 0 || cols <= 0) return rows == 0 || cols == 0 ? true : fail("tcg_layernorm: bad shape");
    OutSpec o;
    o.plain = out;
    o.ld = cols;
    return launch_layernorm(x, cols, gamma, beta, rows, cols, eps, o, ctx().cur);
}

// LayerNorm into fp16 pieces (the kind::f16 GEMM's A operand): hi, lo
// [rows, cols] fp16, ex [cols / 256, rows] one exponent per 256-column block,
// rnorm [rows] each output row's 2-norm (may be null).
bool tcg_layernorm_f16(void *hi, void *lo, int8_t *ex, float *rnorm, const float *x, const float *gamma,
                       const float *beta, int rows, int cols, float eps)
{
    if (!need_ctx()) return false;
    if (rows <= 0 || cols <= 0) return rows == 0 || cols == 0 ? true : fail("tcg_layernorm_f16: bad shape");
    OutSpec o;
    o.fh = hi;
    o.fl = lo;
    o.fe = ex;
    o.fe_rows = rows;
    o.rnorm = rnorm;
    o.ld = cols;
    return launch_layernorm(x, cols, gamma, beta, rows, cols, eps, o, ctx().cur);
}

// bounds[0] = max over rows of ||W[row]||_2, bounds[1] = max |b| (W [rows, K],
// b may be null); overwrites bounds.
bool tcg_weight_bounds(float *bounds, const float *W, int rows, int K, const float *b)
{
    if (!need_ctx()) return false;
    TCG_CUDA(cudaMemsetAsync(bounds, 0, 2 * sizeof(float), ctx().cur));
    return launch_weight_bounds(W, rows, K, b, bounds, ctx().cur);
}

bool tcg_gelu(float *out, const float *x, size_t n)
{
    return need_ctx() && launch_gelu(out, x, n, false, ctx().cur);
}

bool tcg_gelu_quick(float *out, const float *x, size_t n)
{
    return need_ctx() && launch_gelu(out, x, n, true, ctx().cur);
}

bool tcg_softmax_rows(float *out, const float *x, int rows, int cols)
{
    if (!need_ctx()) return false;
    if (rows <= 0 || cols <= 0) return true;
    softmax_kernel<<<ceil_div(rows, 8), 256, 0, ctx().cur>>>(out, x, rows, cols);
    TCG_LAUNCHED();
    return true;
}

bool tcg_mha(float *out, const float *q, const float *k, const float *v, int T, int n_head, int head_dim)
{
    if (!need_ctx()) return false;
    OutSpec o;
    o.plain = out;
    o.ld = n_head * head_dim;
    return launch_mha(q, k, v, n_head * head_dim, T, n_head, head_dim, 1, o, ctx().cur);
}

bool tcg_mha_images(float *out, float *out_hi, float *out_lo, const float *qkv, int T, int n_head, int head_dim,
                    int n_img)
{
    if (!need_ctx()) return false;
    if ((out_hi == nullptr) != (out_lo == nullptr)) return fail("attention: out_hi and out_lo go together");
    if (!out && !out_hi) return fail("attention: no output");
    const int D = n_head * head_dim;
    OutSpec o;
    o.plain = out;
    o.hi = out_hi;
    o.lo = out_lo;
    o.ld = D;
    return launch_mha(qkv, qkv + D, qkv + 2 * D, 3 * D, T, n_head, head_dim, n_img, o, ctx().cur);
}

bool tcg_add(float *out, const float *a, const float *b, size_t n)
{
    if (!need_ctx()) return false;
    if (n == 0) return true;
    add_kernel<<<grid1d(n), 256, 0, ctx().cur>>>(out, a, b, n);
    TCG_LAUNCHED();
    return true;
}

bool tcg_scale(float *out, const float *x, float s, size_t n)
{
    if (!need_ctx()) return false;
    if (n == 0) return true;
    scale_kernel<<<grid1d(n), 256, 0, ctx().cur>>>(out, x, s, n);
    TCG_LAUNCHED();
    return true;
}

}  // extern "C"

// Tuning and test hook: the attention kernel for head_dim 64 and T > 64
// (1, the default: tensor cores where 128 <= T <= 1024, else streamed K/V with
// 64-query blocks; 0: whole K/V in shared memory; 2: streamed K/V with
// 48-query blocks; 3: tensor cores only). Returns the previous setting.
extern "C" int tcg_set_attention_variant(int variant)
{
    const int old = tcg::g_mha_variant;
    tcg::g_mha_variant = variant < 0 ? 0 : (variant > 3 ? 3 : variant);
    return old;
}

// Tuning and test hook: the attention kernel for head_dim 64 and T <= 64
// (1, the default: fp16 two-piece operands on mma.sync; 0: fp32 FMA). Returns the
// previous setting.
extern "C" int tcg_set_attention_short_kernel(int kernel)
{
    const int old = tcg::g_mha_short;
    tcg::g_mha_short = kernel ? 1 : 0;
    return old;
}

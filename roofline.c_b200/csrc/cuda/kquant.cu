// kquant.cu -- the dequant seam on the GPU (roofline.c src/dequant.c:5-80,
// with the Q4_K / Q6_K arms of ggml's block formats) and the fused K-quant
// dequant-matvec.
//
// Layout of one warp's work: a group of 8 superblocks (1152 B of Q4_K or
// 1680 B of Q6_K, both multiples of 16 B) is copied global -> shared with
// 128-bit loads, then every lane decodes 8 consecutive weights of each
// superblock (lane l owns weights 8l..8l+7) and writes them as two float4.
// Arithmetic is the rounding sequence of the C restatement with no
// contraction: Q4_K w = (d*sc)*q - (dmin*m), Q6_K w = (d*sc)*q.
#include "tcg_common.cuh"
#include "tcg_internal.h"

#include <string.h>

namespace tcg {

constexpr int QK = 256;
constexpr int GROUP = 8;          // superblocks staged per warp
constexpr int WARPS = 8;          // warps per CTA

template <int TYPE> struct KQ;
template <> struct KQ<GGML_TYPE_Q4_K> { static constexpr int BYTES = 144; };
template <> struct KQ<GGML_TYPE_Q6_K> { static constexpr int BYTES = 210; };

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

template <int TYPE>
__global__ void __launch_bounds__(WARPS * 32)
dequant_kq_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst, size_t nblocks)
{
    constexpr int BB = KQ<TYPE>::BYTES;
    __shared__ __align__(16) uint8_t buf[WARPS][GROUP * BB];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const size_t ngroups = (nblocks + GROUP - 1) / GROUP;
    for (size_t grp = (size_t)blockIdx.x * WARPS + wid; grp < ngroups; grp += (size_t)gridDim.x * WARPS) {
        const size_t b0 = grp * GROUP;
        const int nb = (int)min((size_t)GROUP, nblocks - b0);
        stage(buf[wid], src + b0 * BB, nb * BB, lane);
        __syncwarp();
        for (int b = 0; b < nb; b++) {
            float w[8];
            decode8<TYPE>(buf[wid] + b * BB, lane, w);
            float4 *o = reinterpret_cast<float4 *>(dst + (b0 + b) * QK + 8 * lane);
            o[0] = make_float4(w[0], w[1], w[2], w[3]);
            o[1] = make_float4(w[4], w[5], w[6], w[7]);
        }
        __syncwarp();
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
    TCG_LAUNCHED();
    return true;
}

template <int TYPE>
static bool matvec_dispatch(float *y, const void *W, const float *x, int N, int K)
{
    // Enough warps to keep ~48 resident per SM streaming weight bytes.
    const long want = (long)ctx().sms * 48;
    if ((long)N >= want) return launch_matvec<TYPE, 1>(y, W, x, N, K);
    if ((long)N * 2 >= want) return launch_matvec<TYPE, 2>(y, W, x, N, K);
    if ((long)N * 4 >= want) return launch_matvec<TYPE, 4>(y, W, x, N, K);
    return launch_matvec<TYPE, 8>(y, W, x, N, K);
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

// numerics.cuh -- device arithmetic whose rounding sequence follows the
// reference's scalar C (src/ops.c), written with explicit _rn intrinsics so
// nvcc cannot contract it into FMAs.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tcg {

// Round-to-nearest (ties away) to tf32: the 10-bit-mantissa value the tensor
// core consumes, returned as an fp32 bit pattern with the low 13 bits zero.
// Integer arithmetic on the sign-magnitude pattern: half a tf32 ulp (bit 12)
// is added to the magnitude and the 13 low bits dropped, so a carry rounds
// the magnitude up (ties included, away from zero) and may step the exponent;
// the same bits as cvt.rna.tf32.f32 for every finite v, without occupying the
// conversion unit that kernels writing hi/lo pairs would otherwise queue on.
__device__ __forceinline__ float to_tf32(float v)
{
    return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xffffe000u);
}

// v = hi + lo + O(2^-22 |v|): the operand split of 3xTF32.
__device__ __forceinline__ void split_tf32(float v, float &hi, float &lo)
{
    hi = to_tf32(v);
    lo = to_tf32(__fsub_rn(v, hi));
}

// The power-of-two exponent e that puts a block whose largest magnitude is m
// in [2^14, 2^15) (inside fp16's normal range), kept in [-63, 63] so that a
// product's unscaling 2^-(ea + eb) is one normal float; 0 when m is 0 or not
// finite.
__device__ __forceinline__ int f16_scale_exp(float m)
{
    const int E = (__float_as_int(m) >> 23) & 0xFF;
    return (m == 0.0f || E == 0xFF) ? 0 : max(-63, min(141 - E, 63));
}

// Four values times f (a power of two) as fp16 pieces: p1 = the value
// rounded to 11 significant bits (exact in fp16), p2 = fp16(value - p1),
// packed four to a uint2 (element 0 in the low half).
__device__ __forceinline__ void f16_pieces4(const float (&v)[4], float f, uint2 &hi, uint2 &lo)
{
    uint32_t h[2], l[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float x0 = __fmul_rn(v[2 * i], f), x1 = __fmul_rn(v[2 * i + 1], f);
        const float p0 = to_tf32(x0), p1 = to_tf32(x1);
        const __half2 a = __floats2half2_rn(p0, p1);
        const __half2 b = __floats2half2_rn(__fsub_rn(x0, p0), __fsub_rn(x1, p1));
        h[i] = *reinterpret_cast<const uint32_t *>(&a);
        l[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
    hi = make_uint2(h[0], h[1]);
    lo = make_uint2(l[0], l[1]);
}

// 0.5f * x * (1.0f + erff(x * (1/sqrt 2)))  -- src/ops.c:82-87
__device__ __forceinline__ float gelu_exact(float x)
{
    const float inv_sqrt2 = 0.70710678118654752440f;
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, inv_sqrt2))));
}

// x / (1.0f + expf(-1.702f * x))  -- src/ops.c:89-93
__device__ __forceinline__ float gelu_quick(float x)
{
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(__fmul_rn(-1.702f, x))));
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

}  // namespace tcg

// numerics.cuh -- device arithmetic whose rounding sequence follows the
// reference's scalar C (src/ops.c), written with explicit _rn intrinsics so
// nvcc cannot contract it into FMAs.
#pragma once

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

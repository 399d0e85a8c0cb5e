/* dequant.h -- ggml tensor types to fp32 (drop-in for roofline.c
 * src/dequant.h:34-45), now with the K-quant arms.
 *
 * Same signatures and contract as the reference: tc_dequant returns false
 * for a type it cannot convert. Unlike the reference, the conversions run
 * on the GPU (tcg_dequant in tcg.h): these host-buffer entry points copy the
 * source to the device, run the sm_100a kernel and copy the fp32 result
 * back. The device must have been selected with tcg_init() first; a call
 * made without a usable GPU returns false (there is no CPU path).
 *
 * Types: F32 (plain copy), F16 (exact conversion, subnormals and NaN
 * payloads kept), Q4_K and Q6_K (256-weight superblocks, bit-identical to
 * ggml's dequantization). n must be a whole number of superblocks for the
 * K-quants.
 */
#ifndef TC_DEQUANT_H
#define TC_DEQUANT_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "arena.h"
#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* src/dequant.h:30-34: exact IEEE binary16 -> binary32 of one value. A pure
 * bit manipulation, evaluated where it is called. */
float tc_f16_to_f32(uint16_t h);

/* src/dequant.h:36-39: `n` elements of type `t` at host `src` into host `dst`. */
bool tc_dequant(float *dst, const void *src, size_t n, ggml_type_t t);

/* src/dequant.h:41-45: fp32 host view of a tensor -- the mapping itself for
 * F32, otherwise an arena allocation filled by tc_dequant. */
const float *tc_dequant_view(const gguf_tensor_t *t, arena_t *a, bool *converted);

#ifdef __cplusplus
}
#endif
#endif /* TC_DEQUANT_H */

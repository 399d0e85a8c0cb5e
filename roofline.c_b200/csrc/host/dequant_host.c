/* dequant_host.c -- the reference's dequant seam (src/dequant.h:30-45) on
 * host buffers, with every conversion but the F32 byte copy done by the
 * GPU kernels of tcg_dequant. */
#include "dequant.h"
#include "tcg_internal.h"

#include <string.h>

/* src/dequant.c:5-38: exact binary16 -> binary32 of one value. */
float tc_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t f = h & 0x3FFu, bits;
    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (f << 13);
    } else if (e) {
        bits = sign | ((e + 112u) << 23) | (f << 13);
    } else if (!f) {
        bits = sign;
    } else {
        uint32_t exp = 113u;
        while (!(f & 0x400u)) { f <<= 1; exp--; }
        bits = sign | (exp << 23) | ((f & 0x3FFu) << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

/* src/dequant.c:40-63 contract: false for a type with no conversion. */
bool tc_dequant(float *dst, const void *src, size_t n, ggml_type_t t)
{
    switch (t) {
    case GGML_TYPE_F32:
        memcpy(dst, src, n * sizeof(float));
        return true;
    case GGML_TYPE_F16:
    case GGML_TYPE_Q4_K:
    case GGML_TYPE_Q6_K:
        if ((t == GGML_TYPE_Q4_K || t == GGML_TYPE_Q6_K) && n % 256u) return false;
        return tcg_dequant_host(dst, src, n, t);
    default:
        return false;
    }
}

/* src/dequant.c:65-80 */
const float *tc_dequant_view(const gguf_tensor_t *t, arena_t *a, bool *converted)
{
    if (t == NULL || t->data == NULL) return NULL;
    if (t->type == GGML_TYPE_F32) {
        if (converted) *converted = false;
        return (const float *)t->data;
    }
    float *buf = (float *)arena_alloc(a, (size_t)t->n_elem * sizeof(float), ARENA_DEFAULT_ALIGN);
    if (buf == NULL) return NULL;
    if (!tc_dequant(buf, t->data, (size_t)t->n_elem, t->type)) return NULL;
    if (converted) *converted = true;
    return buf;
}

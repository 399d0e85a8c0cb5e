/* kquant_port.c -- TEST INFRASTRUCTURE ONLY (the CPU oracle; see oracle.h).
 *
 * Restates the reference's dequant seam (src/dequant.c) and fills in the two
 * K-quant arms it does not have yet (src/dequant.c:60-61). The K-quant block
 * layouts are ggml's published formats, as implemented by the third-party
 * `gguf` Python package 0.19.0 (gguf/quants.py, Q4_K and Q6_K); the reference
 * pins only their sizes (src/gguf.c:83,85; tests/test_gguf.c:217-221).
 *
 * Every float expression below is evaluated exactly as written (the Makefile
 * passes -ffp-contract=off), and the CUDA kernels reproduce the same rounding
 * sequence, so the comparison is bit-exact.
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

/* src/dequant.c:5-38. binary16 fields: 1 sign, 5 exponent (bias 15), 10
 * fraction. Every binary16 value, subnormals included, is a normal or zero
 * binary32, so the conversion is exact; NaN payloads are kept. */
float orc_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t f = h & 0x3FFu;
    uint32_t bits;

    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (f << 13);              /* inf / nan */
    } else if (e != 0u) {
        bits = sign | ((e + (127u - 15u)) << 23) | (f << 13);
    } else if (f == 0u) {
        bits = sign;                                         /* signed zero */
    } else {
        /* value = f * 2^-24; shift the leading one up to bit 10 */
        uint32_t shift = 0;
        while ((f & 0x400u) == 0u) { f <<= 1; shift++; }
        bits = sign | ((113u - shift) << 23) | ((f & 0x3FFu) << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ---- Q4_K: [d f16][dmin f16][scales 12B][qs 128B] = 144 bytes, 256 weights.
 * Eight sub-blocks of 32 weights, each with a 6-bit scale and 6-bit min.
 * Sub-blocks 0..3 keep their scale/min in the low 6 bits of bytes 0..3 / 4..7;
 * sub-blocks 4..7 take their low 4 bits from the nibbles of bytes 8..11 and
 * their top 2 bits from the spare top bits of bytes 0..3 (scale) / 4..7 (min).
 * Weights are stored as pairs of sub-blocks: 32 bytes whose low nibbles are
 * sub-block 2g and whose high nibbles are sub-block 2g+1.
 * w = (d * scale) * q - (dmin * min). */
static void q4k_sub_params(const uint8_t s[12], int j, int *scale, int *min)
{
    if (j < 4) {
        *scale = s[j] & 0x3F;
        *min   = s[j + 4] & 0x3F;
    } else {
        *scale = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *min   = (s[j + 4] >> 4)   | ((s[j] >> 6) << 4);
    }
}

static void q4k_block(float *y, const uint8_t *b)
{
    const float d    = orc_f16_to_f32(rd16(b + 0));
    const float dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4;
    const uint8_t *qs = b + 16;

    for (int g = 0; g < 4; g++) {
        int s_lo, m_lo, s_hi, m_hi;
        q4k_sub_params(sc, 2 * g, &s_lo, &m_lo);
        q4k_sub_params(sc, 2 * g + 1, &s_hi, &m_hi);
        const float a_lo = d * (float)s_lo, c_lo = dmin * (float)m_lo;
        const float a_hi = d * (float)s_hi, c_hi = dmin * (float)m_hi;
        const uint8_t *q = qs + 32 * g;
        float *o = y + 64 * g;
        for (int l = 0; l < 32; l++) {
            const float prod = a_lo * (float)(q[l] & 0x0F);
            o[l] = prod - c_lo;
        }
        for (int l = 0; l < 32; l++) {
            const float prod = a_hi * (float)(q[l] >> 4);
            o[32 + l] = prod - c_hi;
        }
    }
}

/* ---- Q6_K: [ql 128B][qh 64B][scales int8 x16][d f16] = 210 bytes.
 * Two halves of 128 weights. In half h, weight index i = 32*r + l (r = 0..3,
 * l = 0..31) takes its low 4 bits from ql[64h + l + 32*(r&1)] (low nibble for
 * r < 2, high nibble for r >= 2) and its top 2 bits from bits 2r..2r+1 of
 * qh[32h + l]; the 6-bit value is offset by -32. Its scale is the int8
 * scales[8h + 2r + l/16]. w = (d * scale) * q. */
static void q6k_block(float *y, const uint8_t *b)
{
    const uint8_t *ql = b;
    const uint8_t *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    const float d = orc_f16_to_f32(rd16(b + 208));

    for (int h = 0; h < 2; h++) {
        for (int r = 0; r < 4; r++) {
            for (int l = 0; l < 32; l++) {
                const uint8_t lo_byte = ql[64 * h + l + 32 * (r & 1)];
                const int lo = (r < 2) ? (lo_byte & 0x0F) : (lo_byte >> 4);
                const int hi = (qh[32 * h + l] >> (2 * r)) & 3;
                const int q = (lo | (hi << 4)) - 32;
                const float s = d * (float)sc[8 * h + 2 * r + l / 16];
                y[128 * h + 32 * r + l] = s * (float)q;
            }
        }
    }
}

bool orc_dequant(float *dst, const void *src, size_t n, int type)
{
    const uint8_t *p = (const uint8_t *)src;
    switch (type) {
    case ORC_F32:
        memcpy(dst, src, n * sizeof(float));
        return true;
    case ORC_F16:
        for (size_t i = 0; i < n; i++) dst[i] = orc_f16_to_f32(rd16(p + 2 * i));
        return true;
    case ORC_Q4_K:
        if (n % ORC_QK_K) return false;
        for (size_t blk = 0; blk < n / ORC_QK_K; blk++)
            q4k_block(dst + blk * ORC_QK_K, p + blk * ORC_Q4K_BYTES);
        return true;
    case ORC_Q6_K:
        if (n % ORC_QK_K) return false;
        for (size_t blk = 0; blk < n / ORC_QK_K; blk++)
            q6k_block(dst + blk * ORC_QK_K, p + blk * ORC_Q6K_BYTES);
        return true;
    default:
        return false;
    }
}

/* Dequantize row by row (so the whole fp32 matrix is never held) and take
 * each dot product in the reference's sequential fp32 order
 * (tc_ref_gemm with M=1, b_transposed, src/ops.c:16-19). */
bool orc_matvec_q(float *y, const void *W, const float *x, int N, int K, int type)
{
    size_t row_bytes;
    if (type == ORC_Q4_K) row_bytes = (size_t)K / ORC_QK_K * ORC_Q4K_BYTES;
    else if (type == ORC_Q6_K) row_bytes = (size_t)K / ORC_QK_K * ORC_Q6K_BYTES;
    else if (type == ORC_F16) row_bytes = (size_t)K * 2;
    else if (type == ORC_F32) row_bytes = (size_t)K * 4;
    else return false;
    if (K % ORC_QK_K && (type == ORC_Q4_K || type == ORC_Q6_K)) return false;

    float *row = (float *)malloc((size_t)K * sizeof(float));
    if (row == NULL) return false;
    for (int n = 0; n < N; n++) {
        if (!orc_dequant(row, (const uint8_t *)W + (size_t)n * row_bytes, (size_t)K, type)) {
            free(row);
            return false;
        }
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc += x[k] * row[k];
        y[n] = acc;
    }
    free(row);
    return true;
}

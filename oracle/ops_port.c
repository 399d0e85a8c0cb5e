/* ops_port.c -- TEST INFRASTRUCTURE ONLY (the CPU oracle; see oracle.h).
 *
 * Restatement of the reference's scalar fp32 ops (src/ops.c). The numerics
 * contract is the reference's own (src/ops.h:14-17, src/ops.c:44-58): dot
 * products accumulate in fp32 in index order; norm and softmax reductions
 * accumulate in double. The operation order inside each function is kept
 * identical to the reference so that, built with -ffp-contract=off, this file
 * and the reference produce bit-identical results (tests check that).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>

/* Sequential fp32 dot product with strides, index order 0..n-1
 * (the inner loops of src/ops.c:16-22). */
static float dot_seq(const float *a, size_t sa, const float *b, size_t sb, size_t n)
{
    float acc = 0.0f;
    for (size_t i = 0; i < n; i++) acc += a[i * sa] * b[i * sb];
    return acc;
}

/* src/ops.c:5-26 */
void orc_gemm(float *C, const float *A, const float *B, int M, int N, int K, bool b_transposed)
{
    const size_t Ms = (size_t)M, Ns = (size_t)N, Ks = (size_t)K;
    for (size_t m = 0; m < Ms; m++)
        for (size_t n = 0; n < Ns; n++)
            C[m * Ns + n] = b_transposed ? dot_seq(A + m * Ks, 1, B + n * Ks, 1, Ks)
                                         : dot_seq(A + m * Ks, 1, B + n, Ns, Ks);
}

/* src/ops.c:28-35: the GEMM first, the bias added afterwards as its own
 * rounding step. */
void orc_linear(float *y, const float *x, const float *W, const float *bias, int M, int N, int K)
{
    orc_gemm(y, x, W, M, N, K, true);
    if (bias == NULL) return;
    for (size_t m = 0; m < (size_t)M; m++)
        for (size_t n = 0; n < (size_t)N; n++) y[m * (size_t)N + n] += bias[n];
}

/* src/ops.c:37-80: two-pass mean / biased variance in double, the inverse
 * standard deviation rounded to float once, then per element
 * (float)(x - mean) * inv, times gamma, plus beta, each rounded in float. */
void orc_layernorm(float *out, const float *x, const float *gamma, const float *beta,
                   int rows, int cols, float eps)
{
    for (size_t r = 0; r < (size_t)rows; r++) {
        const float *in = x + r * (size_t)cols;
        float *o = out + r * (size_t)cols;
        double s = 0.0;
        for (int c = 0; c < cols; c++) s += (double)in[c];
        const double mean = s / (double)cols;
        double ss = 0.0;
        for (int c = 0; c < cols; c++) {
            const double dv = (double)in[c] - mean;
            ss += dv * dv;
        }
        const double var = ss / (double)cols;
        const float inv = (float)(1.0 / sqrt(var + (double)eps));
        for (int c = 0; c < cols; c++) {
            float v = (float)((double)in[c] - mean) * inv;
            if (gamma) v *= gamma[c];
            if (beta) v += beta[c];
            o[c] = v;
        }
    }
}

/* src/ops.c:82-87 */
void orc_gelu(float *out, const float *x, size_t n)
{
    const float inv_sqrt2 = 0.70710678118654752440f;
    for (size_t i = 0; i < n; i++) out[i] = 0.5f * x[i] * (1.0f + erff(x[i] * inv_sqrt2));
}

/* src/ops.c:89-93 */
void orc_gelu_quick(float *out, const float *x, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = x[i] / (1.0f + expf(-1.702f * x[i]));
}

/* One softmax row as src/ops.c:99-109 does it: max, exp(x - max) in float,
 * the sum of those in double, one float reciprocal, then a float multiply. */
static void softmax_row(float *o, const float *in, int cols)
{
    float mx = in[0];
    for (int c = 1; c < cols; c++) if (in[c] > mx) mx = in[c];
    double sum = 0.0;
    for (int c = 0; c < cols; c++) { o[c] = expf(in[c] - mx); sum += (double)o[c]; }
    const float inv = (float)(1.0 / sum);
    for (int c = 0; c < cols; c++) o[c] *= inv;
}

/* src/ops.c:95-110 */
void orc_softmax_rows(float *out, const float *x, int rows, int cols)
{
    for (size_t r = 0; r < (size_t)rows; r++)
        softmax_row(out + r * (size_t)cols, x + r * (size_t)cols, cols);
}

/* src/ops.c:112-151. Per head and query: fp32 scores (dot, then * scale),
 * max from -inf, exp in float with a double sum, one float reciprocal,
 * and the weighted sum of v rows accumulated in float in key order. */
void orc_mha(float *out, const float *q, const float *k, const float *v,
             int T, int n_head, int head_dim)
{
    const size_t D = (size_t)n_head * (size_t)head_dim, hd = (size_t)head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *w = (float *)malloc((size_t)T * sizeof(float));
    if (w == NULL) abort();

    for (size_t h = 0; h < (size_t)n_head; h++) {
        const size_t col = h * hd;
        for (size_t t = 0; t < (size_t)T; t++) {
            float mx = -INFINITY;
            for (size_t s = 0; s < (size_t)T; s++) {
                float sc = dot_seq(q + t * D + col, 1, k + s * D + col, 1, hd);
                sc *= scale;
                w[s] = sc;
                if (sc > mx) mx = sc;
            }
            double sum = 0.0;
            for (size_t s = 0; s < (size_t)T; s++) {
                w[s] = expf(w[s] - mx);
                sum += (double)w[s];
            }
            const float inv = (float)(1.0 / sum);
            float *o = out + t * D + col;
            for (size_t d = 0; d < hd; d++) o[d] = 0.0f;
            for (size_t s = 0; s < (size_t)T; s++) {
                const float p = w[s] * inv;
                const float *vr = v + s * D + col;
                for (size_t d = 0; d < hd; d++) o[d] += p * vr[d];
            }
        }
    }
    free(w);
}

/* src/ops.c:153-161 */
void orc_add(float *out, const float *a, const float *b, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

void orc_scale(float *out, const float *x, float s, size_t n)
{
    for (size_t i = 0; i < n; i++) out[i] = x[i] * s;
}

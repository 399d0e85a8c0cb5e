/* ops.h -- roofline.c's op API (src/ops.h:30-63), same names, arguments and
 * meaning, on HOST buffers, computed by libtcg's sm_100a kernels.
 *
 * Each call copies its inputs to the device, runs the kernel on the calling
 * thread's library stream and copies the result back before it returns, so
 * a caller of the reference's scalar ops (its tests, a future CLI) links
 * libtcg.so in their place and changes nothing. The results meet the
 * reference's own golden-vector tolerances (tests/test_ops.c:74-148): the
 * GEMMs run as 3xTF32 on the tensor cores (fp32-accurate), LayerNorm and the
 * softmax keep the reference's double sums.
 *
 * The reference's ops return nothing, so these cannot report failure. A
 * thread that has not called tcg_init gets device 0 (or $TCG_DEVICE) on its
 * first call; if there is no usable device, or a copy or kernel fails, the
 * call prints the reason to stderr and aborts -- it never falls back to a
 * CPU computation. Inputs and the output may alias (all inputs are copied in
 * first). For work that stays on the device, tcg.h has the same ops on
 * device pointers (tcg_linear, tcg_layernorm, ...).
 */
#ifndef TC_OPS_H
#define TC_OPS_H

#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* C[M,N] = A[M,K] * B, B [K,N], or [N,K] when b_transposed
 * (src/ops.h:30-33). */
void tc_ref_gemm(float *C, const float *A, const float *B,
                 int M, int N, int K, bool b_transposed);

/* y[M,N] = x[M,K] * W[N,K]^T + b[N]; bias may be NULL (src/ops.h:35-37). */
void tc_ref_linear(float *y, const float *x, const float *W, const float *bias,
                   int M, int N, int K);

/* Per row: (x - mean) / sqrt(var + eps) * gamma + beta, biased variance
 * (src/ops.h:39-42). */
void tc_ref_layernorm(float *out, const float *x, const float *gamma,
                      const float *beta, int rows, int cols, float eps);

/* 0.5 x (1 + erf(x / sqrt 2)) (src/ops.h:44-45). */
void tc_ref_gelu(float *out, const float *x, size_t n);

/* x * sigmoid(1.702 x) (src/ops.h:47-51). */
void tc_ref_gelu_quick(float *out, const float *x, size_t n);

/* Row-wise softmax, max-subtracted (src/ops.h:53-54). */
void tc_ref_softmax_rows(float *out, const float *x, int rows, int cols);

/* Bidirectional multi-head attention, q, k, v, out [T, n_head * head_dim],
 * scale 1/sqrt(head_dim) (src/ops.h:56-61). The scores stay on chip, so
 * `scratch` is accepted and not used. */
void tc_ref_mha(float *out, const float *q, const float *k, const float *v,
                int T, int n_head, int head_dim, float *scratch);

/* out = a + b; out = s * x (src/ops.h:62-63). */
void tc_ref_add(float *out, const float *a, const float *b, size_t n);
void tc_ref_scale(float *out, const float *x, float s, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* TC_OPS_H */

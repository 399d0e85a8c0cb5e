// ops.cuh -- launchers shared by the op API (ops.cu) and the ViT pipeline.
#pragma once

#include "tcg_common.cuh"

namespace tcg {

// Where an activation goes: plain fp32, and/or the tf32 hi/lo pair the
// 3xTF32 GEMMs read (hi = rn_tf32(v), lo = rn_tf32(v - hi)), or the fp16
// pieces the kind::f16 GEMM reads (fh, fl: row stride ld, in halves; fe: the
// exponent of each (row, 256-column block), fe[block * fe_rows + row];
// LayerNorm only). Row stride ld.
struct OutSpec {
    float *plain = nullptr;
    float *hi = nullptr;
    float *lo = nullptr;
    int ld = 0;
    void *fh = nullptr;
    void *fl = nullptr;
    int8_t *fe = nullptr;
    int fe_rows = 0;
    float *rnorm = nullptr;    // LayerNorm with fp16 pieces: each output row's 2-norm
};

// bounds[0] = the largest 2-norm of W's rows ([rows, K]), bounds[1] = the
// largest |b| (b: rows values, or none); bounds must start at zero.
bool launch_weight_bounds(const float *W, int rows, int K, const float *b, float *bounds, cudaStream_t s);

// fp32 rows -> fp16 pieces (gemm_tc.cu): mode 0 / 2 one exponent per (row,
// 128- / 256-element K-block), mode 1 one per row.
bool launch_split_f16(const float *src, int rows, int K, void *hi, void *lo, int8_t *ex, int mode, cudaStream_t s);
// the configuration of the kind::f16 GEMM on fp16 pieces
int gemm_f16_cfg();

// K-quant blocks straight to their tf32 pairs (kquant.cu).
bool launch_dequant_split(const void *src, float *hi, float *lo, size_t n, ggml_type_t t, cudaStream_t s);

// LayerNorm of `rows` rows of `cols` (src/ops.c:37-80 numerics: double
// two-pass stats). Input row r at x + r*ld_in.
bool launch_layernorm(const float *x, int ld_in, const float *g, const float *b, int rows, int cols,
                      float eps, const OutSpec &out, cudaStream_t s);

// Attention over n_img images of T tokens (src/ops.c:112-151). Image i,
// token t, head h reads q at q + (i*T + t)*ldi + h*hd (same for k, v).
// head_dim 64, 128 <= T <= 1024 on the tensor cores (attn_tc.cu); false when the shape does not fit.
bool launch_mha64_tc_long(const float *q, const float *k, const float *v, int ldi, int T, int n_head, int n_img,
                          const OutSpec &out, cudaStream_t s);

bool launch_mha(const float *q, const float *k, const float *v, int ldi, int T, int n_head, int hd,
                int n_img, const OutSpec &out, cudaStream_t s);

// fp32 CUDA-core GEMM: C = A * op(B) (+ bias[n]); A [M,K] row stride lda,
// op(B) = B^T for B [N,K] (b_transposed) else B [K,N]; C row stride ldc.
bool launch_gemm_simt(float *C, int ldc, const float *A, int lda, const float *B, int ldb,
                      const float *bias, int M, int N, int K, bool b_transposed, cudaStream_t s);

// hi/lo split of n contiguous floats.
bool launch_split(const float *src, float *hi, float *lo, size_t n, cudaStream_t s);

// dst pair [C, R] = tf32 hi/lo of src [R, C] transposed.
bool launch_transpose_split(const float *src, int R, int C, float *hi, float *lo, cudaStream_t s);

// im2patch (src/vit.c:283-303) of n_img images [3, S, S] straight into the
// hi/lo operand pair [n_img*G*G, 3*P*P].
bool launch_patches(const float *px, int n_img, int S, int P, float *hi, float *lo, cudaStream_t s);

// x[i*T + 0, :] = cls + pos[0, :] for every image (src/vit.c:346-347, row 0).
bool launch_cls_rows(float *x, const float *cls, const float *pos, int n_img, int T, int D, cudaStream_t s);

// out[n] = act(x[n]) elementwise: 0 identity-add, 1 gelu, 2 quick gelu.
bool launch_gelu(float *out, const float *x, size_t n, bool quick, cudaStream_t s);

}  // namespace tcg

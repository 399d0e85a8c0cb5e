/* oracle.h -- TEST INFRASTRUCTURE ONLY. Never linked into, loaded by, or
 * called from the product library (roofline.c_b200/). Only tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline leg of bench.py use it,
 * and only as the checker.
 *
 * A plain-C restatement of roofline.c's compute path, used as the CPU oracle
 * the CUDA kernels are compared against:
 *
 *   orc_f16_to_f32          src/dequant.c:5-38
 *   orc_dequant             src/dequant.c:40-63, plus the Q4_K / Q6_K arms the
 *                           reference leaves to "stage 02" (src/dequant.c:60-61).
 *                           Those two arms restate ggml's published K-quant
 *                           block formats (the layout implemented by the `gguf`
 *                           Python package 0.19.0, gguf/quants.py, classes
 *                           Q4_K and Q6_K), which is third-party code absent
 *                           from the reference tree; the block sizes are pinned
 *                           by the reference at src/gguf.c:83,85.
 *   orc_gemm / orc_linear   src/ops.c:5-35
 *   orc_layernorm           src/ops.c:37-80
 *   orc_gelu / _quick       src/ops.c:82-93
 *   orc_softmax_rows        src/ops.c:95-110
 *   orc_mha                 src/ops.c:112-151
 *   orc_add / orc_scale     src/ops.c:153-161
 *   orc_matvec_q            the composition the reference would run for a
 *                           quantized decode matvec: dequant (above) followed
 *                           by tc_ref_linear with M=1 (src/ops.c:28-35).
 *   orc_vit_forward         src/vit.c:283-391 (im2patch + tc_vit_encode)
 *
 * Built by oracle/Makefile with -std=c11 -ffp-contract=off so that every
 * float expression rounds exactly as written, like the reference's own
 * -std=c11 build (ISO C mode: no FMA contraction).
 */
#ifndef ORACLE_H
#define ORACLE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

/* ggml type ids, on-disk values (src/gguf.h:59-80). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_K = 12, ORC_Q6_K = 14 };

#define ORC_QK_K      256   /* elements per K-quant superblock            */
#define ORC_Q4K_BYTES 144   /* 2 d + 2 dmin + 12 scales + 128 nibbles      */
#define ORC_Q6K_BYTES 210   /* 128 ql + 64 qh + 16 int8 scales + 2 d       */

float orc_f16_to_f32(uint16_t h);
bool  orc_dequant(float *dst, const void *src, size_t n, int type);
bool  orc_matvec_q(float *y, const void *W, const float *x, int N, int K, int type);

void orc_gemm(float *C, const float *A, const float *B, int M, int N, int K, bool b_transposed);
void orc_linear(float *y, const float *x, const float *W, const float *bias, int M, int N, int K);
void orc_layernorm(float *out, const float *x, const float *gamma, const float *beta,
                   int rows, int cols, float eps);
void orc_gelu(float *out, const float *x, size_t n);
void orc_gelu_quick(float *out, const float *x, size_t n);
void orc_softmax_rows(float *out, const float *x, int rows, int cols);
void orc_mha(float *out, const float *q, const float *k, const float *v,
             int T, int n_head, int head_dim);
void orc_add(float *out, const float *a, const float *b, size_t n);
void orc_scale(float *out, const float *x, float s, size_t n);

/* ViT weights by pointer; the test harness fills this from a GGUF file. */
typedef struct {
    const float *ln1_g, *ln1_b, *qkv_w, *qkv_b, *out_w, *out_b;
    const float *ln2_g, *ln2_b, *up_w, *up_b, *down_w, *down_b;
} orc_vit_block_t;

typedef struct {
    int n_layer, d_model, n_head, d_ffn, patch, image, d_out;
    float ln_eps;
    int quick_gelu;
    const float *patch_embd, *cls_token, *pos_embd;
    const float *ln_pre_g, *ln_pre_b, *ln_post_g, *ln_post_b, *proj;
    const orc_vit_block_t *blocks;
} orc_vit_t;

/* One image. Taps may be NULL; each non-NULL tap receives [T, D] floats
 * (embedding: d_out floats in `out`). Returns false on allocation failure. */
bool orc_vit_forward(const orc_vit_t *m, const float *pixels, float *out,
                     float *tap_ln_pre, float *tap_blk0, float *tap_blk_last,
                     float *tap_ln_post);

#endif

/* vit.h -- CLIP ViT image encoder, fp32 (drop-in for roofline.c
 * src/vit.h:34-85), computed on a B200.
 *
 * tc_vit_load parses and validates the GGUF exactly as the reference does
 * (architecture, hyper-parameters, explicit activation, CLS pooling, every
 * tensor present with the right element count) and resolves host fp32
 * weight views. tc_vit_encode keeps the reference's signature and contract
 * (one normalised [3, image, image] image in, d_out floats out, the same
 * five taps) but runs the batched sm_100a pipeline of tcg.h with a batch of
 * one: on the first call it uploads the weights to the current device
 * (tcg_init must have been called) and keeps them until tc_vit_free.
 *
 * The struct is the reference's with one field appended (`dev`, the device
 * model handle, NULL until the first upload); code that reads the
 * reference's fields compiles unchanged.
 */
#ifndef TC_VIT_H
#define TC_VIT_H

#include <stdbool.h>
#include <stddef.h>

#include "arena.h"
#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* PyTorch layouts as stored ("[out, in]" = nn.Linear weight). */
typedef struct {
    const float *ln1_g, *ln1_b;
    const float *qkv_w, *qkv_b;     /* [3D, D], [3D]: q, k, v row blocks   */
    const float *out_w, *out_b;     /* [D, D], [D]                         */
    const float *ln2_g, *ln2_b;
    const float *up_w, *up_b;       /* [F, D], [F]                         */
    const float *down_w, *down_b;   /* [D, F], [D]                         */
} tc_vit_block_t;

typedef struct {
    int n_layer, d_model, n_head, head_dim, d_ffn;
    int patch, image, grid, n_token, d_out;
    float ln_eps;
    bool quick_gelu;                /* from clip-vit.activation            */
    float mean[3], std[3];          /* clip-vit.preprocess.* (not applied) */

    const float *patch_embd;        /* [D, 3*P*P]                          */
    const float *cls_token;         /* [D]                                 */
    const float *pos_embd;          /* [T, D]                              */
    const float *ln_pre_g, *ln_pre_b;
    const float *ln_post_g, *ln_post_b;
    const float *proj;              /* [D, d_out], used untransposed        */
    tc_vit_block_t *blocks;

    gguf_t gguf;
    size_t weight_bytes;            /* arena bytes spent converting non-F32 */
    char err[256];

    void *dev;                      /* tcg_vit_t*, owned; NULL until upload */
} tc_vit_t;

/* src/vit.h:63-68 */
bool tc_vit_load(tc_vit_t *out, const char *path, arena_t *a);
void tc_vit_free(tc_vit_t *m);

/* src/vit.h:70-73: intermediate activations, rows x cols, host memory. */
typedef void (*tc_vit_tap_fn)(void *ud, const char *name, const float *data, int rows, int cols);

/* src/vit.h:75-81. `scratch` supplies the host staging for taps and is
 * released before returning. False (reason in m->err) on any device error. */
bool tc_vit_encode(const tc_vit_t *m, const float *pixels, float *out,
                   arena_t *scratch, tc_vit_tap_fn tap, void *ud);

/* src/vit.h:83-84: host scratch bytes tc_vit_encode may take from `scratch`
 * (the reference's figure, which covers the tap staging used here). */
size_t tc_vit_scratch_bytes(const tc_vit_t *m);

#ifdef __cplusplus
}
#endif
#endif /* TC_VIT_H */

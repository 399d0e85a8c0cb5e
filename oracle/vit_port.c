/* vit_port.c -- TEST INFRASTRUCTURE ONLY (the CPU oracle; see oracle.h).
 *
 * Restatement of the reference's single-image CLIP ViT forward,
 * tc_vit_encode (src/vit.c:305-391) with im2patch (src/vit.c:283-303), over
 * the ops restated in ops_port.c. Same dataflow and the same op order:
 * patch GEMM, CLS row, + position, ln_pre, L pre-LN blocks (three row-block
 * projections of the fused qkv weight, MHA, out-proj, residual, ln2, up,
 * GELU, down, residual), ln_post over every row, and the projection of the
 * CLS row with v.proj used untransposed.
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

/* Token t = gy*G + gx holds channel-major patch values with kx fastest, the
 * flattening that a [D, 3, P, P] conv weight implies (src/vit.c:277-303). */
static void patches_of(const orc_vit_t *m, const float *px, float *dst)
{
    const int P = m->patch, S = m->image, G = S / P;
    for (int t = 0; t < G * G; t++) {
        const int gy = t / G, gx = t % G;
        for (int c = 0; c < 3; c++)
            for (int ky = 0; ky < P; ky++) {
                const float *src = px + ((size_t)c * S + (size_t)(gy * P + ky)) * S + (size_t)gx * P;
                memcpy(dst, src, (size_t)P * sizeof(float));
                dst += P;
            }
    }
}

bool orc_vit_forward(const orc_vit_t *m, const float *pixels, float *out,
                     float *tap_ln_pre, float *tap_blk0, float *tap_blk_last,
                     float *tap_ln_post)
{
    const int D = m->d_model, F = m->d_ffn, P = m->patch, G = m->image / m->patch;
    const int T = G * G + 1, K0 = 3 * P * P;
    const size_t TD = (size_t)T * D;

    float *x = malloc(TD * sizeof(float)), *h = malloc(TD * sizeof(float));
    float *q = malloc(TD * sizeof(float)), *k = malloc(TD * sizeof(float));
    float *v = malloc(TD * sizeof(float)), *att = malloc(TD * sizeof(float));
    float *ffn = malloc((size_t)T * F * sizeof(float));
    float *pt = malloc((size_t)(T - 1) * K0 * sizeof(float));
    bool ok = x && h && q && k && v && att && ffn && pt;
    if (!ok) goto done;

    patches_of(m, pixels, pt);
    orc_linear(x + D, pt, m->patch_embd, NULL, T - 1, D, K0);
    memcpy(x, m->cls_token, (size_t)D * sizeof(float));
    orc_add(x, x, m->pos_embd, TD);
    orc_layernorm(x, x, m->ln_pre_g, m->ln_pre_b, T, D, m->ln_eps);
    if (tap_ln_pre) memcpy(tap_ln_pre, x, TD * sizeof(float));

    for (int i = 0; i < m->n_layer; i++) {
        const orc_vit_block_t *b = &m->blocks[i];
        const size_t blk = (size_t)D * D;
        orc_layernorm(h, x, b->ln1_g, b->ln1_b, T, D, m->ln_eps);
        orc_linear(q, h, b->qkv_w, b->qkv_b, T, D, D);
        orc_linear(k, h, b->qkv_w + blk, b->qkv_b + D, T, D, D);
        orc_linear(v, h, b->qkv_w + 2 * blk, b->qkv_b + 2 * D, T, D, D);
        orc_mha(att, q, k, v, T, m->n_head, D / m->n_head);
        orc_linear(h, att, b->out_w, b->out_b, T, D, D);
        orc_add(x, x, h, TD);
        orc_layernorm(h, x, b->ln2_g, b->ln2_b, T, D, m->ln_eps);
        orc_linear(ffn, h, b->up_w, b->up_b, T, F, D);
        if (m->quick_gelu) orc_gelu_quick(ffn, ffn, (size_t)T * F);
        else               orc_gelu(ffn, ffn, (size_t)T * F);
        orc_linear(h, ffn, b->down_w, b->down_b, T, D, F);
        orc_add(x, x, h, TD);
        if (i == 0 && tap_blk0) memcpy(tap_blk0, x, TD * sizeof(float));
        if (i == m->n_layer - 1 && tap_blk_last) memcpy(tap_blk_last, x, TD * sizeof(float));
    }

    orc_layernorm(x, x, m->ln_post_g, m->ln_post_b, T, D, m->ln_eps);
    if (tap_ln_post) memcpy(tap_ln_post, x, TD * sizeof(float));
    orc_gemm(out, x, m->proj, 1, m->d_out, D, false);

done:
    free(x); free(h); free(q); free(k); free(v); free(att); free(ffn); free(pt);
    return ok;
}

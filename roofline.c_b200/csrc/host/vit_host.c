/* vit_host.c -- tc_vit_load / tc_vit_free / tc_vit_encode /
 * tc_vit_scratch_bytes (roofline.c src/vit.h:63-84) over the device
 * pipeline of tcg.h.
 *
 * The loader applies the reference's refusals (src/vit.c:135-261): the
 * architecture must be clip-vit, every hyper-parameter present and
 * consistent, the activation named explicitly (gelu or gelu_quick, never
 * guessed), pooling absent or cls, and every tensor present with the
 * expected element count. Tensor names and metadata keys are the GGUF
 * contract of the reference's exporter, so they are the same strings.
 */
#include "vit.h"

#include "dequant.h"
#include "tcg_internal.h"

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

__attribute__((format(printf, 2, 3)))
static bool refuse(tc_vit_t *m, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(m->err, sizeof m->err, fmt, ap);
    va_end(ap);
    gguf_close(&m->gguf);
    return false;
}

/* Resolve one tensor to an fp32 host view after checking its element count
 * (the count, not the dims: a [D,3,P,P] conv weight is read as [D, 3P^2]). */
static const float *resolve(tc_vit_t *m, arena_t *a, const char *name, size_t n_elem)
{
    const gguf_tensor_t *t = gguf_tensor(&m->gguf, name);
    if (!t) {
        snprintf(m->err, sizeof m->err, "missing tensor '%s'", name);
        return NULL;
    }
    if (t->n_elem != n_elem) {
        snprintf(m->err, sizeof m->err, "tensor '%s' has %llu elements, expected %zu",
                 name, (unsigned long long)t->n_elem, n_elem);
        return NULL;
    }
    bool converted = false;
    const float *p = tc_dequant_view(t, a, &converted);
    if (!p) {
        snprintf(m->err, sizeof m->err, "cannot materialize '%s' (%s)", name, ggml_type_name(t->type));
        return NULL;
    }
    if (converted) m->weight_bytes += n_elem * sizeof(float);
    return p;
}

static bool read_f32x3(const gguf_t *g, const char *key, float out[3])
{
    const gguf_kv_t *kv = gguf_find(g, key);
    if (!kv || kv->type != GGUF_T_ARRAY || kv->v.arr.type != GGUF_T_FLOAT32 || kv->v.arr.len != 3) return false;
    memcpy(out, kv->v.arr.data, 3 * sizeof(float));
    return true;
}

bool tc_vit_load(tc_vit_t *out, const char *path, arena_t *a)
{
    tc_vit_t *m = out;
    memset(m, 0, sizeof *m);
    if (!gguf_open(&m->gguf, path, a)) {
        snprintf(m->err, sizeof m->err, "%s", m->gguf.err);
        return false;
    }
    const gguf_t *g = &m->gguf;
    gguf_str_t s;
    if (!gguf_get_str(g, "general.architecture", &s) || !gguf_str_eq(s, "clip-vit"))
        return refuse(m, "not a clip-vit file");

    m->n_layer = (int)gguf_u64_or(g, "clip-vit.block_count", 0);
    m->d_model = (int)gguf_u64_or(g, "clip-vit.embedding_length", 0);
    m->n_head = (int)gguf_u64_or(g, "clip-vit.attention.head_count", 0);
    m->d_ffn = (int)gguf_u64_or(g, "clip-vit.feed_forward_length", 0);
    m->patch = (int)gguf_u64_or(g, "clip-vit.patch_size", 0);
    m->image = (int)gguf_u64_or(g, "clip-vit.image_size", 0);
    m->d_out = (int)gguf_u64_or(g, "clip-vit.projection_dim", 0);
    m->ln_eps = gguf_f32_or(g, "clip-vit.layer_norm_epsilon", 1e-5f);
    if (m->n_layer <= 0 || m->d_model <= 0 || m->n_head <= 0 || m->d_ffn <= 0 || m->patch <= 0 ||
        m->image <= 0 || m->d_out <= 0)
        return refuse(m, "incomplete architecture metadata");
    if (m->d_model % m->n_head) return refuse(m, "d_model %d not divisible by %d heads", m->d_model, m->n_head);
    if (m->image % m->patch) return refuse(m, "image %d not divisible by patch %d", m->image, m->patch);
    m->head_dim = m->d_model / m->n_head;
    m->grid = m->image / m->patch;
    m->n_token = m->grid * m->grid + 1;
    const uint64_t ctx_len = gguf_u64_or(g, "clip-vit.context_length", 0);
    if (ctx_len && ctx_len != (uint64_t)m->n_token)
        return refuse(m, "context_length %llu but grid implies %d tokens", (unsigned long long)ctx_len, m->n_token);

    if (!gguf_get_str(g, "clip-vit.activation", &s))
        return refuse(m, "no clip-vit.activation — re-export; GELU form must not be guessed");
    if (gguf_str_eq(s, "gelu")) m->quick_gelu = false;
    else if (gguf_str_eq(s, "gelu_quick")) m->quick_gelu = true;
    else {
        char b[64];
        return refuse(m, "unsupported activation '%s'", gguf_str_cstr(b, sizeof b, s));
    }
    if (gguf_get_str(g, "clip-vit.pooling", &s) && !gguf_str_eq(s, "cls")) {
        char b[64];
        return refuse(m, "pooling '%s' not implemented (only cls)", gguf_str_cstr(b, sizeof b, s));
    }
    read_f32x3(g, "clip-vit.preprocess.mean", m->mean);
    read_f32x3(g, "clip-vit.preprocess.std", m->std);

    const size_t D = (size_t)m->d_model, F = (size_t)m->d_ffn, T = (size_t)m->n_token, P = (size_t)m->patch;
    struct { const float **dst; const char *name; size_t n; } top[] = {
        { &m->patch_embd, "v.patch_embd.weight", D * 3 * P * P },
        { &m->cls_token, "v.cls_token", D },
        { &m->pos_embd, "v.pos_embd", T * D },
        { &m->ln_pre_g, "v.ln_pre.weight", D },
        { &m->ln_pre_b, "v.ln_pre.bias", D },
        { &m->ln_post_g, "v.ln_post.weight", D },
        { &m->ln_post_b, "v.ln_post.bias", D },
        { &m->proj, "v.proj", D * (size_t)m->d_out },
    };
    for (size_t i = 0; i < sizeof top / sizeof top[0]; i++)
        if (!(*top[i].dst = resolve(m, a, top[i].name, top[i].n))) { gguf_close(&m->gguf); return false; }

    m->blocks = (tc_vit_block_t *)arena_alloc(a, sizeof(tc_vit_block_t) * (size_t)m->n_layer,
                                              _Alignof(tc_vit_block_t));
    if (!m->blocks) return refuse(m, "arena exhausted (blocks)");
    for (int i = 0; i < m->n_layer; i++) {
        tc_vit_block_t *b = &m->blocks[i];
        struct { const float **dst; const char *suffix; size_t n; } per[] = {
            { &b->ln1_g, "ln1.weight", D }, { &b->ln1_b, "ln1.bias", D },
            { &b->qkv_w, "attn_qkv.weight", 3 * D * D }, { &b->qkv_b, "attn_qkv.bias", 3 * D },
            { &b->out_w, "attn_out.weight", D * D }, { &b->out_b, "attn_out.bias", D },
            { &b->ln2_g, "ln2.weight", D }, { &b->ln2_b, "ln2.bias", D },
            { &b->up_w, "ffn_up.weight", F * D }, { &b->up_b, "ffn_up.bias", F },
            { &b->down_w, "ffn_down.weight", D * F }, { &b->down_b, "ffn_down.bias", D },
        };
        for (size_t j = 0; j < sizeof per / sizeof per[0]; j++) {
            char name[96];
            snprintf(name, sizeof name, "v.blk.%d.%s", i, per[j].suffix);
            if (!(*per[j].dst = resolve(m, a, name, per[j].n))) { gguf_close(&m->gguf); return false; }
        }
    }
    return true;
}

void tc_vit_free(tc_vit_t *m)
{
    if (!m) return;
    if (m->dev) {
        tcg_vit_release((tcg_vit_t *)m->dev);
        m->dev = NULL;
    }
    gguf_close(&m->gguf);
}

size_t tc_vit_scratch_bytes(const tc_vit_t *m)
{
    const size_t T = (size_t)m->n_token, D = (size_t)m->d_model, F = (size_t)m->d_ffn;
    return (6 * T * D + T * F + T) * sizeof(float) + 8 * ARENA_DEFAULT_ALIGN;
}

bool tc_vit_encode(const tc_vit_t *m, const float *pixels, float *out, arena_t *scratch,
                   tc_vit_tap_fn tap, void *ud)
{
    /* The device copy of the weights is a cache owned by the model; creating
     * it does not change anything tc_vit_encode's caller can observe. */
    tc_vit_t *mm = (tc_vit_t *)m;
    if (!mm->dev) {
        mm->dev = tcg_vit_upload(m, 1);
        if (!mm->dev) {
            snprintf(mm->err, sizeof mm->err, "device upload failed: %s", tcg_last_error());
            return false;
        }
    }
    const size_t mark = arena_mark(scratch);
    float *staging = NULL;
    if (tap) {
        const size_t n = tcg_vit_tap_staging_floats((const tcg_vit_t *)mm->dev, 1);
        staging = (float *)arena_alloc(scratch, n * sizeof(float), ARENA_DEFAULT_ALIGN);
        if (!staging) {
            snprintf(mm->err, sizeof mm->err, "scratch arena too small for tap staging");
            return false;
        }
    }
    const bool ok = tcg_vit_encode_batch_staged((tcg_vit_t *)mm->dev, pixels, 1, out, tap, ud, staging);
    if (!ok) snprintf(mm->err, sizeof mm->err, "%s", tcg_last_error());
    arena_release(scratch, mark);
    return ok;
}

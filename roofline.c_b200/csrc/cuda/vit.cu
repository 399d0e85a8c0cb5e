// vit.cu -- the batched CLIP ViT forward on one B200 (tcg_vit_*), the device
// counterpart of roofline.c's tc_vit_encode (src/vit.c:305-391).
//
// Per forward of n images (M = n*T token rows):
//   patches    pixels -> im2patch tf32 hi/lo                      [n*G*G, 3P^2]
//   GEMM       patch embed; epilogue adds the position row and stores token
//              r of image i at row i*T + 1 + r                    -> x
//   cls        x[i*T] = cls + pos[0]
//   LN         ln_pre in place on x                               (tap ln_pre)
//   L blocks   LN1 -> h(hi/lo); GEMM qkv (+bias) -> qkv; attention -> a(hi/lo);
//              GEMM out (+bias, +x) -> x; LN2 -> h; GEMM up (+bias, GELU)
//              -> f(hi/lo); GEMM down (+bias, +x) -> x      (taps blk0, blk_last)
//   LN         ln_post on the CLS rows, as a tf32 pair (all rows too, plain,
//              when tapping)                                       (tap ln_post)
//   GEMM       pooled[n, D] x proj[D, d_out] (proj held transposed) (tap embedding)
// All GEMMs are the 3xTF32 tcgen05 kernel; everything after the patch gather
// is recorded once per batch size as a CUDA graph.
#include "gemm.cuh"
#include "tcg_internal.h"

#include <algorithm>
#include <chrono>
#include <map>
#include <memory>
#include <mutex>
#include <string.h>
#include <string>
#include <thread>
#include <vector>

struct tcg_vit {
    int L, D, H, hd, F, P, S, G, T, d_out;
    float eps;
    bool quick;
    int max_batch;
    int device;
    bool graphs = true;
    // GEMMs on fp16 pieces (kind::f16; every weight fp32 on the device and
    // d_model, d_ffn multiples of 256); the patch GEMM too where 3 P^2 is
    bool f16 = false, patch_f16 = false;

    // fp32 weights, one allocation (the unit of the NCCL broadcast)
    float *wslab = nullptr;
    size_t wslab_floats = 0;
    // tf32 hi/lo of every GEMM weight that is not kept packed
    float *sslab = nullptr;
    size_t sslab_floats = 0;
    // Q4_K blocks of the GEMM weights kept packed (their GEMMs dequantise
    // them tile by tile in shared memory)
    uint8_t *qslab = nullptr;
    size_t qslab_bytes = 0;
    // the tf32 pair a packed weight is dequantised into before its GEMM at
    // large batches (the largest packed weight's size; reused GEMM by GEMM)
    float *jit_hi = nullptr, *jit_lo = nullptr;

    struct Layer {
        const float *ln1_g, *ln1_b, *qkv_b, *out_b, *ln2_g, *ln2_b, *up_b, *down_b;
        const float *qkv_h, *qkv_l, *out_h, *out_l, *up_h, *up_l, *down_h, *down_l;
        const uint8_t *qkv_q = nullptr, *out_q = nullptr, *up_q = nullptr, *down_q = nullptr;
        // fp16 pieces: each weight row's exponent (the _h/_l fields hold fp16)
        const int8_t *qkv_e = nullptr, *out_e = nullptr, *up_e = nullptr, *down_e = nullptr;
    };
    std::vector<Layer> layers;
    const float *patch_h = nullptr, *patch_l = nullptr, *cls = nullptr, *pos = nullptr;
    const uint8_t *patch_q = nullptr;
    const int8_t *patch_e = nullptr;
    const float *ln_pre_g = nullptr, *ln_pre_b = nullptr, *ln_post_g = nullptr, *ln_post_b = nullptr;
    const float *proj = nullptr;
    const float *projT_h = nullptr, *projT_l = nullptr;   // v.proj transposed to [d_out, D], split

    // activations
    tcg_arena_t act{};
    float *px = nullptr, *x = nullptr, *h_hi = nullptr, *h_lo = nullptr, *qkv = nullptr;
    float *f_hi = nullptr, *f_lo = nullptr, *pooled_hi = nullptr, *pooled_lo = nullptr, *out = nullptr;
    float *p_hi = nullptr, *p_lo = nullptr;   // alias f_hi / f_lo
    // fp16-piece activations: exponents per (row, 256-column block); h's
    // pieces live in h_hi / h_lo, f's and the patches' in f_lo (hi half
    // first), their fp32 source in f_hi
    int8_t *h_e = nullptr, *f_e = nullptr, *p_e = nullptr;
    // fp16 pieces: LN2's output row norms and each layer's up-projection
    // bounds (largest weight-row norm, largest |bias|): the GELU output's
    // per-row scale is taken from them in the up projection's epilogue
    float *rnorm = nullptr, *up_bounds = nullptr;
    tcg::GemmWork work;                       // this model's GEMM stream-K memory (in the arena)

    struct Plans {
        tcg::GemmPlan patch, proj;
        std::vector<tcg::GemmPlan> qkv, out, up, down;
        cudaGraphExec_t graph = nullptr;
    };
    std::map<int, std::unique_ptr<Plans>> plans;

    // asynchronous submissions: two pixel slots and a copy stream
    float *px_slot[2] = { nullptr, nullptr };   // [0] is px; [1] allocated on first submission
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t copied[2] = {}, done[2] = {};
    bool in_flight[2] = { false, false };
    int next_ticket = 0;

    ~tcg_vit()
    {
        for (auto &kv : plans)
            if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
        tcg_arena_destroy(&act);
        if (wslab) cudaFree(wslab);
        if (sslab) cudaFree(sslab);
        if (qslab) cudaFree(qslab);
        if (jit_hi) cudaFree(jit_hi);
        for (int i = 0; i < 2; i++) {
            if (px_slot[i] && px_slot[i] != px) cudaFree(px_slot[i]);
            if (copied[i]) cudaEventDestroy(copied[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
    }
};

namespace tcg {

// Weight tensors in slab order: (element count, host pointer, device slot).
struct WEntry {
    size_t n;
    const float *host;
    const float **dev;
};

static size_t align_floats(size_t n) { return (n + 63) & ~(size_t)63; }   // 256-byte slots

static std::vector<WEntry> weight_table(tcg_vit *v, const tc_vit_t *m)
{
    const size_t D = v->D, F = v->F, P = v->P, T = v->T;
    std::vector<WEntry> t;
    t.push_back({ D * 3 * P * P, m->patch_embd, nullptr });   // [0] patch_embd (split only)
    t.push_back({ D, m->cls_token, &v->cls });
    t.push_back({ T * D, m->pos_embd, &v->pos });
    t.push_back({ D, m->ln_pre_g, &v->ln_pre_g });
    t.push_back({ D, m->ln_pre_b, &v->ln_pre_b });
    t.push_back({ D, m->ln_post_g, &v->ln_post_g });
    t.push_back({ D, m->ln_post_b, &v->ln_post_b });
    t.push_back({ D * (size_t)v->d_out, m->proj, &v->proj });
    for (int i = 0; i < v->L; i++) {
        const tc_vit_block_t &b = m->blocks[i];
        tcg_vit::Layer &y = v->layers[i];
        t.push_back({ D, b.ln1_g, &y.ln1_g });
        t.push_back({ D, b.ln1_b, &y.ln1_b });
        t.push_back({ 3 * D * D, b.qkv_w, nullptr });
        t.push_back({ 3 * D, b.qkv_b, &y.qkv_b });
        t.push_back({ D * D, b.out_w, nullptr });
        t.push_back({ D, b.out_b, &y.out_b });
        t.push_back({ D, b.ln2_g, &y.ln2_g });
        t.push_back({ D, b.ln2_b, &y.ln2_b });
        t.push_back({ F * D, b.up_w, nullptr });
        t.push_back({ F, b.up_b, &y.up_b });
        t.push_back({ D * F, b.down_w, nullptr });
        t.push_back({ D, b.down_b, &y.down_b });
    }
    return t;
}

// 1 (default): GEMM weights stored as Q4_K in the GGUF stay packed on the
// device (tcg_vit_set_packed_weights).
int g_vit_packed = 1;

// 1 (default): models whose weights are all fp32 run their GEMMs on fp16
// pieces (tcg_vit_set_f16); 0: on tf32 pairs.
int g_vit_f16 = 1;

// The GGUF tensor of a GEMM weight when it is kept packed: Q4_K rows of whole
// superblocks, read in place from the mapping.
static const gguf_tensor_t *packed_tensor(const tc_vit_t *m, const char *name)
{
    if (!g_vit_packed) return nullptr;
    const gguf_tensor_t *t = gguf_tensor(&m->gguf, name);
    if (!t || t->type != GGML_TYPE_Q4_K || !t->data || t->n_dims != 2 || t->dims[0] % 256) return nullptr;
    return t;
}

// Allocate the slabs and activation arena, point every field; weights are
// not copied here. qtable / qoff describe the packed GEMM weights (their
// bytes as 4-byte words) and their places in the packed slab.
static tcg_vit *vit_alloc(const tc_vit_t *m, int max_batch, std::vector<WEntry> &table,
                          std::vector<size_t> &offsets, std::vector<WEntry> &qtable, std::vector<size_t> &qoff)
{
    if (max_batch <= 0) { fail("tcg_vit_upload: max_batch must be positive"); return nullptr; }
    if (m->image % m->patch || m->d_model % m->n_head) { fail("tcg_vit_upload: inconsistent model dims"); return nullptr; }
    std::unique_ptr<tcg_vit> v(new tcg_vit());
    v->L = m->n_layer; v->D = m->d_model; v->H = m->n_head; v->hd = m->head_dim; v->F = m->d_ffn;
    v->P = m->patch; v->S = m->image; v->G = m->grid; v->T = m->n_token; v->d_out = m->d_out;
    v->eps = m->ln_eps; v->quick = m->quick_gelu; v->max_batch = max_batch; v->device = ctx().device;
    if (v->T != v->G * v->G + 1 || v->hd * v->H != v->D) { fail("tcg_vit_upload: inconsistent model dims"); return nullptr; }
    if ((v->D & 3) || (v->F & 3) || ((3 * v->P * v->P) & 3))
        { fail("tcg_vit_upload: d_model, d_ffn and 3*patch^2 must be multiples of 4"); return nullptr; }
    v->layers.resize(v->L);

    table = weight_table(v.get(), m);
    // GEMM weights kept packed: no fp32 copy on the device, their blocks in the
    // packed slab instead
    struct Packed {
        size_t entry;
        const gguf_tensor_t *t;
        const uint8_t **dst;
    };
    std::vector<Packed> packed;
    auto consider = [&](size_t entry, const char *name, const uint8_t **dst) {
        if (const gguf_tensor_t *t = packed_tensor(m, name)) packed.push_back({ entry, t, dst });
    };
    consider(0, "v.patch_embd.weight", &v->patch_q);
    for (int i = 0; i < v->L; i++) {
        const size_t b = 8 + 12 * (size_t)i;   // first entry of block i in weight_table
        char name[96];
        tcg_vit::Layer &y = v->layers[i];
        snprintf(name, sizeof name, "v.blk.%d.attn_qkv.weight", i); consider(b + 2, name, &y.qkv_q);
        snprintf(name, sizeof name, "v.blk.%d.attn_out.weight", i); consider(b + 4, name, &y.out_q);
        snprintf(name, sizeof name, "v.blk.%d.ffn_up.weight", i); consider(b + 8, name, &y.up_q);
        snprintf(name, sizeof name, "v.blk.%d.ffn_down.weight", i); consider(b + 10, name, &y.down_q);
    }
    qtable.clear();
    qoff.clear();
    size_t qfloats = 0;
    for (const Packed &pk : packed) {
        table[pk.entry].n = 0;
        qtable.push_back({ (size_t)pk.t->nbytes / 4, (const float *)pk.t->data, nullptr });
        qoff.push_back(qfloats);
        qfloats += align_floats((size_t)pk.t->nbytes / 4);
    }
    if (qfloats) {
        v->qslab_bytes = qfloats * 4;
        if (cudaMalloc(&v->qslab, v->qslab_bytes) != cudaSuccess) {
            cudaGetLastError();
            fail("tcg_vit_upload: cannot allocate %zu MB of packed weights", v->qslab_bytes >> 20);
            return nullptr;
        }
        for (size_t i = 0; i < packed.size(); i++) *packed[i].dst = v->qslab + 4 * qoff[i];
        size_t most = 0;
        for (const Packed &pk : packed) most = std::max(most, (size_t)pk.t->n_elem);
        if (cudaMalloc(&v->jit_hi, 2 * align_floats(most) * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            fail("tcg_vit_upload: cannot allocate %zu MB for dequantised weights", 8 * most >> 20);
            return nullptr;
        }
        v->jit_lo = v->jit_hi + align_floats(most);
    }
    v->f16 = g_vit_f16 && packed.empty() && v->D % 256 == 0 && v->F % 256 == 0;
    v->patch_f16 = v->f16 && (3 * v->P * v->P) % 256 == 0;
    offsets.resize(table.size());
    size_t total = 0;
    for (size_t i = 0; i < table.size(); i++) {
        offsets[i] = total;
        total += align_floats(table[i].n);
    }
    v->wslab_floats = total;
    if (cudaMalloc(&v->wslab, total * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        fail("tcg_vit_upload: cannot allocate %zu MB of weights", total * 4 >> 20);
        return nullptr;
    }
    for (size_t i = 0; i < table.size(); i++)
        if (table[i].dev) *table[i].dev = v->wslab + offsets[i];

    const size_t D = v->D, F = v->F, K0 = 3 * (size_t)v->P * v->P;
    // tf32 pairs of the GEMM weights that are not packed: sized, then placed
    float *s = nullptr;
    size_t need = 0;
    auto take = [&](size_t n, bool keep) -> float * {
        if (!keep) return nullptr;
        float *p = s ? s + need : nullptr;
        need += align_floats(n);
        return p;
    };
    // a weight of `rows` rows of n / rows: its tf32 pair, or its fp16 pieces
    // (n halves each) and one exponent per row
    auto take_w = [&](const float *&h, const float *&l, const int8_t *&e, size_t n, size_t rows, bool keep, bool f16) {
        if (!f16) {
            h = take(n, keep);
            l = take(n, keep);
            return;
        }
        h = take((n + 1) / 2, keep);
        l = take((n + 1) / 2, keep);
        e = (const int8_t *)take((rows + 3) / 4, keep);
    };
    auto place = [&]() {
        need = 0;
        take_w(v->patch_h, v->patch_l, v->patch_e, D * K0, D, !v->patch_q, v->patch_f16);
        for (auto &y : v->layers) {
            take_w(y.qkv_h, y.qkv_l, y.qkv_e, 3 * D * D, 3 * D, !y.qkv_q, v->f16);
            take_w(y.out_h, y.out_l, y.out_e, D * D, D, !y.out_q, v->f16);
            take_w(y.up_h, y.up_l, y.up_e, F * D, F, !y.up_q, v->f16);
            take_w(y.down_h, y.down_l, y.down_e, D * F, D, !y.down_q, v->f16);
        }
        v->projT_h = take(D * (size_t)v->d_out, true); v->projT_l = take(D * (size_t)v->d_out, true);
    };
    place();
    v->sslab_floats = need;
    if (cudaMalloc(&v->sslab, v->sslab_floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        fail("tcg_vit_upload: cannot allocate %zu MB of split weights", v->sslab_floats * 4 >> 20);
        return nullptr;
    }
    s = v->sslab;
    place();

    const size_t n = (size_t)max_batch, T = v->T, G2 = (size_t)v->G * v->G;
    const size_t f_floats = std::max(n * T * F, n * G2 * K0);
    const int ctas = ctx().sms > 0 ? ctx().sms : 148;
    const size_t ws_floats = gemm_work_ws_floats(ctas), flag_count = gemm_work_flag_count(ctas);
    const size_t e_bytes = n * T * (D + F) / 256 + n * G2 * K0 / 256 + 3 * 256 +   // fp16-piece exponents,
                           (n * T + 2 * (size_t)v->L) * sizeof(float) + 2 * 256;        // row norms, bounds
    const size_t want = (n * 3 * v->S * v->S + n * T * D * 3 + n * T * 3 * D + 2 * f_floats +
                         2 * n * D + n * v->d_out + ws_floats + flag_count) * sizeof(float) + e_bytes + 16 * 256;
    v->act = tcg_arena_create(want, "vit activations");
    if (!tcg_arena_ok(&v->act)) return nullptr;
    auto alloc = [&](size_t floats) { return (float *)tcg_arena_alloc(&v->act, floats * sizeof(float), 256); };
    v->px = alloc(n * 3 * v->S * v->S);
    v->x = alloc(n * T * D);
    v->h_hi = alloc(n * T * D);
    v->h_lo = alloc(n * T * D);
    v->qkv = alloc(n * T * 3 * D);
    v->f_hi = alloc(f_floats);
    v->f_lo = alloc(f_floats);
    v->pooled_hi = alloc(n * D);
    v->pooled_lo = alloc(n * D);
    v->out = alloc(n * v->d_out);
    v->p_hi = v->f_hi;
    v->p_lo = v->f_lo;
    if (v->f16) {
        v->h_e = (int8_t *)tcg_arena_alloc(&v->act, n * T * D / 256, 256);
        v->f_e = (int8_t *)tcg_arena_alloc(&v->act, n * T * F / 256, 256);
        v->p_e = v->patch_f16 ? (int8_t *)tcg_arena_alloc(&v->act, n * G2 * K0 / 256, 256) : nullptr;
        v->rnorm = alloc(n * T);
        v->up_bounds = alloc(2 * (size_t)v->L);
    }
    v->work.ws = alloc(ws_floats);
    v->work.flags = (int *)alloc(flag_count);
    v->work.ctas = ctas;
    if (!v->work.flags) return nullptr;
    if (cudaMemset(v->work.flags, 0, flag_count * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        fail("tcg_vit_upload: cannot clear the GEMM flags");
        return nullptr;
    }
    return v.release();
}

// Device-side split of the GEMM weights out of the fp32 slab.
static bool split_weights(tcg_vit *v, const std::vector<WEntry> &table, const std::vector<size_t> &off)
{
    cudaStream_t s = ctx().cur;
    const size_t D = v->D, F = v->F, K0 = 3 * (size_t)v->P * v->P;
    // packed weights have no fp32 copy to split
    auto split = [&](size_t entry, const float *hi, const float *lo, size_t n) {
        return !hi || launch_split(v->wslab + off[entry], (float *)hi, (float *)lo, n, s);
    };
    // fp16 pieces: rows x K, one exponent per row
    auto split16 = [&](size_t entry, const float *hi, const float *lo, const int8_t *e, size_t rows, size_t K) {
        return !hi || launch_split_f16(v->wslab + off[entry], (int)rows, (int)K, (void *)hi, (void *)lo,
                                       (int8_t *)e, 1, s);
    };
    if (!(v->patch_f16 ? split16(0, v->patch_h, v->patch_l, v->patch_e, D, K0) : split(0, v->patch_h, v->patch_l, D * K0)))
        return false;
    if (v->f16) TCG_CUDA(cudaMemsetAsync(v->up_bounds, 0, 2 * (size_t)v->L * sizeof(float), s));
    for (int i = 0; i < v->L; i++) {
        const size_t b = 8 + 12 * (size_t)i;   // first entry of block i in weight_table
        tcg_vit::Layer &y = v->layers[i];
        const bool ok = v->f16 ? split16(b + 2, y.qkv_h, y.qkv_l, y.qkv_e, 3 * D, D) &&
                                     split16(b + 4, y.out_h, y.out_l, y.out_e, D, D) &&
                                     split16(b + 8, y.up_h, y.up_l, y.up_e, F, D) &&
                                     split16(b + 10, y.down_h, y.down_l, y.down_e, D, F)
                               : split(b + 2, y.qkv_h, y.qkv_l, 3 * D * D) && split(b + 4, y.out_h, y.out_l, D * D) &&
                                     split(b + 8, y.up_h, y.up_l, F * D) && split(b + 10, y.down_h, y.down_l, D * F);
        if (!ok) return false;
        if (v->f16 && !launch_weight_bounds(v->wslab + off[b + 8], (int)F, (int)D, y.up_b, v->up_bounds + 2 * i, s))
            return false;
    }
    {   // v.proj is [D, d_out] (used untransposed, src/vit.c:384-386): store it as the [d_out, D] operand
        if (!launch_transpose_split(v->proj, v->D, v->d_out, (float *)v->projT_h, (float *)v->projT_l, s))
            return false;
    }
    (void)table;
    return true;
}

// Token rows from which packed weights are dequantised before their GEMMs
// (tcg_vit_set_jit_rows). Measured on ViT-B/32 with Q4_K block linears
// (B200, ms per forward, dequantised before the GEMM / inside it): batch 4
// 1.61 / 1.78, 32 2.55 / 4.11, 256 12.1 / 22.5 -- inside the GEMM every
// 128-row tile dequantises the whole weight again, so it only pays where a
// GEMM has a single row tile.
long g_vit_jit_rows = 129;

// One GEMM of the forward, after the dequantisation of its weight when the
// plan asks for it.
static bool run_gemm(const GemmPlan &p, cudaStream_t s, int *err)
{
    if (p.jit_q && !launch_dequant_split(p.jit_q, p.jit_hi, p.jit_lo, p.jit_n, GGML_TYPE_Q4_K, s)) return false;
    return gemm_run(p, s, err);
}

static tcg_vit::Plans *plans_for(tcg_vit *v, int n)
{
    auto it = v->plans.find(n);
    if (it != v->plans.end()) return it->second.get();
    std::unique_ptr<tcg_vit::Plans> p(new tcg_vit::Plans());
    const int D = v->D, F = v->F, T = v->T, G2 = v->G * v->G, K0 = 3 * v->P * v->P, M = n * T;

    GemmEpi e;
    e.rowadd = v->pos;
    e.ld_rowadd = D;
    e.rgroup = G2;
    e.rstride = T;
    e.roff = 1;
    e.out.plain = v->x;
    e.out.ld = D;
    const GemmWork *w = &v->work;
    const int tp = gemm_throughput_cfg();
    // A GEMM whose weight is packed dequantises it tile by tile in shared
    // memory when the batch is small (the weight read dominates); from
    // g_vit_jit_rows rows on, where every 128-row tile would dequantise the
    // whole weight again, the weight is dequantised once into the model's
    // tf32 pair (L2-resident) just before the GEMM, which then runs as usual.
    const bool jit = (long)n * T >= g_vit_jit_rows;
    auto plan = [&](GemmPlan &gp, const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
                    const uint8_t *bq, int Mg, int Ng, int Kg, GemmEpi ep) {
        if (bq && jit) {
            if (!gemm_plan(gp, a_hi, a_lo, v->jit_hi, v->jit_lo, Mg, Ng, Kg, ep, gemm_vit_cfg(Mg, Ng, Kg), w))
                return false;
            gp.jit_q = bq;
            gp.jit_hi = v->jit_hi;
            gp.jit_lo = v->jit_lo;
            gp.jit_n = (size_t)Ng * Kg;
            return true;
        }
        if (bq) {
            ep.bq = bq;
            ep.bq_row = (size_t)(Kg / 256) * 144;
            return gemm_plan(gp, a_hi, a_lo, nullptr, nullptr, Mg, Ng, Kg, ep, gemm_q4k_cfg(), w);
        }
        return gemm_plan(gp, a_hi, a_lo, b_hi, b_lo, Mg, Ng, Kg, ep, gemm_vit_cfg(Mg, Ng, Kg), w);
    };
    // fp16 pieces: A's exponents per (row, 256-column block), B's per row
    auto plan16 = [&](GemmPlan &gp, const void *a_hi, const void *a_lo, const int8_t *a_e, const float *b_hi,
                      const float *b_lo, const int8_t *b_e, int Mg, int Ng, int Kg, GemmEpi ep) {
        ep.xa = a_e;
        ep.xb = b_e;
        ep.xa_blk = 256;
        return gemm_plan(gp, (const float *)a_hi, (const float *)a_lo, b_hi, b_lo, Mg, Ng, Kg, ep, gemm_f16_cfg(), w);
    };
    const int Mp = n * G2;
    const bool ok_patch = v->patch_f16
        ? plan16(p->patch, v->f_lo, v->f_lo + (size_t)Mp * K0 / 2, v->p_e, v->patch_h, v->patch_l, v->patch_e, Mp, D,
                 K0, e)
        : plan(p->patch, v->p_hi, v->p_lo, v->patch_h, v->patch_l, v->patch_q, Mp, D, K0, e);
    if (!ok_patch) return nullptr;

    GemmEpi pe;                                   // embedding = pooled x proj, into v->out
    pe.out.plain = v->out;
    pe.out.ld = v->d_out;
    if (!gemm_plan(p->proj, v->pooled_hi, v->pooled_lo, v->projT_h, v->projT_l, n, v->d_out, D, pe, tp, w))
        return nullptr;

    p->qkv.resize(v->L); p->out.resize(v->L); p->up.resize(v->L); p->down.resize(v->L);
    for (int i = 0; i < v->L; i++) {
        const tcg_vit::Layer &y = v->layers[i];
        GemmEpi q;
        q.bias = y.qkv_b;
        q.out.plain = v->qkv;
        q.out.ld = 3 * D;
        GemmEpi o;
        o.bias = y.out_b;
        o.residual = v->x;
        o.out.plain = v->x;
        o.out.ld = D;
        GemmEpi u;
        u.bias = y.up_b;
        u.act = v->quick ? 2 : 1;
        const float *fp_lo0 = v->f_lo + (size_t)M * F / 2;   // the f pieces: hi halves, then lo halves
        if (v->f16) {
            // fp16 pieces of the GELU output, one exponent per row from LN2's row norm and the bounds
            u.out.fh = v->f_lo;
            u.out.fl = (void *)fp_lo0;
            u.out.fe = v->f_e;
            u.rnorm = v->rnorm;
            u.bounds = v->up_bounds + 2 * i;
        } else {
            u.out.hi = v->f_hi;
            u.out.lo = v->f_lo;
        }
        u.out.ld = F;
        GemmEpi d;
        d.bias = y.down_b;
        d.residual = v->x;
        d.out.plain = v->x;
        d.out.ld = D;
        if (v->f16) {
            GemmEpi d16 = d;
            d16.xa = v->f_e;                        // one exponent per row (the GELU output's bound)
            d16.xb = y.down_e;
            d16.xa_blk = 0;
            if (!plan16(p->qkv[i], v->h_hi, v->h_lo, v->h_e, y.qkv_h, y.qkv_l, y.qkv_e, M, 3 * D, D, q) ||
                !plan16(p->out[i], v->h_hi, v->h_lo, v->h_e, y.out_h, y.out_l, y.out_e, M, D, D, o) ||
                !plan16(p->up[i], v->h_hi, v->h_lo, v->h_e, y.up_h, y.up_l, y.up_e, M, F, D, u) ||
                !gemm_plan(p->down[i], v->f_lo, fp_lo0, y.down_h, y.down_l, M, D, F, d16, gemm_f16_cfg(), w))
                return nullptr;
            continue;
        }
        if (!plan(p->qkv[i], v->h_hi, v->h_lo, y.qkv_h, y.qkv_l, y.qkv_q, M, 3 * D, D, q) ||
            !plan(p->out[i], v->h_hi, v->h_lo, y.out_h, y.out_l, y.out_q, M, D, D, o) ||   // a aliases h
            !plan(p->up[i], v->h_hi, v->h_lo, y.up_h, y.up_l, y.up_q, M, F, D, u) ||
            !plan(p->down[i], v->f_hi, v->f_lo, y.down_h, y.down_l, y.down_q, M, D, F, d))
            return nullptr;
    }
    tcg_vit::Plans *raw = p.get();
    v->plans[n] = std::move(p);
    return raw;
}

typedef void (*TapFn)(void *ud, const char *name, const float *data, int rows, int cols);

// Optional CUDA-event bracketing of every launch of an eager forward, by
// kernel class, for the benchmark's per-kernel roofline figures.
enum { K_GEMM = 0, K_ATTN = 1, K_NORM = 2, K_OTHER = 3, K_KINDS = 4 };

struct Prof {
    std::vector<cudaEvent_t> pool;
    std::vector<int> kind;       // per recorded launch
    size_t used = 0;
    long launches = 0;           // all launches, profiled or not
    bool on = false;

    void begin(int k)
    {
        launches++;
        if (!on) return;
        if (used + 2 > pool.size()) {
            for (int i = 0; i < 256; i++) {
                cudaEvent_t e;
                cudaEventCreate(&e);
                pool.push_back(e);
            }
        }
        cudaEventRecord(pool[used], ctx().cur);
        kind.push_back(k);
    }
    void end()
    {
        if (!on) return;
        cudaEventRecord(pool[used + 1], ctx().cur);
        used += 2;
    }
};
static Prof g_prof;   // one benchmark thread drives it

#define PROF(kind, stmt)              \
    do {                              \
        g_prof.begin(kind);           \
        const bool ok_ = (stmt);      \
        g_prof.end();                 \
        if (!ok_) return false;       \
    } while (0)

// Host-side tap delivery: copy `rows_per_img` x D rows of each image (row
// stride ld between images) and call the user callback per image.
struct Tapper {
    TapFn fn;
    void *ud;
    float *host;          // staging, at least n*T*max(D, d_out) floats
    bool deliver(const char *name, const float *dev, int n, int rows, int cols, size_t img_stride)
    {
        if (!fn) return true;
        cudaStream_t s = ctx().cur;
        TCG_CUDA(cudaMemcpy2DAsync(host, (size_t)rows * cols * sizeof(float), dev, img_stride * sizeof(float),
                                   (size_t)rows * cols * sizeof(float), n, cudaMemcpyDeviceToHost, s));
        TCG_CUDA(cudaStreamSynchronize(s));
        for (int i = 0; i < n; i++) fn(ud, name, host + (size_t)i * rows * cols, rows, cols);
        return true;
    }
};

// Everything between the patch gather and the projection.
static bool forward_body(tcg_vit *v, tcg_vit::Plans *p, int n, Tapper *tap)
{
    cudaStream_t s = ctx().cur;
    int *err = ctx().d_err;
    const int D = v->D, T = v->T, M = n * T;
    OutSpec xs; xs.plain = v->x; xs.ld = D;
    OutSpec hs; hs.hi = v->h_hi; hs.lo = v->h_lo; hs.ld = D;

    PROF(K_GEMM, run_gemm(p->patch, s, err));
    PROF(K_OTHER, launch_cls_rows(v->x, v->cls, v->pos, n, T, D, s));
    PROF(K_NORM, launch_layernorm(v->x, D, v->ln_pre_g, v->ln_pre_b, M, D, v->eps, xs, s));
    if (tap && !tap->deliver("ln_pre", v->x, n, T, D, (size_t)T * D)) return false;

    // fp16 pieces: LayerNorm and the up projection write them; the attention
    // output goes through f_hi as fp32 and is split
    OutSpec h16; h16.fh = v->h_hi; h16.fl = v->h_lo; h16.fe = v->h_e; h16.fe_rows = M; h16.ld = D;
    OutSpec h16n = h16; h16n.rnorm = v->rnorm;     // LN2: also the row norms for the GELU output's scale
    OutSpec a32; a32.plain = v->f_hi; a32.ld = D;
    for (int i = 0; i < v->L; i++) {
        const tcg_vit::Layer &y = v->layers[i];
        if (v->f16) {
            PROF(K_NORM, launch_layernorm(v->x, D, y.ln1_g, y.ln1_b, M, D, v->eps, h16, s));
            PROF(K_GEMM, run_gemm(p->qkv[i], s, err));
            PROF(K_ATTN, launch_mha(v->qkv, v->qkv + D, v->qkv + 2 * D, 3 * D, T, v->H, v->hd, n, a32, s));
            PROF(K_OTHER, launch_split_f16(v->f_hi, M, D, v->h_hi, v->h_lo, v->h_e, 2, s));
            PROF(K_GEMM, run_gemm(p->out[i], s, err));
            PROF(K_NORM, launch_layernorm(v->x, D, y.ln2_g, y.ln2_b, M, D, v->eps, h16n, s));
            PROF(K_GEMM, run_gemm(p->up[i], s, err));
            PROF(K_GEMM, run_gemm(p->down[i], s, err));
        } else {
            PROF(K_NORM, launch_layernorm(v->x, D, y.ln1_g, y.ln1_b, M, D, v->eps, hs, s));
            PROF(K_GEMM, run_gemm(p->qkv[i], s, err));
            PROF(K_ATTN, launch_mha(v->qkv, v->qkv + D, v->qkv + 2 * D, 3 * D, T, v->H, v->hd, n, hs, s));
            PROF(K_GEMM, run_gemm(p->out[i], s, err));
            PROF(K_NORM, launch_layernorm(v->x, D, y.ln2_g, y.ln2_b, M, D, v->eps, hs, s));
            PROF(K_GEMM, run_gemm(p->up[i], s, err));
            PROF(K_GEMM, run_gemm(p->down[i], s, err));
        }
        if (tap && i == 0 && !tap->deliver("blk0", v->x, n, T, D, (size_t)T * D)) return false;
        if (tap && i == v->L - 1 && !tap->deliver("blk_last", v->x, n, T, D, (size_t)T * D)) return false;
    }

    if (tap) {
        // ln_post over every row (into the free qkv buffer) for the tap
        OutSpec ls; ls.plain = v->qkv; ls.ld = D;
        PROF(K_NORM, launch_layernorm(v->x, D, v->ln_post_g, v->ln_post_b, M, D, v->eps, ls, s));
        if (!tap->deliver("ln_post", v->qkv, n, T, D, (size_t)T * D)) return false;
    }
    // ln_post of the CLS rows as the tf32 pair the projection GEMM reads
    OutSpec ps; ps.hi = v->pooled_hi; ps.lo = v->pooled_lo; ps.ld = D;
    PROF(K_NORM, launch_layernorm(v->x, T * D, v->ln_post_g, v->ln_post_b, n, D, v->eps, ps, s));
    PROF(K_GEMM, run_gemm(p->proj, s, err));
    return true;
}

static bool forward(tcg_vit *v, const float *px, int n, float *out, Tapper *tap)
{
    if (ctx().device != v->device) return fail("model lives on device %d, thread uses %d", v->device, ctx().device);
    if (n <= 0) return true;
    if (n > v->max_batch) return fail("batch of %d exceeds the model's max_batch %d", n, v->max_batch);
    cudaStream_t s = ctx().cur;
    tcg_vit::Plans *p = plans_for(v, n);
    if (!p) return false;
    if (v->patch_f16) {
        // im2patch as fp32 rows, then their fp16 pieces
        const int Mp = n * v->G * v->G, K0 = 3 * v->P * v->P;
        PROF(K_OTHER, launch_patches(px, n, v->S, v->P, v->p_hi, nullptr, s));
        PROF(K_OTHER, launch_split_f16(v->p_hi, Mp, K0, v->f_lo, v->f_lo + (size_t)Mp * K0 / 2, v->p_e, 2, s));
    } else {
        PROF(K_OTHER, launch_patches(px, n, v->S, v->P, v->p_hi, v->p_lo, s));
    }
    if (tap || !v->graphs || g_prof.on) {
        if (!forward_body(v, p, n, tap)) return false;
    } else if (!p->graph) {
        // First call at this batch size: run eagerly (this also performs the
        // one-time kernel attribute setup outside any capture), then record
        // the same launches for the next calls.
        if (!forward_body(v, p, n, nullptr)) return false;
        cudaGraph_t g = nullptr;
        TCG_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        const bool ok = forward_body(v, p, n, nullptr);
        const cudaError_t ce = cudaStreamEndCapture(s, &g);
        if (!ok) { if (g) cudaGraphDestroy(g); return false; }
        TCG_CUDA(ce);
        const cudaError_t ie = cudaGraphInstantiate(&p->graph, g, 0);
        cudaGraphDestroy(g);
        TCG_CUDA(ie);
    } else {
        TCG_CUDA(cudaGraphLaunch(p->graph, s));
    }
    if (out != v->out)
        TCG_CUDA(cudaMemcpyAsync(out, v->out, (size_t)n * v->d_out * sizeof(float), cudaMemcpyDeviceToDevice, s));
    if (tap && !tap->deliver("embedding", out, n, 1, v->d_out, (size_t)v->d_out)) return false;
    return true;
}

// Kernel launches of one tap-free forward (graph or eager: the same kernels).
static int launches_per_forward(const tcg_vit *v) { return 2 + 4 + 7 * v->L; }

}  // namespace tcg

// ------------------------------------------------------------ weight upload
//
// The weights are zero-copy views into the GGUF mapping (src/gguf.h:3-10):
// pageable memory, which the copy engine cannot read directly. Three ways to
// move them into the device slab (tcg_vit_set_upload_mode):
//   0  one cudaMemcpyAsync per tensor from the mapping (the driver stages
//      pageable memory through its own pinned buffer, one chunk at a time);
//   1  staged (default): the mapping is read into two page-locked chunks in
//      turn by a few host threads while the copy engine moves the other chunk
//      to the device, so reading the mapping and the PCIe transfer overlap;
//   2  registered: the mapped data section is page-locked in place
//      (cudaHostRegister, read-only) and copied tensor by tensor.
int g_upload_mode = 1;
static thread_local double g_upload_ms = 0.0;
static thread_local std::string g_upload_fallback;    // why mode 2 fell back to the staged copy

using namespace tcg;

namespace {

constexpr size_t UP_CHUNK = 32u << 20;       // bytes per page-locked chunk
constexpr int UP_THREADS = 8;                // host threads filling a chunk

// The two page-locked chunks of a device, allocated by its first staged
// upload and kept for the life of the process (page-locking 64 MB costs tens
// of milliseconds, as much as the copy of a ViT-B/32); uploads to one device
// take turns on them.
struct UpStage {
    std::mutex mu;
    unsigned char *chunk[2] = { nullptr, nullptr };
    cudaEvent_t done[2] = { nullptr, nullptr };
};
UpStage g_up_stage[64];

// A piece of a tensor placed in a chunk: its device destination, its offset
// in the chunk, its host source and length.
struct UpPiece {
    float *dst;
    size_t at;
    const unsigned char *src;
    size_t bytes;
};

void fill_chunk(unsigned char *chunk, const std::vector<UpPiece> &pieces)
{
    // split the chunk's bytes evenly over the threads, piece boundaries aside
    size_t total = 0;
    for (const UpPiece &p : pieces) total += p.bytes;
    const size_t share = (total + UP_THREADS - 1) / UP_THREADS;
    auto work = [&](int t) {
        const size_t lo = share * t, hi = std::min(total, lo + share);
        size_t base = 0;
        for (const UpPiece &p : pieces) {
            const size_t a = std::max(lo, base), b = std::min(hi, base + p.bytes);
            if (a < b) memcpy(chunk + p.at + (a - base), p.src + (a - base), b - a);
            base += p.bytes;
        }
    };
    std::vector<std::thread> ts;
    for (int t = 1; t < UP_THREADS; t++) ts.emplace_back(work, t);
    work(0);
    for (std::thread &t : ts) t.join();
}

bool upload_staged(const std::vector<WEntry> &table, const std::vector<size_t> &off, float *slab, cudaStream_t s)
{
    UpStage &st = g_up_stage[ctx().device & 63];
    std::lock_guard<std::mutex> lock(st.mu);
    unsigned char **chunk = st.chunk;
    cudaEvent_t *done = st.done;
    bool ok = true;
    for (int b = 0; b < 2 && ok; b++) {
        if (!chunk[b] && cudaHostAlloc((void **)&chunk[b], UP_CHUNK, cudaHostAllocDefault) != cudaSuccess) {
            chunk[b] = nullptr;
            ok = false;
        }
        if (ok && !done[b] && cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming) != cudaSuccess) {
            done[b] = nullptr;
            ok = false;
        }
    }
    if (!ok) fail("weight upload: cannot allocate %zu MB of page-locked staging", 2 * UP_CHUNK >> 20);
    size_t ti = 0, toff = 0;                 // next tensor, bytes of it already placed
    for (int b = 0; ok && ti < table.size(); b ^= 1) {
        std::vector<UpPiece> pieces;
        size_t used = 0;
        while (ti < table.size() && used < UP_CHUNK) {
            const size_t bytes = table[ti].n * sizeof(float);
            const size_t take = std::min(bytes - toff, UP_CHUNK - used);
            pieces.push_back({ slab + off[ti] + toff / sizeof(float), used,
                               reinterpret_cast<const unsigned char *>(table[ti].host) + toff, take });
            used += (take + 15) & ~(size_t)15;
            toff += take;
            if (toff == bytes) { ti++; toff = 0; }
        }
        // the chunk's previous copies have left it before it is refilled
        if (cudaEventSynchronize(done[b]) != cudaSuccess) { ok = false; break; }
        fill_chunk(chunk[b], pieces);
        for (const UpPiece &p : pieces)
            if (cudaMemcpyAsync(p.dst, chunk[b] + p.at, p.bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) ok = false;
        if (ok && cudaEventRecord(done[b], s) != cudaSuccess) ok = false;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) ok = false;
    if (!ok) {
        cudaGetLastError();
        if (!tcg_last_error()[0]) fail("weight upload: staged copy failed");
    }
    return ok;
}

bool upload_registered(const tc_vit_t *m, const std::vector<WEntry> &table, const std::vector<size_t> &off,
                       float *slab, cudaStream_t s)
{
    // the page-aligned span of the mapping that holds the tensor data
    const size_t page = 4096;
    const uintptr_t a0 = (uintptr_t)m->gguf.data & ~(uintptr_t)(page - 1);
    const uintptr_t a1 = ((uintptr_t)m->gguf.data + m->gguf.data_size + page - 1) & ~(uintptr_t)(page - 1);
    const uintptr_t m0 = (uintptr_t)m->gguf.map, m1 = m0 + m->gguf.map_size;
    if (!m->gguf.data || a0 < m0 || a1 > ((m1 + page - 1) & ~(uintptr_t)(page - 1)))
        return fail("weight upload: tensor data outside the mapping");
    const cudaError_t re = cudaHostRegister((void *)a0, a1 - a0, cudaHostRegisterReadOnly);
    if (re != cudaSuccess) {
        cudaGetLastError();
        return fail("weight upload: cudaHostRegister of %zu MB failed: %s", (size_t)(a1 - a0) >> 20,
                    cudaGetErrorString(re));
    }
    bool ok = true;
    for (size_t i = 0; ok && i < table.size(); i++)
        ok = cudaMemcpyAsync(slab + off[i], table[i].host, table[i].n * sizeof(float), cudaMemcpyHostToDevice, s) ==
             cudaSuccess;
    if (cudaStreamSynchronize(s) != cudaSuccess) ok = false;
    cudaHostUnregister((void *)a0);
    if (!ok) {
        cudaGetLastError();
        return fail("weight upload: registered copy failed");
    }
    return true;
}

// The host weights of table into the slab, by the current mode; returns
// with the copies complete.
bool upload_tensors(const tc_vit_t *m, const std::vector<WEntry> &table, const std::vector<size_t> &off, float *slab,
                    cudaStream_t s)
{
    for (size_t i = 0; i < table.size(); i++)
        if (!table[i].host) return fail("weight upload: weight %zu unresolved", i);
    const auto t0 = std::chrono::steady_clock::now();
    g_upload_fallback.clear();
    bool ok;
    if (g_upload_mode == 1) {
        ok = upload_staged(table, off, slab, s);
    } else if (g_upload_mode == 2) {
        // where the system refuses to page-lock the file mapping (a memlock
        // limit, or no read-only registration), the staged copy does the work
        ok = upload_registered(m, table, off, slab, s);
        if (!ok) {
            g_upload_fallback = tcg_last_error();
            ok = upload_staged(table, off, slab, s);
        }
    } else {
        ok = true;
        for (size_t i = 0; ok && i < table.size(); i++)
            ok = cudaMemcpyAsync(slab + off[i], table[i].host, table[i].n * sizeof(float), cudaMemcpyHostToDevice,
                                 s) == cudaSuccess;
        if (cudaStreamSynchronize(s) != cudaSuccess) ok = false;
        if (!ok) {
            cudaGetLastError();
            fail("weight upload: copy failed");
        }
    }
    g_upload_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ok;
}

}  // namespace

extern "C" {

// Upload mode of later tcg_vit_upload / tcg_vit_upload_bcast calls (0 per
// tensor from the mapping, 1 staged through page-locked chunks, 2 mapping
// registered in place); returns the previous one.
int tcg_vit_set_upload_mode(int mode)
{
    const int old = g_upload_mode;
    if (mode >= 0 && mode <= 2) g_upload_mode = mode;
    return old;
}

// Wall time of this thread's latest host-to-device weight copy, ms.
double tcg_vit_last_upload_ms(void) { return g_upload_ms; }

// Test hook: why this thread's latest upload in mode 2 fell back to the
// staged copy ("" when it did not).
const char *tcg_vit_upload_fallback(void) { return g_upload_fallback.c_str(); }

tcg_vit_t *tcg_vit_upload(const tc_vit_t *m, int max_batch)
{
    if (!need_ctx()) return nullptr;
    std::vector<WEntry> table, qtable;
    std::vector<size_t> off, qoff;
    tcg_vit *v = vit_alloc(m, max_batch, table, off, qtable, qoff);
    if (!v) return nullptr;
    cudaStream_t s = ctx().cur;
    if (!upload_tensors(m, table, off, v->wslab, s) ||
        (!qtable.empty() && !upload_tensors(m, qtable, qoff, (float *)v->qslab, s))) {
        delete v;
        return nullptr;
    }
    if (!split_weights(v, table, off) || cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        delete v;
        if (!tcg_last_error()[0]) fail("tcg_vit_upload: weight preparation failed");
        return nullptr;
    }
    return v;
}

void tcg_vit_release(tcg_vit_t *v)
{
    if (!v) return;
    if (ctx().ready) cudaStreamSynchronize(ctx().cur);
    delete v;
}

int tcg_vit_max_batch(const tcg_vit_t *v) { return v ? v->max_batch : 0; }

size_t tcg_vit_device_bytes(const tcg_vit_t *v)
{
    return v ? (v->wslab_floats + v->sslab_floats) * sizeof(float) + v->qslab_bytes + v->act.cap : 0;
}

// Bytes of GEMM weights one forward reads: the tf32 pairs of the split ones
// and the Q4_K blocks of the packed ones.
size_t tcg_vit_gemm_weight_bytes(const tcg_vit_t *v)
{
    if (!v) return 0;
    const size_t pair = (v->sslab_floats - 2 * (size_t)v->D * v->d_out) * sizeof(float);   // all but the projection
    return pair + v->qslab_bytes;
}

// Token rows (batch x tokens) from which a forward dequantises each packed
// weight into a tf32 pair just before its GEMM instead of inside it; applies
// to batch sizes planned afterwards. Returns the previous value.
long tcg_vit_set_jit_rows(long rows)
{
    const long old = g_vit_jit_rows;
    if (rows > 0) g_vit_jit_rows = rows;
    return old;
}

// 1 (default): GEMM weights stored as Q4_K stay packed on the device at
// later uploads; 0 dequantises them at load like every other type. Returns
// the previous setting.
int tcg_vit_set_packed_weights(int on)
{
    const int old = g_vit_packed;
    g_vit_packed = on ? 1 : 0;
    return old;
}

int tcg_vit_set_f16(int on)
{
    const int old = g_vit_f16;
    g_vit_f16 = on ? 1 : 0;
    return old;
}

int tcg_vit_uses_f16(const tcg_vit_t *v) { return v && v->f16 ? 1 + (v->patch_f16 ? 1 : 0) : 0; }

void tcg_vit_use_graphs(tcg_vit_t *v, bool on)
{
    if (v) v->graphs = on;
}

bool tcg_vit_encode_device(tcg_vit_t *v, const float *pixels, int n_images, float *out)
{
    if (!need_ctx()) return false;
    if (!v) return fail("tcg_vit_encode_device: null model");
    return forward(v, pixels, n_images, out, nullptr);
}

int tcg_vit_launches_per_forward(const tcg_vit_t *v) { return v ? launches_per_forward(v) : 0; }

void tcg_vit_profile_begin(void)
{
    g_prof.kind.clear();
    g_prof.used = 0;
    g_prof.on = true;
}

bool tcg_vit_profile_end(float ms[4], int count[4])
{
    g_prof.on = false;
    for (int k = 0; k < K_KINDS; k++) { ms[k] = 0.0f; count[k] = 0; }
    if (!need_ctx()) return false;
    TCG_CUDA(cudaStreamSynchronize(ctx().cur));
    for (size_t i = 0; i < g_prof.kind.size(); i++) {
        float t = 0.0f;
        TCG_CUDA(cudaEventElapsedTime(&t, g_prof.pool[2 * i], g_prof.pool[2 * i + 1]));
        ms[g_prof.kind[i]] += t;
        count[g_prof.kind[i]]++;
    }
    g_prof.kind.clear();
    g_prof.used = 0;
    return true;
}

size_t tcg_vit_tap_staging_floats(const tcg_vit_t *v, int n_images)
{
    return v ? (size_t)n_images * v->T * (v->D > v->d_out ? v->D : v->d_out) : 0;
}

bool tcg_vit_encode_batch_staged(tcg_vit_t *v, const float *pixels, int n_images, float *out,
                                 tc_vit_tap_fn tap, void *ud, float *staging)
{
    if (!need_ctx()) return false;
    if (!v) return fail("tcg_vit_encode_batch: null model");
    if (n_images <= 0) return true;
    if (n_images > v->max_batch) return fail("batch of %d exceeds the model's max_batch %d", n_images, v->max_batch);
    if (tap && !staging) return fail("tcg_vit_encode_batch: no tap staging");
    for (int i = 0; i < 2; i++)         // finish asynchronous submissions first: they share the buffers
        if (v->in_flight[i]) {
            TCG_CUDA(cudaEventSynchronize(v->done[i]));
            v->in_flight[i] = false;
        }
    cudaStream_t s = ctx().cur;
    const size_t px_bytes = (size_t)n_images * 3 * v->S * v->S * sizeof(float);
    TCG_CUDA(cudaMemcpyAsync(v->px, pixels, px_bytes, cudaMemcpyHostToDevice, s));
    Tapper t{ (TapFn)tap, ud, staging };
    if (!forward(v, v->px, n_images, v->out, tap ? &t : nullptr)) return false;
    TCG_CUDA(cudaMemcpyAsync(out, v->out, (size_t)n_images * v->d_out * sizeof(float), cudaMemcpyDeviceToHost, s));
    TCG_CUDA(cudaStreamSynchronize(s));
    return true;
}

bool tcg_vit_submit(tcg_vit_t *v, const float *pixels, int n_images, float *out, int *ticket)
{
    if (!need_ctx()) return false;
    if (!v) return fail("tcg_vit_submit: null model");
    if (n_images <= 0 || n_images > v->max_batch)
        return fail("tcg_vit_submit: batch of %d outside 1..max_batch %d", n_images, v->max_batch);
    if (ctx().device != v->device) return fail("model lives on device %d, thread uses %d", v->device, ctx().device);
    const size_t px_bytes = (size_t)v->max_batch * 3 * v->S * v->S * sizeof(float);
    if (!v->copy_stream) {      // first submission: the second pixel slot and the copy stream
        TCG_CUDA(cudaStreamCreateWithFlags(&v->copy_stream, cudaStreamNonBlocking));
        for (int i = 0; i < 2; i++) {
            TCG_CUDA(cudaEventCreateWithFlags(&v->copied[i], cudaEventDisableTiming));
            TCG_CUDA(cudaEventCreateWithFlags(&v->done[i], cudaEventDisableTiming));
        }
        v->px_slot[0] = v->px;
        TCG_CUDA(cudaMalloc(&v->px_slot[1], px_bytes));
    }
    const int slot = v->next_ticket & 1;
    if (v->in_flight[slot]) {   // the submission two back used this slot: let it finish
        TCG_CUDA(cudaEventSynchronize(v->done[slot]));
        v->in_flight[slot] = false;
    }
    cudaStream_t s = ctx().cur;
    const size_t bytes = (size_t)n_images * 3 * v->S * v->S * sizeof(float);
    TCG_CUDA(cudaMemcpyAsync(v->px_slot[slot], pixels, bytes, cudaMemcpyHostToDevice, v->copy_stream));
    TCG_CUDA(cudaEventRecord(v->copied[slot], v->copy_stream));
    TCG_CUDA(cudaStreamWaitEvent(s, v->copied[slot], 0));
    if (!forward(v, v->px_slot[slot], n_images, v->out, nullptr)) return false;
    TCG_CUDA(cudaMemcpyAsync(out, v->out, (size_t)n_images * v->d_out * sizeof(float), cudaMemcpyDeviceToHost, s));
    TCG_CUDA(cudaEventRecord(v->done[slot], s));
    v->in_flight[slot] = true;
    if (ticket) *ticket = v->next_ticket;
    v->next_ticket++;
    return true;
}

bool tcg_vit_wait(tcg_vit_t *v, int ticket)
{
    if (!need_ctx()) return false;
    if (!v || ticket < 0 || ticket >= v->next_ticket) return fail("tcg_vit_wait: no such submission");
    const int slot = ticket & 1;
    if (!v->in_flight[slot]) return true;
    TCG_CUDA(cudaEventSynchronize(v->done[slot]));      // this ticket or the newer one in its slot
    if (ticket == v->next_ticket - 1 || ticket == v->next_ticket - 2) v->in_flight[slot] = false;
    return true;
}

bool tcg_vit_encode_batch(tcg_vit_t *v, const float *pixels, int n_images, float *out, tc_vit_tap_fn tap, void *ud)
{
    std::vector<float> staging;
    if (tap && v && n_images > 0) staging.resize(tcg_vit_tap_staging_floats(v, n_images));
    return tcg_vit_encode_batch_staged(v, pixels, n_images, out, tap, ud, tap ? staging.data() : nullptr);
}

tcg_vit_t *tcg_vit_upload_bcast(const tc_vit_t *m, int max_batch, int rank, int nranks, const unsigned char id[128])
{
    if (!need_ctx()) return nullptr;
    std::vector<WEntry> table, qtable;
    std::vector<size_t> off, qoff;
    tcg_vit *v = vit_alloc(m, max_batch, table, off, qtable, qoff);
    if (!v) return nullptr;
    cudaStream_t s = ctx().cur;
    bool ok = true;
    if (rank == 0)
        ok = upload_tensors(m, table, off, v->wslab, s) &&
             (qtable.empty() || upload_tensors(m, qtable, qoff, (float *)v->qslab, s));
    // every rank enters the collective, so a failed upload on rank 0 still
    // lets the others finish (they receive whatever rank 0 holds)
    // the packed slab too (every rank found the same packed tensors in its copy of the model)
    if (!broadcast_once(v->wslab, v->wslab_floats, rank, nranks, id, v->qslab, v->qslab_bytes / 4)) ok = false;
    if (ok) ok = split_weights(v, table, off) && cudaStreamSynchronize(s) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        delete v;
        return nullptr;
    }
    return v;
}

}  // extern "C"

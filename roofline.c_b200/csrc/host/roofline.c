/* roofline.c -- the B200 roofline of a GGUF model, replacing the fixed
 * 68 GB/s ceiling of roofline.c's tc-inspect (tools/tc_inspect.c:201-223).
 *
 * Same premise as the reference: weights are read once per unit of work (a
 * token for a decoder, an image at batch 1 for an encoder), so the memory
 * ceiling is HBM bandwidth / weight bytes. Added here: the compute ceiling
 * (tensor throughput / FLOPs per unit) and the batch at which the two meet.
 * For a clip-vit GGUF the FLOPs per image come from its metadata (patch
 * embedding, qkv / out / MLP GEMMs, attention, projection; elementwise work
 * left out); for anything else 2 FLOPs per weight per token. */
#include "tcg.h"

#include <math.h>
#include <string.h>

static uint64_t u64_key(const gguf_t *g, const char *k) { return gguf_u64_or(g, k, 0); }

bool tc_roofline_b200(const gguf_t *g, double hbm_gbs, double tensor_tflops, tc_roofline_t *out)
{
    if (!g || !out) return false;
    memset(out, 0, sizeof *out);
    if (!(hbm_gbs > 0.0) || !(tensor_tflops > 0.0)) return false;
    double bytes = 0.0, elems = 0.0;
    for (uint64_t i = 0; i < g->n_tensors; i++) {
        bytes += (double)g->tensors[i].nbytes;
        elems += (double)g->tensors[i].n_elem;
    }
    out->weight_bytes = bytes;
    out->hbm_gbs = hbm_gbs;
    out->tensor_tflops = tensor_tflops;
    gguf_str_t a;
    out->encoder = gguf_get_str(g, "general.architecture", &a) &&
                   (gguf_str_eq(a, "clip-vit") || gguf_str_eq(a, "clip-vit-fixtures"));
    if (out->encoder) {
        const double L = (double)u64_key(g, "clip-vit.block_count"), D = (double)u64_key(g, "clip-vit.embedding_length");
        const double F = (double)u64_key(g, "clip-vit.feed_forward_length"), P = (double)u64_key(g, "clip-vit.patch_size");
        const double S = (double)u64_key(g, "clip-vit.image_size"), E = (double)u64_key(g, "clip-vit.projection_dim");
        const double G2 = P > 0.0 ? floor(S / P) * floor(S / P) : 0.0, T = G2 + 1.0;
        out->flops_per_unit = 2.0 * G2 * D * 3.0 * P * P +
                              L * (2.0 * T * D * 3.0 * D + 2.0 * T * D * D + 4.0 * T * D * F + 4.0 * T * T * D) +
                              2.0 * D * E;
    } else {
        out->flops_per_unit = 2.0 * elems;
    }
    out->mem_units_per_s = bytes > 0.0 ? hbm_gbs * 1e9 / bytes : 0.0;
    out->compute_units_per_s = out->flops_per_unit > 0.0 ? tensor_tflops * 1e12 / out->flops_per_unit : 0.0;
    out->ridge_batch = out->mem_units_per_s > 0.0 ? out->compute_units_per_s / out->mem_units_per_s : 0.0;
    return true;
}

/* tc_inspect_b200.c -- `tc-inspect-b200 model.gguf [--hbm-gbs X] [--tflops Y]`:
 * the tensor summary of roofline.c's tc-inspect (tools/tc_inspect.c) with the
 * bandwidth ceiling computed for a B200 instead of the fixed 68 GB/s, plus
 * the compute ceiling. Defaults: 6545 GB/s HBM (a measured device-to-device
 * copy on B200) and 275 TFLOP/s, the fp32-accurate 3xTF32 rate (a measured
 * 1650 TFLOP/s dense bf16 / 2 for tf32 / 3 products); pass --tflops 1650
 * for a bf16 model. No GPU is needed. */
#include "tcg.h"

#include <inttypes.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char **argv)
{
    const char *path = NULL;
    double hbm = 6545.0, tflops = 275.0;
    for (int i = 1; i < argc; i++) {
        if (strcmp(argv[i], "--hbm-gbs") == 0 && i + 1 < argc) hbm = atof(argv[++i]);
        else if (strcmp(argv[i], "--tflops") == 0 && i + 1 < argc) tflops = atof(argv[++i]);
        else if (argv[i][0] != '-' && !path) path = argv[i];
        else {
            fprintf(stderr, "usage: tc-inspect-b200 <model.gguf> [--hbm-gbs X] [--tflops Y]\n");
            return 2;
        }
    }
    if (!path) {
        fprintf(stderr, "usage: tc-inspect-b200 <model.gguf> [--hbm-gbs X] [--tflops Y]\n");
        return 2;
    }
    arena_t a = arena_create((size_t)64 << 20, "inspect");
    gguf_t g;
    if (!gguf_open(&g, path, &a)) {
        fprintf(stderr, "tc-inspect-b200: %s\n", g.err);
        arena_destroy(&a);
        return 1;
    }
    /* bytes per ggml type */
    uint64_t count[64] = { 0 }, bytes[64] = { 0 };
    for (uint64_t i = 0; i < g.n_tensors; i++) {
        const int t = (int)g.tensors[i].type & 63;
        count[t]++;
        bytes[t] += g.tensors[i].nbytes;
    }
    printf("%s: GGUF v%u, %" PRIu64 " tensors, %" PRIu64 " metadata keys\n", path, g.version, g.n_tensors, g.n_kv);
    for (int t = 0; t < 64; t++)
        if (count[t]) printf("  %-6s %6" PRIu64 " tensors %14" PRIu64 " bytes\n", ggml_type_name((ggml_type_t)t), count[t], bytes[t]);
    tc_roofline_t r;
    if (!tc_roofline_b200(&g, hbm, tflops, &r)) {
        fprintf(stderr, "tc-inspect-b200: bad peaks\n");
        gguf_close(&g);
        arena_destroy(&a);
        return 1;
    }
    const char *unit = r.encoder ? "img/s" : "tok/s";
    printf("roofline on B200 (%.0f GB/s HBM, %.0f TFLOP/s):\n", r.hbm_gbs, r.tensor_tflops);
    printf("  weights          %.1f MB read per %s\n", r.weight_bytes / 1e6, r.encoder ? "image at batch 1" : "token");
    printf("  memory ceiling   %.1f %s at batch 1\n", r.mem_units_per_s, unit);
    printf("  compute ceiling  %.1f %s (%.4g GFLOP per %s)\n", r.compute_units_per_s, unit, r.flops_per_unit / 1e9,
           r.encoder ? "image" : "token");
    printf("  ridge            batch %.1f (compute-bound above)\n", r.ridge_batch);
    gguf_close(&g);
    arena_destroy(&a);
    return 0;
}

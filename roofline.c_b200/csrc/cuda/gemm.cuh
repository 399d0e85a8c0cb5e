// gemm.cuh -- the 3xTF32 tcgen05 GEMM that carries roofline.c's linears
// (tc_ref_linear, src/ops.c:28-35: y = x W^T + b) and its fused epilogues.
#pragma once

#include <cuda.h>
#include "ops.cuh"

namespace tcg {

// What happens to an accumulator element before it is stored.
//   v = acc                         (fp32 sum of the three tf32 products)
//   v = v + bias[n]                 if bias
//   v = v + rowadd[src_row, n]      if rowadd (position embedding)
//   v = act(v)                      act: 0 none, 1 gelu, 2 quick gelu
//   v = residual[dst_row, n] + v    if residual (may alias out.plain)
// GEMM row r is stored at dst_row(r) = (r / rgroup) * rstride + roff + r % rgroup,
// and rowadd's row is src_row(r) = r % rgroup + roff.
struct GemmEpi {
    const float *bias = nullptr;
    const float *rowadd = nullptr;
    int ld_rowadd = 0;
    const float *residual = nullptr;
    int act = 0;
    OutSpec out;
    int rgroup = 1 << 30, rstride = 0, roff = 0;
    // set by gemm_plan: N, every leading dimension a multiple of 4 and every
    // pointer 16-byte aligned, so the epilogue may move float4s
    bool vec = false;
    // set by gemm_plan: vec, no row remapping and no rowadd; the outputs are
    // written by bulk tensor stores (GemmPlan's output maps)
    bool tma = false;
    // B held packed in Q4_K blocks (the packed-weight configurations): row n
    // of B at bq + n * bq_row bytes, 144 bytes per 256 weights. The kernel
    // dequantises each K-step into its tf32 hi/lo shared-memory tiles.
    const uint8_t *bq = nullptr;
    size_t bq_row = 0;
    // fp16-piece operands (the fp16 configuration): A row m's K-block c
    // (xa_blk elements) was scaled by 2^xa[c * M + m] before it was split
    // (undone in the drain), B row n by 2^xb[n] over all of K (per tile)
    const int8_t *xa = nullptr;
    const int8_t *xb = nullptr;
    int xa_blk = 128;        // elements per K-block of A (128 or 256: one TMEM chunk each; 0: one per row, xa[m])
    // fp16-piece output (out.fh, out.fl, out.fe: one exponent per row), the
    // exponent taken from a bound on every value of the row:
    // |value| <= rnorm[row] * bounds[0] + bounds[1] (the row's input norm times
    // the largest weight-row norm, plus the largest |bias|, which bounds a
    // linear layer's output and, after it, GELU's)
    const float *rnorm = nullptr;
    const float *bounds = nullptr;
};

// Device memory for the stream-K split of a GEMM's last, partial wave of
// tiles: one partial accumulator tile (128 x 256 fp32 at most) per CTA and one
// flag per epilogue warp of each CTA. The flags are zero between launches
// (each owner clears what it consumed), so a GemmWork serves any number of
// GEMMs that run one after another on one stream, never two at once.
struct GemmWork {
    float *ws = nullptr;
    int *flags = nullptr;
    int ctas = 0;        // CTAs it has room for
};
size_t gemm_work_ws_floats(int ctas);
size_t gemm_work_flag_count(int ctas);
GemmWork *ctx_gemm_work();                         // the context's own, allocated on first use
bool gemm_work_reset(const GemmWork &w, cudaStream_t s);   // zero the flags after an aborted launch

// One GEMM: C[M,N] = A[M,K] * B[N,K]^T with both operands given as tf32
// hi/lo pairs, row-major with row stride K. Tensor maps are encoded once.
struct GemmPlan {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
    CUtensorMap o_plain, o_hi, o_lo;     // output maps, 32 x 8 boxes (epi.tma)
    int M = 0, N = 0, K = 0;
    int cfg = -1;        // kernel configuration index
    int grid = 0;
    GemmEpi epi;
    GemmWork work;       // stream-K memory (null: every tile whole)
    int sk = 0;          // 1: the last partial wave of tiles is split by K chunks
    // set by callers that keep B packed but run this plan on tf32 pairs: the
    // Q4_K blocks to dequantise into (jit_hi, jit_lo) just before the GEMM
    const uint8_t *jit_q = nullptr;
    float *jit_hi = nullptr, *jit_lo = nullptr;
    size_t jit_n = 0;
};

// work: memory for stream-K; without it every tile is computed whole.
bool gemm_plan(GemmPlan &p, const float *a_hi, const float *a_lo, const float *b_hi, const float *b_lo,
               int M, int N, int K, const GemmEpi &epi, int force_cfg = -1, const GemmWork *work = nullptr);
bool gemm_run(const GemmPlan &p, cudaStream_t s, int *err);

// The configuration for throughput (the ViT forward): folded small terms,
// stream-K capable; the automatic choice (force_cfg -1) is the accurate one.
int gemm_throughput_cfg();
// the configuration of one ViT GEMM of M x N x K (gemm_tc.cu)
int gemm_vit_cfg(int M, int N, int K);

// Tile widths available (index = cfg); for tests and tuning.
int gemm_num_cfgs();
int gemm_cfg_bn(int cfg);
// The configuration whose B operand is Q4_K blocks (GemmEpi::bq).
int gemm_q4k_cfg();

}  // namespace tcg

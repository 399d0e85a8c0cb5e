/* tcg.h -- the C ABI of the B200 compute layer (libtcg.so).
 *
 * roofline.c has no backend layer (its ARCHITECTURE.md plans one as a
 * vtable); this is it, for one target: hand-written sm_100a kernels behind
 * plain C entry points taking raw pointers and sizes. Every function here
 * takes DEVICE pointers unless its comment says host. The host-buffer API of
 * the reference (dequant.h, vit.h) is built on top of these.
 *
 * Conventions
 *   - bool return; on false, tcg_last_error() holds a one-line reason
 *     (the reference's bool + err[256] convention, src/gguf.h:143).
 *   - All work is queued on the calling thread's library stream (created by
 *     tcg_init, replaceable with tcg_set_stream) and is asynchronous unless
 *     stated; tcg_sync() waits for it.
 *   - Nothing here falls back to the CPU: without a usable device every
 *     compute entry point returns false.
 */
#ifndef TCG_H
#define TCG_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "arena.h"
#include "gguf.h"
#include "vit.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- status */

const char *tcg_last_error(void);
const char *tcg_version(void);

/* --------------------------------------------------- device / stream */

/* Select `device` for this thread and create its stream. Idempotent. */
bool  tcg_init(int device);
int   tcg_device_count(void);
int   tcg_sm_count(void);
bool  tcg_sync(void);
void *tcg_get_stream(void);                 /* cudaStream_t                  */
bool  tcg_set_stream(void *stream);         /* NULL: back to the library's   */

/* Device-side failure flag shared by every kernel that waits on a barrier:
 * non-zero after a bounded wait gave up. Reading it synchronizes. Clearing it
 * also resets the op API's GEMM stream-K flags; a ViT model (tcg_vit_*) that
 * saw a device error is released and uploaded again. */
int   tcg_device_error(void);
bool  tcg_clear_device_error(void);

/* -------------------------------------------------- memory plumbing */

void *tcg_malloc(size_t bytes);
bool  tcg_free(void *p);
void *tcg_host_alloc(size_t bytes);         /* page-locked host memory       */
bool  tcg_host_free(void *p);
bool  tcg_h2d(void *dst, const void *src, size_t bytes);   /* async          */
bool  tcg_d2h(void *dst, const void *src, size_t bytes);   /* async          */
bool  tcg_d2d(void *dst, const void *src, size_t bytes);   /* async          */
bool  tcg_memset(void *dst, int value, size_t bytes);      /* async          */

/* Read every byte of a device buffer once (128-bit loads, nothing written):
 * the floor under a bandwidth-bound kernel on the same bytes, timed the same
 * way (the benchmark's ceiling for the matvec). Asynchronous. */
bool  tcg_read_ceiling(const void *p, size_t bytes);

/* Hold the library stream for `us` microseconds (1 thread, at most 20,000):
 * queued before a timed sequence of launches, it lets the host queue the
 * whole sequence first, so the sequence runs back to back. Asynchronous. */
bool  tcg_device_delay_us(int us);

/* CUDA events on the library stream, slots 0..63. elapsed() waits for b. */
bool  tcg_event_record(int slot);
float tcg_event_elapsed_ms(int slot_a, int slot_b);

/* ------------------------------------------------------ device arena
 * The reference's arena discipline (src/arena.h:37-69) over one device
 * allocation: bump, LIFO mark/release, no per-object free. */

typedef struct {
    unsigned char *base;   /* device address                                */
    size_t cap, used, peak;
    const char *name;
} tcg_arena_t;

tcg_arena_t tcg_arena_create(size_t cap, const char *name);
void   tcg_arena_destroy(tcg_arena_t *a);
bool   tcg_arena_ok(const tcg_arena_t *a);
void  *tcg_arena_alloc(tcg_arena_t *a, size_t size, size_t align);
size_t tcg_arena_mark(const tcg_arena_t *a);
void   tcg_arena_release(tcg_arena_t *a, size_t mark);
void   tcg_arena_reset(tcg_arena_t *a);

/* ------------------------------------------------ dequant (src/dequant.c)
 * Replaces tc_dequant (src/dequant.c:40-63) on device buffers: F32 copy,
 * F16 exact conversion (tc_f16_to_f32, src/dequant.c:5-38, for every one of
 * the 65,536 inputs), and the Q4_K / Q6_K arms the reference leaves for
 * later (src/dequant.c:60-61), bit-identical to ggml's block dequantization.
 * One warp per superblock, 128-bit loads and stores. */
bool tcg_dequant(float *dst, const void *src, size_t n, ggml_type_t t);

/* Replaces tc_dequant_view (src/dequant.c:65-80) with device memory from
 * `a`: the tensor's bytes are uploaded and converted to fp32. */
const float *tcg_dequant_view(const gguf_tensor_t *t, tcg_arena_t *a, bool *converted);

/* Raw upload of a tensor's payload (K-quant blocks stay packed for the
 * fused consumers). */
const void *tcg_tensor_upload(const gguf_tensor_t *t, tcg_arena_t *a);

/* ------------------------------------------ fused dequant-matvec (new)
 * y[N] = W[N,K] x[K] with W in Q4_K / Q6_K blocks (row-major, K a multiple
 * of 256), dequantized in registers and never written out; fp32
 * accumulation. Equivalent to tc_dequant followed by tc_ref_linear with M=1
 * (src/ops.c:28-35), up to summation order. */
bool tcg_matvec_q(float *y, const void *W, const float *x, int N, int K, ggml_type_t t);

/* Decode-pass promise for tcg_matvec_q (default 0): 1 asserts that no kernel
 * queued before a matvec writes its weight matrix (weights uploaded once).
 * Successive matvecs then overlap: each fetches its weights while the one
 * before it finishes, and reads x only after that one completes. Returns the
 * previous setting. */
int  tcg_matvec_set_static_weights(int on);

/* --------------------------------------------------- ops (src/ops.h)
 * Same argument order and meaning as the reference's tc_ref_* (src/ops.h:
 * 30-63), device pointers. GEMMs run on the tcgen05 tensor cores as 3xTF32
 * (fp32-accurate) when K*4 and the row strides are 16-byte multiples and the
 * pointers 16-byte aligned, else on an fp32 CUDA-core kernel. */
bool tcg_gemm(float *C, const float *A, const float *B, int M, int N, int K, bool b_transposed);
bool tcg_linear(float *y, const float *x, const float *W, const float *bias, int M, int N, int K);
/* The tf32 operand pair of the 3xTF32 GEMMs: hi = rn_tf32(v),
 * lo = rn_tf32(v - hi), so v = hi + lo to ~2^-22 relative. */
bool tcg_split_tf32(float *hi, float *lo, const float *src, size_t n);
/* tcg_linear on operands already held as tf32 pairs (both row-major with
 * row stride K, 16-byte aligned, K a multiple of 4): the tensor-core kernel
 * alone, for callers that keep weights split once and reuse them. */
bool tcg_linear_split(float *y, const float *x_hi, const float *x_lo, const float *w_hi, const float *w_lo,
                      const float *bias, int M, int N, int K);
/* tcg_linear for callers that must not have a call allocate device memory
 * (no counterpart in the reference): a latency-critical loop that cannot
 * afford the device-wide synchronization cudaFree brings, or a program that
 * divides the GPU's memory once at start-up with its own allocator. The tf32
 * copies of x and W go to a fixed array inside the library instead of
 * tcg_linear's grow-on-demand buffer, so the call itself never allocates
 * (tcg_init still sets up the device once, before).
 * Limits: K a positive multiple of 4, x and W 16-byte aligned, and
 * (M + N) * K at most TCG_NOALLOC_SCRATCH_BYTES / 8 (2,097,152 floats);
 * anything larger is refused with a message.
 * The array lives on every device that runs this call, from the first call
 * until the process exits. That first call on each device looks up the
 * array's device address, so make it before any stream capture. All calls
 * share the array: calls whose kernels could overlap on the GPU (other
 * streams or host threads) race on it and must be serialised by the caller. */
#define TCG_NOALLOC_SCRATCH_BYTES (16u << 20)
bool tcg_linear_noalloc(float *y, const float *x, const float *W, const float *bias, int M, int N, int K);
/* tcg_linear with W [N, K] kept packed in Q4_K blocks on the device (row n
 * at W + n * K/256 * 144 bytes; K a multiple of 256, x and W 16-byte
 * aligned): the tensor-core GEMM dequantises each tile of W into shared
 * memory with the dequant seam's exact rounding and splits it into its tf32
 * pair there, so W is read as 0.56 bytes per weight instead of 8. The result
 * equals dequantising W (tcg_dequant) and calling tcg_linear_split on the
 * split pair with the same tile shape. Other types are refused. */
bool tcg_linear_q(float *y, const float *x, const void *W, const float *bias, int M, int N, int K, ggml_type_t t);
bool tcg_layernorm(float *out, const float *x, const float *gamma, const float *beta,
                   int rows, int cols, float eps);
bool tcg_gelu(float *out, const float *x, size_t n);
bool tcg_gelu_quick(float *out, const float *x, size_t n);
bool tcg_softmax_rows(float *out, const float *x, int rows, int cols);
/* tc_ref_mha without the scratch argument: the scores stay on chip. */
bool tcg_mha(float *out, const float *q, const float *k, const float *v,
             int T, int n_head, int head_dim);
/* tcg_mha over n_img images whose q, k and v share one row of width
 * 3 * n_head * head_dim (one GEMM over the fused [3D, D] weight whose three
 * row blocks src/vit.c:271-278 applies as three linears; this library's ViT
 * encoder keeps that layout): image i's rows are i*T .. i*T + T - 1.
 * Output [n_img * T, n_head * head_dim] as fp32 (out) and/or as its tf32
 * hi/lo pair (out_hi, out_lo; both or neither). */
bool tcg_mha_images(float *out, float *out_hi, float *out_lo, const float *qkv,
                    int T, int n_head, int head_dim, int n_img);
bool tcg_add(float *out, const float *a, const float *b, size_t n);
bool tcg_scale(float *out, const float *x, float s, size_t n);

/* ------------------------------------------------- batched ViT (new)
 * The forward of tc_vit_encode (src/vit.c:305-391) over a batch of images.
 * Weights are uploaded once (fp32 plus the tf32 hi/lo split the 3xTF32
 * GEMMs consume); activations live in a device arena sized for max_batch. */

typedef struct tcg_vit tcg_vit_t;

tcg_vit_t *tcg_vit_upload(const tc_vit_t *m, int max_batch);
void       tcg_vit_release(tcg_vit_t *v);
int        tcg_vit_max_batch(const tcg_vit_t *v);
size_t     tcg_vit_device_bytes(const tcg_vit_t *v);
/* Record the layer loop as a CUDA graph per batch size (default on). */
void       tcg_vit_use_graphs(tcg_vit_t *v, bool on);
/* How later uploads move the weights from the GGUF mapping (pageable memory,
 * src/gguf.h:3-10) to the device: 0 one copy per tensor from the mapping,
 * 1 (default) through two page-locked chunks that host threads fill while
 * the copy engine drains the other, 2 the mapping page-locked in place
 * (cudaHostRegister, read-only; where the system refuses that, the staged
 * copy of mode 1). Returns the previous mode. */
int        tcg_vit_set_upload_mode(int mode);
/* Wall time of this thread's latest weight upload (the host-to-device part
 * of tcg_vit_upload, or of rank 0's tcg_vit_upload_bcast), milliseconds. */
double     tcg_vit_last_upload_ms(void);

/* 1 (default): GEMM weights stored as Q4_K in the GGUF (qkv, out, up, down,
 * patch embedding) stay packed on the device at later uploads, and their
 * GEMMs dequantise them tile by tile in shared memory (tcg_linear_q's
 * kernel); 0 uploads the fp32 copy tc_vit_load made. Returns the previous
 * setting. */
int        tcg_vit_set_packed_weights(int on);
/* From this many token rows (batch x tokens, default 129) a forward
 * dequantises each packed weight into a tf32 pair (L2-resident) just before
 * its GEMM instead of tile by tile inside it, where every 128-row tile would
 * redo the work. Applies to batch sizes planned afterwards; returns the
 * previous value. */
long       tcg_vit_set_jit_rows(long rows);
/* Bytes of GEMM weights one forward reads: the tf32 pairs or fp16 pieces of
 * the split weights plus the Q4_K blocks of the packed ones. */
size_t     tcg_vit_gemm_weight_bytes(const tcg_vit_t *v);
/* 1 (default): a model whose weights are all fp32 on the device, with
 * d_model and d_ffn multiples of 256, runs its GEMMs on fp16 pieces (every
 * operand split into two fp16 values of 11 significant bits after a
 * power-of-two scale per row or per 256-element block: the precision of a
 * tf32 pair at twice the tensor rate); the patch embedding too when 3*patch^2
 * is a multiple of 256. 0: tf32 pairs. Applies to later uploads; returns the
 * previous setting. */
int        tcg_vit_set_f16(int on);
/* 0: the model's GEMMs run on tf32 pairs; 1: on fp16 pieces except the patch
 * embedding; 2: all but the final projection on fp16 pieces. */
int        tcg_vit_uses_f16(const tcg_vit_t *v);

/* HOST buffers: pixels [n, 3, image, image] (already normalised), out
 * [n, d_out]. Copies in, runs, copies out, and returns after the result is
 * in `out`. `tap` (may be NULL) is called once per image per tap point
 * (ln_pre, blk0, blk_last, ln_post, embedding), in image order, with host
 * data. Page-locked buffers (tcg_host_alloc) make the copies asynchronous. */
bool tcg_vit_encode_batch(tcg_vit_t *v, const float *pixels, int n_images, float *out,
                          tc_vit_tap_fn tap, void *ud);

/* DEVICE buffers, asynchronous, no taps. */
bool tcg_vit_encode_device(tcg_vit_t *v, const float *pixels, int n_images, float *out);

/* HOST buffers, asynchronous (for serving loops): the pixels are copied in
 * on the model's own copy stream, the forward runs on the library stream
 * once they have landed, and the embeddings are copied to `out`; the call
 * returns at once with a ticket. Two submissions can be in flight (the
 * copy of one overlaps the forward of the other); a third waits for the
 * oldest. `pixels` and `out` must stay untouched until tcg_vit_wait
 * returns for that ticket; page-locked buffers make the copies truly
 * asynchronous. tcg_vit_encode_batch first finishes any pending submission. */
bool tcg_vit_submit(tcg_vit_t *v, const float *pixels, int n_images, float *out, int *ticket);
bool tcg_vit_wait(tcg_vit_t *v, int ticket);

/* Instrumentation. Kernel launches of one forward; and, between begin and
 * end, every forward runs eagerly with CUDA events around each launch, whose
 * device time end() sums per kernel class: [0] tensor-core GEMMs,
 * [1] attention, [2] LayerNorm, [3] the rest (gather, CLS rows, projection). */
int  tcg_vit_launches_per_forward(const tcg_vit_t *v);
void tcg_vit_profile_begin(void);
bool tcg_vit_profile_end(float ms[4], int count[4]);

/* ------------------------------------------- image preprocessing (new)
 * open_clip's eval transform, which the reference leaves to the caller
 * (src/vit.h:75-78) and whose parameters its GGUF records
 * (clip-vit.preprocess.*): resize the shorter side to `image` with Pillow's
 * resampling (the 8-bit result bit-identical to Pillow's Image.resize),
 * centre crop, x / 255, minus mean, divided by std. DEVICE buffers: rgb
 * [n, height, width, 3] uint8 interleaved, pixels [n, 3, image, image] fp32,
 * ready for tcg_vit_encode_device. interpolation 0 bicubic, 1 bilinear.
 * Asynchronous; uses the library's device scratch. */
bool tcg_preprocess_rgb8(float *pixels, const uint8_t *rgb, int n, int height, int width, int image,
                         const float mean[3], const float std[3], int interpolation);
/* The same with the model's image size, mean and std (tc_vit_load) and its
 * clip-vit.preprocess.interpolation / resize_mode keys (bicubic when absent;
 * any other filter or resize rule is refused). */
bool tcg_vit_preprocess(const tc_vit_t *m, float *pixels, const uint8_t *rgb, int n, int height, int width);

/* ------------------------------------------------ roofline (new)
 * The B200 roofline of a GGUF model, in place of the fixed 68 GB/s ceiling
 * of the reference's tc-inspect (tools/tc_inspect.c:201-223): weights read
 * once per unit of work (a token; an image at batch 1 for clip-vit), so the
 * memory ceiling is hbm_gbs / weight bytes; the compute ceiling is
 * tensor_tflops / FLOPs per unit (clip-vit: from its metadata; otherwise 2
 * per weight); ridge_batch is where they meet. Host only, no GPU. */
typedef struct {
    double weight_bytes, hbm_gbs, tensor_tflops;
    double flops_per_unit, mem_units_per_s, compute_units_per_s, ridge_batch;
    bool encoder;
} tc_roofline_t;
bool tc_roofline_b200(const gguf_t *g, double hbm_gbs, double tensor_tflops, tc_roofline_t *out);

/* ------------------------------------------------ multi-GPU (NCCL)
 * One process per GPU. Rank 0 creates the id and hands it to the others by
 * any host channel; every rank then calls tcg_vit_upload_bcast with its
 * own host model (only rank 0's weights are read: they are uploaded there
 * and broadcast over NVLink once, with no collective in the forward). */
bool tcg_nccl_unique_id(unsigned char id[128]);
tcg_vit_t *tcg_vit_upload_bcast(const tc_vit_t *m, int max_batch, int rank, int nranks,
                                const unsigned char id[128]);

#ifdef __cplusplus
}
#endif
#endif /* TCG_H */

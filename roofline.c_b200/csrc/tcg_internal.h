/* tcg_internal.h -- entry points shared between the C host layer and the
 * CUDA layer of libtcg that are not part of the public headers. */
#ifndef TCG_INTERNAL_H
#define TCG_INTERNAL_H

#include "tcg.h"

#ifdef __cplusplus
extern "C" {
#endif

/* tc_dequant's device path: host src -> device, convert, -> host dst. */
bool tcg_dequant_host(float *dst, const void *src, size_t n, ggml_type_t t);

/* tcg_vit_encode_batch with caller-provided host staging for the taps
 * (n * n_token * max(d_model, d_out) floats; unused when tap is NULL). */
bool tcg_vit_encode_batch_staged(tcg_vit_t *v, const float *pixels, int n_images, float *out,
                                 tc_vit_tap_fn tap, void *ud, float *staging);

/* Floats of tap staging tcg_vit_encode_batch_staged needs for n images. */
size_t tcg_vit_tap_staging_floats(const tcg_vit_t *v, int n_images);

#ifdef __cplusplus
}

namespace tcg {
// One NCCL communicator from `id`, rank 0's buf (and buf2, when given)
// broadcast to every rank over it, then the communicator is released.
bool broadcast_once(void *buf, size_t count_floats, int rank, int nranks, const unsigned char id[128],
                    void *buf2 = nullptr, size_t count2 = 0);
}
#endif

#endif /* TCG_INTERNAL_H */

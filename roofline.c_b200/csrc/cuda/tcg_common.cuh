// tcg_common.cuh -- shared host/device helpers of libtcg (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "tcg.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libtcg is written for sm_100a (B200) only"
#endif

namespace tcg {

// Per-thread library context: the selected device, its stream and the
// device-side error word that bounded waits write when they give up.
struct Ctx {
    bool ready = false;
    int device = -1;
    int sms = 0;
    cudaStream_t own = nullptr;   // created by tcg_init
    cudaStream_t cur = nullptr;   // own, or the caller's (tcg_set_stream)
    int *d_err = nullptr;         // device word, 0 = healthy
    cudaEvent_t ev[64] = {};
    void *scratch = nullptr;      // grow-only device scratch for the op API
    size_t scratch_bytes = 0;
    void *gemm_work = nullptr;    // the op API's GemmWork (gemm_tc.cu)
};

Ctx &ctx();
bool need_ctx();                                    // false + message if no device
bool fail(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
bool cuda_fail(cudaError_t e, const char *what, const char *file, int line);
void *scratch(size_t bytes);                        // ctx scratch, grown on demand

inline unsigned ceil_div(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

}  // namespace tcg

#define TCG_CUDA(call)                                                        \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) return tcg::cuda_fail(e_, #call, __FILE__, __LINE__); \
    } while (0)

// After a launch: catch configuration errors without synchronizing.
#define TCG_LAUNCHED() TCG_CUDA(cudaGetLastError())

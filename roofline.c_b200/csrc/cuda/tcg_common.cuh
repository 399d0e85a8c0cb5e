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
    void *stage = nullptr;        // grow-only device copies of host-buffer op calls (ops_api.cu)
    size_t stage_bytes = 0;
};

Ctx &ctx();
bool need_ctx();                                    // false + message if no device
bool fail(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
bool cuda_fail(cudaError_t e, const char *what, const char *file, int line);
void *scratch(size_t bytes);                        // ctx scratch, grown on demand
void *stage_buffer(size_t bytes);                   // ctx staging for host-buffer ops, grown on demand

inline unsigned ceil_div(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

// Programmatic dependent launch. A kernel launched with launch_pdl() is
// scheduled as the CTAs of the kernel before it on the stream retire, instead
// of after that kernel's completion has been processed; it does its local
// prologue (shared-memory barriers, TMEM allocation), then pdl_wait(), which
// returns once every earlier kernel of the stream has completed with its
// writes visible, before its first global load or store. No kernel signals
// its dependents early (griddepcontrol.launch_dependents): dependents that
// start during a tail crowd onto the few idle SMs and then run unbalanced.
// Without the launch attribute pdl_wait() does nothing.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

extern int g_pdl;   // 1: launch_pdl() sets the attribute (default); 0: plain stream order


// Fills attrs[0] with the PDL attribute when enabled; returns the count used.
inline unsigned pdl_attr(cudaLaunchAttribute *attrs)
{
    if (!g_pdl) return 0;
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    return 1;
}

template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*fn)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A &&...args)
{
    cudaLaunchAttribute attrs[1];
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    lc.attrs = attrs;
    lc.numAttrs = pdl_attr(attrs);
    return cudaLaunchKernelEx(&lc, fn, static_cast<A &&>(args)...);
}

}  // namespace tcg

#define TCG_CUDA(call)                                                        \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) return tcg::cuda_fail(e_, #call, __FILE__, __LINE__); \
    } while (0)

// After a launch: catch configuration errors without synchronizing.
#define TCG_LAUNCHED() TCG_CUDA(cudaGetLastError())

// noalloc.cu -- tcg_linear for callers that must not allocate device memory.
//
// tcg_linear (gemm_tc.cu) keeps the tf32 hi/lo copies of its two operands in
// a scratch buffer that the library cudaMallocs on first use and grows (a
// cudaFree + cudaMalloc) when a larger product comes along. Some callers
// cannot let a call do that:
//   * a latency-critical loop sharing the GPU with other streams -- cudaFree
//     synchronizes the whole device, and cudaMalloc may too;
//   * a host program whose device memory is carved up once at start-up by
//     its own allocator, where any later allocation can fail or fragment.
// tcg_linear_noalloc does the same computation with its scratch in a
// fixed-size array of this file instead: TCG_NOALLOC_SCRATCH_BYTES, held by
// every GPU that loads this part of the library until the process exits.
//
// Because every call shares that one array, calls whose kernels overlap on
// the GPU (other streams, other host threads on the same device) race on it;
// the caller serialises them. The array keeps the last call's contents;
// nothing in it has to start at zero, since each call writes every value it
// later reads.
#include "gemm.cuh"

#include <mutex>

namespace {

constexpr size_t SCRATCH_FLOATS = (size_t)TCG_NOALLOC_SCRATCH_BYTES / sizeof(float);

// The operand pairs of one call: x_hi, x_lo [M*K], w_hi, w_lo [N*K], each
// rounded up to a multiple of 4 floats (16 bytes) so every part stays
// TMA-aligned.
static __device__ __align__(256) float g_scratch[SCRATCH_FLOATS];

// Device address of g_scratch per device index. In host code `g_scratch`
// names a host-side stand-in, never a device address, so the address comes
// from cudaGetSymbolAddress with the device current (the first call on each
// device does this, which is why that first call belongs outside any stream
// capture). Host threads with their own contexts on one device may make
// that first call together: std::call_once lets exactly one of them look the
// address up and publishes it to the others.
float *g_scratch_dev[64];
cudaError_t g_scratch_err[64];
std::once_flag g_scratch_once[64];

}  // namespace

using namespace tcg;

extern "C" bool tcg_linear_noalloc(float *y, const float *x, const float *W, const float *bias, int M, int N, int K)
{
    if (!need_ctx()) return false;
    if (M < 0 || N < 0 || K < 0) return fail("tcg_linear_noalloc: negative size");
    if (M == 0 || N == 0) return true;
    if (K == 0 || (K & 3) || ((uintptr_t)x & 15) || ((uintptr_t)W & 15) || ((uintptr_t)y & 3))
        return fail("tcg_linear_noalloc: needs K a positive multiple of 4 and 16-byte-aligned x and W");
    const size_t xa = ((size_t)M * K + 3) & ~(size_t)3, wa = ((size_t)N * K + 3) & ~(size_t)3;
    if (2 * (xa + wa) > SCRATCH_FLOATS)
        return fail("tcg_linear_noalloc: (M + N) * K = %zu floats needs %zu bytes of scratch; the built-in "
                    "scratch holds %zu bytes ((M + N) * K up to %zu)",
                    ((size_t)M + N) * K, 2 * (xa + wa) * sizeof(float), (size_t)TCG_NOALLOC_SCRATCH_BYTES,
                    SCRATCH_FLOATS / 2);

    const int dev = ctx().device;
    if (dev < 0 || dev >= 64) return fail("tcg_linear_noalloc: device index %d out of range", dev);
    std::call_once(g_scratch_once[dev], [dev] {
        void *p = nullptr;
        g_scratch_err[dev] = cudaGetSymbolAddress(&p, g_scratch);
        if (g_scratch_err[dev] == cudaSuccess && !p) g_scratch_err[dev] = cudaErrorInvalidSymbol;
        if (g_scratch_err[dev] != cudaSuccess) cudaGetLastError();
        else g_scratch_dev[dev] = static_cast<float *>(p);
    });
    if (g_scratch_err[dev] != cudaSuccess)
        return fail("tcg_linear_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(g_scratch_err[dev]));
    float *xh = g_scratch_dev[dev], *xl = xh + xa, *wh = xl + xa, *wl = wh + wa;

    cudaStream_t s = ctx().cur;
    if (!launch_split(x, xh, xl, (size_t)M * K, s) || !launch_split(W, wh, wl, (size_t)N * K, s)) return false;
    GemmEpi e;
    e.bias = bias;
    e.out.plain = y;
    e.out.ld = N;
    GemmPlan p;
    if (!gemm_plan(p, xh, xl, wh, wl, M, N, K, e)) return false;
    return gemm_run(p, s, ctx().d_err);
}

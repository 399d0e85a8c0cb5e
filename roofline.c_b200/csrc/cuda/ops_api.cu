// ops_api.cu -- roofline.c's op API (src/ops.h:30-63) on host buffers.
//
// The reference's tc_ref_* take host arrays and return nothing. Here each one
// copies its inputs into the calling thread's staging buffer on the device
// (grown on demand, one cudaMalloc at a time), runs the sm_100a kernel of the
// matching tcg_* entry point on the library stream, copies the result back
// and waits for it. There is no CPU path: without a device, or when a copy,
// a kernel or a bounded device wait fails, the call reports the reason on
// stderr and aborts, since the reference's signatures leave no way to return
// an error.
#include "tcg_common.cuh"
#include "ops.h"

#include <stdio.h>
#include <stdlib.h>

namespace {

[[noreturn]] void die(const char *what, const char *why)
{
    fprintf(stderr, "libtcg %s: %s\n", what, why);
    fflush(stderr);
    abort();
}

// A thread that never called tcg_init gets $TCG_DEVICE (default 0).
void ensure_device(const char *what)
{
    if (tcg::ctx().ready) return;
    const char *e = getenv("TCG_DEVICE");
    if (!tcg_init(e && *e ? atoi(e) : 0)) die(what, tcg_last_error());
}

// The call's device arrays, carved from the staging buffer at 256-byte
// offsets: first sized (add), then placed (at).
struct Layout {
    size_t off[6] = {}, total = 0;
    int n = 0;
    void add(size_t floats)
    {
        off[n++] = total;
        total += (floats * sizeof(float) + 255) & ~(size_t)255;
    }
};

struct Call {
    const char *what;
    float *dev[6] = {};
    explicit Call(const char *w, const Layout &l) : what(w)
    {
        ensure_device(w);
        unsigned char *base = (unsigned char *)tcg::stage_buffer(l.total ? l.total : 256);
        if (!base) die(what, tcg_last_error());
        for (int i = 0; i < l.n; i++) dev[i] = (float *)(base + l.off[i]);
    }
    void in(int i, const float *h, size_t floats)
    {
        if (floats && !tcg_h2d(dev[i], h, floats * sizeof(float))) die(what, tcg_last_error());
    }
    void ok(bool launched)
    {
        if (!launched) die(what, tcg_last_error());
    }
    void out(float *h, int i, size_t floats)
    {
        if (floats && !tcg_d2h(h, dev[i], floats * sizeof(float))) die(what, tcg_last_error());
        if (!tcg_sync()) die(what, tcg_last_error());
        const int e = tcg_device_error();
        if (e != 0) {
            char msg[96];
            snprintf(msg, sizeof msg, "a bounded device wait gave up (code %d)", e);
            die(what, msg);
        }
    }
};

}  // namespace

extern "C" {

void tc_ref_gemm(float *C, const float *A, const float *B, int M, int N, int K, bool b_transposed)
{
    if (M <= 0 || N <= 0) return;
    const size_t a = (size_t)M * (K > 0 ? K : 0), b = (size_t)N * (K > 0 ? K : 0), c = (size_t)M * N;
    Layout l;
    l.add(a); l.add(b); l.add(c);
    Call x("tc_ref_gemm", l);
    x.in(0, A, a);
    x.in(1, B, b);
    x.ok(tcg_gemm(x.dev[2], x.dev[0], x.dev[1], M, N, K, b_transposed));
    x.out(C, 2, c);
}

void tc_ref_linear(float *y, const float *xin, const float *W, const float *bias, int M, int N, int K)
{
    if (M <= 0 || N <= 0) return;
    const size_t a = (size_t)M * (K > 0 ? K : 0), w = (size_t)N * (K > 0 ? K : 0), c = (size_t)M * N;
    Layout l;
    l.add(a); l.add(w); l.add(bias ? (size_t)N : 0); l.add(c);
    Call x("tc_ref_linear", l);
    x.in(0, xin, a);
    x.in(1, W, w);
    if (bias) x.in(2, bias, (size_t)N);
    x.ok(tcg_linear(x.dev[3], x.dev[0], x.dev[1], bias ? x.dev[2] : nullptr, M, N, K));
    x.out(y, 3, c);
}

void tc_ref_layernorm(float *out, const float *xin, const float *gamma, const float *beta, int rows, int cols,
                      float eps)
{
    if (rows <= 0 || cols <= 0) return;
    const size_t n = (size_t)rows * cols;
    Layout l;
    l.add(n); l.add((size_t)cols); l.add((size_t)cols); l.add(n);
    Call x("tc_ref_layernorm", l);
    x.in(0, xin, n);
    x.in(1, gamma, (size_t)cols);
    x.in(2, beta, (size_t)cols);
    x.ok(tcg_layernorm(x.dev[3], x.dev[0], x.dev[1], x.dev[2], rows, cols, eps));
    x.out(out, 3, n);
}

static void unary(const char *what, bool (*fn)(float *, const float *, size_t), float *out, const float *xin,
                  size_t n)
{
    if (n == 0) return;
    Layout l;
    l.add(n); l.add(n);
    Call x(what, l);
    x.in(0, xin, n);
    x.ok(fn(x.dev[1], x.dev[0], n));
    x.out(out, 1, n);
}

void tc_ref_gelu(float *out, const float *x, size_t n) { unary("tc_ref_gelu", tcg_gelu, out, x, n); }

void tc_ref_gelu_quick(float *out, const float *x, size_t n)
{
    unary("tc_ref_gelu_quick", tcg_gelu_quick, out, x, n);
}

void tc_ref_softmax_rows(float *out, const float *xin, int rows, int cols)
{
    if (rows <= 0 || cols <= 0) return;
    const size_t n = (size_t)rows * cols;
    Layout l;
    l.add(n); l.add(n);
    Call x("tc_ref_softmax_rows", l);
    x.in(0, xin, n);
    x.ok(tcg_softmax_rows(x.dev[1], x.dev[0], rows, cols));
    x.out(out, 1, n);
}

void tc_ref_mha(float *out, const float *q, const float *k, const float *v, int T, int n_head, int head_dim,
                float *scratch)
{
    (void)scratch;                       // the scores never leave the chip
    if (T <= 0 || n_head <= 0 || head_dim <= 0) return;
    const size_t n = (size_t)T * n_head * head_dim;
    Layout l;
    l.add(n); l.add(n); l.add(n); l.add(n);
    Call x("tc_ref_mha", l);
    x.in(0, q, n);
    x.in(1, k, n);
    x.in(2, v, n);
    x.ok(tcg_mha(x.dev[3], x.dev[0], x.dev[1], x.dev[2], T, n_head, head_dim));
    x.out(out, 3, n);
}

void tc_ref_add(float *out, const float *a, const float *b, size_t n)
{
    if (n == 0) return;
    Layout l;
    l.add(n); l.add(n); l.add(n);
    Call x("tc_ref_add", l);
    x.in(0, a, n);
    x.in(1, b, n);
    x.ok(tcg_add(x.dev[2], x.dev[0], x.dev[1], n));
    x.out(out, 2, n);
}

void tc_ref_scale(float *out, const float *xin, float s, size_t n)
{
    if (n == 0) return;
    Layout l;
    l.add(n); l.add(n);
    Call x("tc_ref_scale", l);
    x.in(0, xin, n);
    x.ok(tcg_scale(x.dev[1], x.dev[0], s, n));
    x.out(out, 1, n);
}

}  // extern "C"

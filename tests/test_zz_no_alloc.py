"""tcg_linear_noalloc: the linear layer for callers that must not have a
call allocate device memory (a latency-critical loop that cannot take the
device-wide synchronization of cudaFree, or a program whose device memory
is divided once at start-up). Its scratch is a fixed array inside the
library, shared by every call.

Checked here: two calls in a row, of different shapes, each against the
ordinary tcg_linear on the same inputs (within the GEMM tolerance of the
other GPU tests), and the refusal of a product too large for the array.
This file sorts last so that a run stopping at its first failure has run
every other test first; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import tcg

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-5


def _linear(fn, x, W, b):
    M, K = x.shape
    N = W.shape[0]
    with tcg.DeviceBuffer.from_array(x) as dx, tcg.DeviceBuffer.from_array(W) as dw, \
            tcg.DeviceBuffer.from_array(b) as db, tcg.DeviceBuffer(M * N * 4) as dy:
        tcg.check(fn(dy.ptr, dx.ptr, dw.ptr, db.ptr, M, N, K), fn.__name__)
        return dy.download((M, N))


def test_noalloc_matches_tcg_linear_on_two_calls(gpu):
    L = tcg.lib()
    rng = np.random.default_rng(11)
    for M, N, K in ((300, 768, 768), (129, 200, 588)):       # two calls in a row, different shapes
        x = rng.standard_normal((M, K)).astype(np.float32)
        W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32)
        want = _linear(L.tcg_linear, x, W, b)
        got = _linear(L.tcg_linear_noalloc, x, W, b)
        err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
        assert err <= GEMM_TOL, (M, N, K, err)
    assert L.tcg_device_error() == 0


def test_noalloc_refuses_what_does_not_fit(gpu):
    L = tcg.lib()
    limit = (16 << 20) // 8                                    # TCG_NOALLOC_SCRATCH_BYTES / 8 floats
    K = 1024
    M = limit // K                                             # (M + N) * K > limit with N = 64
    with tcg.DeviceBuffer(16) as d:
        assert not L.tcg_linear_noalloc(d.ptr, d.ptr, d.ptr, None, M, 64, K)
    assert b"scratch" in L.tcg_last_error()

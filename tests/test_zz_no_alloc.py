"""tcg_linear_noalloc: the linear layer for callers that must not have a
call allocate device memory (a latency-critical loop that cannot take the
device-wide synchronization of cudaFree, or a program whose device memory
is divided once at start-up). Its scratch is a fixed array inside the
library, shared by every call.

Checked here:
* two calls in a row, of different shapes, each against the ordinary
  tcg_linear on the same inputs and against the CPU oracle's linear, within
  the GEMM tolerance of the other GPU tests;
* the exact capacity: (M + N) * K = 2,097,152 floats fills the array to its
  last byte and is accepted (and correct), one K-row more is refused;
* that the calls leave the op API's own grow-on-demand scratch as it was.
This file sorts last so that a run stopping at its first failure has run
every other test first; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import oracle
import tcg

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-5
LIMIT = (16 << 20) // 8                  # TCG_NOALLOC_SCRATCH_BYTES / 8: (M + N) * K in floats


def _linear(fn, x, W, b):
    M, K = x.shape
    N = W.shape[0]
    with tcg.DeviceBuffer.from_array(x) as dx, tcg.DeviceBuffer.from_array(W) as dw, \
            tcg.DeviceBuffer.from_array(b) as db, tcg.DeviceBuffer(M * N * 4) as dy:
        tcg.check(fn(dy.ptr, dx.ptr, dw.ptr, db.ptr, M, N, K), fn.__name__)
        return dy.download((M, N))


def _rel(got, want):
    want = np.asarray(want, np.float64)
    return np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()


def _case(rng, M, N, K):
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    return x, W, b


def test_noalloc_matches_tcg_linear_and_oracle_on_two_calls(gpu):
    L = tcg.lib()
    rng = np.random.default_rng(11)
    cases = [_case(rng, M, N, K) for M, N, K in ((300, 768, 768), (129, 200, 588))]
    before = L.tcg_op_scratch_bytes()
    got = [_linear(L.tcg_linear_noalloc, *c) for c in cases]          # two calls in a row
    assert L.tcg_op_scratch_bytes() == before                         # nothing of the op API's grew
    for (x, W, b), g in zip(cases, got):
        M, K = x.shape
        N = W.shape[0]
        assert _rel(g, _linear(L.tcg_linear, x, W, b)) <= GEMM_TOL, (M, N, K)
        assert _rel(g, oracle.linear(x, W, b, M, N, K)) <= GEMM_TOL, (M, N, K)
    assert L.tcg_device_error() == 0


def test_noalloc_exact_capacity(gpu):
    L = tcg.lib()
    rng = np.random.default_rng(12)
    M, N, K = 1984, 64, 1024                                          # (M + N) * K == LIMIT
    assert (M + N) * K == LIMIT
    x, W, b = _case(rng, M, N, K)
    before = L.tcg_op_scratch_bytes()
    got = _linear(L.tcg_linear_noalloc, x, W, b)
    assert L.tcg_op_scratch_bytes() == before
    assert _rel(got, oracle.linear(x, W, b, M, N, K)) <= GEMM_TOL
    with tcg.DeviceBuffer(16) as d:                                    # one K-row more
        assert not L.tcg_linear_noalloc(d.ptr, d.ptr, d.ptr, None, M + 1, N, K)
    assert b"scratch" in L.tcg_last_error()
    assert L.tcg_device_error() == 0

"""Failure paths that can be exercised without faulting the GPU.

* A bounded device wait that runs out: the stream-K hand-over of the GEMM
  (a contributor CTA raises a flag that the tile's owner waits on) with the
  flags withheld by a test hook and a 2 ms limit. The owner gives up, the
  kernel winds down and returns, the device error word reads the wait's code
  (8), and after tcg_clear_device_error() the same GEMM is correct again.
  No trap, no bad address, no endless loop: the wait simply ends.
* Device-arena exhaustion: NULL plus a reason, mark/release still working
  (the reference's arena contract, src/arena.h:37-69, on device memory).
"""
import ctypes

import numpy as np
import pytest

import oracle
import tcg

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-5


def _put(a):
    return tcg.DeviceBuffer.from_array(np.ascontiguousarray(a, np.float32))


def test_streamk_wait_gives_up_and_recovers(gpu):
    L = tcg.lib()
    M, N, K = 1600, 768, 3072            # 78 tiles of 128 x 128, 12 chunks each: split over 148 CTAs
    rng = np.random.default_rng(5)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    want = oracle.linear(x, W, b, M, N, K)
    cfg = L.tcg_gemm_throughput_cfg()
    old_sk = L.tcg_gemm_set_streamk(2)
    assert L.tcg_device_error() == 0
    with _put(x) as dx, _put(W) as dw, _put(b) as db, tcg.DeviceBuffer(M * N * 4) as dy:
        try:
            assert L.tcg_test_gemm_withhold_flags(1, 2.0)
            try:
                tcg.check(L.tcg_linear_cfg(dy.ptr, dx.ptr, dw.ptr, db.ptr, M, N, K, cfg), "withheld")
                plan = (ctypes.c_int * 4)()
                L.tcg_gemm_last_plan(plan)
                assert plan[1] == 1, list(plan)          # the launch really used the hand-over
                assert L.tcg_sync()                      # the kernel returned
                assert L.tcg_device_error() == 8         # the owner's flag wait gave up
            finally:
                assert L.tcg_test_gemm_withhold_flags(0, 0.0)
            assert L.tcg_clear_device_error()
            assert L.tcg_device_error() == 0
            tcg.check(L.tcg_linear_cfg(dy.ptr, dx.ptr, dw.ptr, db.ptr, M, N, K, cfg), "after recovery")
            got = dy.download((M, N))
        finally:
            L.tcg_gemm_set_streamk(old_sk)
    err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert err <= GEMM_TOL, err
    assert L.tcg_device_error() == 0


def test_device_arena_exhaustion(gpu):
    L = tcg.lib()
    a = L.tcg_arena_create(1 << 20, b"small")
    assert L.tcg_arena_ok(ctypes.byref(a))
    try:
        p = L.tcg_arena_alloc(ctypes.byref(a), 600 << 10, 256)
        assert p and p % 256 == 0
        mark = L.tcg_arena_mark(ctypes.byref(a))
        assert not L.tcg_arena_alloc(ctypes.byref(a), 600 << 10, 256)     # 424 KiB left
        msg = L.tcg_last_error()
        assert b"exhausted" in msg and b"small" in msg, msg
        assert L.tcg_arena_mark(ctypes.byref(a)) == mark                  # a refusal leaves it as it was
        q = L.tcg_arena_alloc(ctypes.byref(a), (1 << 20) - (600 << 10), 256)
        assert q == p + (600 << 10)                                       # exactly the rest fits
        assert not L.tcg_arena_alloc(ctypes.byref(a), 1, 1)
        L.tcg_arena_release(ctypes.byref(a), mark)
        assert L.tcg_arena_alloc(ctypes.byref(a), 1024, 256) == q         # LIFO release
        assert a.peak == 1 << 20
        assert not L.tcg_arena_alloc(ctypes.byref(a), 16, 3)               # alignment not a power of two
        assert b"power of two" in L.tcg_last_error()
    finally:
        L.tcg_arena_destroy(ctypes.byref(a))
    assert not L.tcg_arena_ok(ctypes.byref(a))

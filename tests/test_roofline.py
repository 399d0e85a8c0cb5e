"""The B200 roofline of a GGUF model (tc_roofline_b200, bin/tc-inspect-b200),
which replaces the fixed 68 GB/s of the reference's tc-inspect
(tools/tc_inspect.c:201-223): the same weights-once-per-unit memory
ceiling, plus the compute ceiling and the ridge batch. Host only."""
import ctypes
import os
import subprocess

import pytest

import tcg
import tcg_gguf as G
from fixtures_io import GOLDEN

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "roofline.c_b200", "bin", "tc-inspect-b200")


def _roofline(path, hbm, tflops):
    L = tcg.lib()
    a = L.arena_create(64 << 20, b"t")
    g = tcg.Gguf()
    assert L.gguf_open(ctypes.byref(g), path.encode(), ctypes.byref(a)), g.err
    r = tcg.Roofline()
    try:
        assert L.tc_roofline_b200(ctypes.byref(g), hbm, tflops, ctypes.byref(r))
        assert not L.tc_roofline_b200(ctypes.byref(g), 0.0, tflops, ctypes.byref(r))
        assert L.tc_roofline_b200(ctypes.byref(g), hbm, tflops, ctypes.byref(r))
    finally:
        L.gguf_close(ctypes.byref(g))
        L.arena_destroy(ctypes.byref(a))
    return r


@pytest.mark.parametrize("name", ["vit-b32", "vit-l14"])
def test_encoder_roofline(cache_dir, name):
    path, cfg = G.cached_vit_gguf(cache_dir, name, 0, n_layer=2)
    r = _roofline(path, 6545.0, 275.0)
    assert r.encoder
    D, F, T, L = cfg["d_model"], cfg["d_ffn"], cfg["n_token"], cfg["n_layer"]
    G2, K0 = (cfg["image"] // cfg["patch"]) ** 2, 3 * cfg["patch"] ** 2
    flops = 2 * G2 * D * K0 + L * (2 * T * D * 3 * D + 2 * T * D * D + 4 * T * D * F + 4 * T * T * D) + 2 * D * cfg["d_out"]
    assert r.flops_per_unit == pytest.approx(flops, rel=1e-12)
    n_params = sum(w.size for w in G.make_vit_weights(cfg, 0).values())
    assert r.weight_bytes == 4 * n_params
    assert r.mem_units_per_s == pytest.approx(6545e9 / r.weight_bytes)
    assert r.compute_units_per_s == pytest.approx(275e12 / flops)
    assert r.ridge_batch == pytest.approx(r.compute_units_per_s / r.mem_units_per_s)


def test_decoder_rule_and_cli():
    path = os.path.join(GOLDEN, "ops.gguf")
    r = _roofline(path, 8000.0, 1000.0)
    assert not r.encoder
    assert r.mem_units_per_s == pytest.approx(8000e9 / r.weight_bytes)
    assert r.flops_per_unit == pytest.approx(2 * r.weight_bytes / 4)      # F32 fixture: 2 FLOPs per weight
    if not os.path.exists(CLI):
        pytest.skip("bin/tc-inspect-b200 not built")
    out = subprocess.run([CLI, path, "--hbm-gbs", "8000", "--tflops", "1000"], capture_output=True, text=True,
                         timeout=60)
    assert out.returncode == 0, out.stderr
    assert "roofline on B200 (8000 GB/s HBM, 1000 TFLOP/s)" in out.stdout
    assert "tok/s at batch 1" in out.stdout
    bad = subprocess.run([CLI, os.path.join(GOLDEN, "make_golden.py")], capture_output=True, text=True, timeout=60)
    assert bad.returncode == 1 and "not a GGUF" in bad.stderr

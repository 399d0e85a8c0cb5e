"""libtcg.so loads on a machine without a GPU and exports every function the
headers in include/ declare; compute entry points fail cleanly (false plus a
reason) when no device was selected, instead of computing anything on the
CPU."""
import ctypes as C
import threading

import numpy as np

import tcg


def test_every_declared_function_is_exported(tcg_lib):
    names = tcg.header_functions()
    assert len(names) > 80
    missing = [n for n in names if not hasattr(tcg_lib, n)]
    assert not missing, missing


def test_exports_are_only_the_public_prefixes(tcg_lib):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", tcg.LIB_PATH], capture_output=True, text=True).stdout
    syms = [l.split()[-1] for l in out.splitlines() if l.strip()]
    stray = [s for s in syms if not s.startswith(("tc_", "tcg_", "arena_", "gguf_", "ggml_"))]
    assert not stray, stray


def test_compute_without_device_fails_loudly(tcg_lib):
    result = {}

    def body():                      # a fresh thread has no device context
        dst = np.zeros(256, np.float32)
        src = np.zeros(144, np.uint8)
        result["dequant"] = tcg_lib.tcg_dequant(dst.ctypes.data, src.ctypes.data, 256, 12)
        result["dequant_err"] = tcg_lib.tcg_last_error()
        result["host"] = tcg_lib.tc_dequant(dst.ctypes.data, src.ctypes.data, 256, 12)
        result["mv"] = tcg_lib.tcg_matvec_q(None, None, None, 1, 256, 12)
        result["ln"] = tcg_lib.tcg_layernorm(None, None, None, None, 1, 4, C.c_float(1e-5))

    t = threading.Thread(target=body)
    t.start()
    t.join()
    assert result["dequant"] is False and b"tcg_init" in result["dequant_err"]
    assert result["host"] is False and result["mv"] is False and result["ln"] is False


def test_f32_dequant_is_a_host_copy(tcg_lib):
    # the F32 arm is the reference's memcpy (src/dequant.c:43-49); no device
    src = np.arange(10, dtype=np.float32)
    dst = np.zeros(10, np.float32)
    assert tcg_lib.tc_dequant(dst.ctypes.data, src.ctypes.data, 10, 0)
    assert np.array_equal(dst, src)
    assert not tcg_lib.tc_dequant(dst.ctypes.data, src.ctypes.data, 10, 13)   # Q5_K: none


def test_f16_scalar_matches_oracle(tcg_lib):
    import oracle
    want = oracle.f16_to_f32_all()
    h = np.arange(0, 65536, 97, dtype=np.uint16)
    got = np.array([tcg_lib.tc_f16_to_f32(int(v)) for v in h], np.float32)
    w = want[h]
    ok = np.isnan(w) & np.isnan(got) | (got.view(np.uint32) == w.view(np.uint32))
    assert ok.all()

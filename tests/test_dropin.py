"""The drop-in, checked by the reference's own test programs.

roofline.c's tests/test_arena.c, test_gguf.c and test_ops.c (with its
tests/tt.h) are compiled unmodified against this repository's include/
(arena.h, gguf.h, ops.h) and linked with libtcg.so instead of the
reference's library, by `make -C oracle droptests REF=<reference tree>`
(run by __graft_entry__.build() where the reference tree is present); the
binaries, in oracle/_ref/, travel with the repository. test_arena and
test_gguf exercise the host layer (arena, GGUF loader) and run here;
test_ops calls tc_ref_gemm / linear / layernorm / gelu / softmax / mha
(include/ops.h), which run on the GPU, against the reference's golden
vectors (tests/golden/ops.gguf is the byte copy of its tests/fixtures/
ops.gguf) with its own tolerances.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref")
GOLDEN = os.path.join(ROOT, "tests", "golden")


def _run(name, cwd=None):
    exe = os.path.join(BIN, f"test_{name}_tcg")
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (make -C oracle droptests REF=<reference tree>)")
    r = subprocess.run([exe], cwd=cwd, capture_output=True, text=True, timeout=600)
    libs = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert "libtcg.so" in libs and "libtcref" not in libs, libs
    return r


@pytest.mark.parametrize("name,checks", [("arena", 54), ("gguf", 71)])
def test_reference_host_tests_against_libtcg(name, checks):
    r = _run(name, cwd=ROOT)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"{checks} checks ok" in r.stdout, r.stdout


@pytest.mark.gpu
def test_reference_op_tests_against_libtcg(tmp_path):
    os.makedirs(tmp_path / "tests" / "fixtures")
    shutil.copyfile(os.path.join(GOLDEN, "ops.gguf"), tmp_path / "tests" / "fixtures" / "ops.gguf")
    r = _run("ops", cwd=str(tmp_path))
    assert r.returncode == 0, r.stdout + r.stderr
    assert "14 checks ok" in r.stdout, r.stdout

"""Readers for the committed golden fixtures (test infrastructure).

read_gguf() is a deliberately small, independent GGUF v3 reader (F32
tensors and scalar metadata only) so that the fixture checks do not depend
on the library under test.
"""
import os
import struct

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def read_gguf(path: str):
    buf = open(path, "rb").read()
    pos = 0

    def take(fmt):
        nonlocal pos
        vals = struct.unpack_from("<" + fmt, buf, pos)
        pos += struct.calcsize("<" + fmt)
        return vals

    def text():
        (n,) = take("Q")
        nonlocal pos
        s = buf[pos:pos + n].decode()
        pos += n
        return s

    magic, version, n_t, n_kv = take("IIQQ")
    assert magic == 0x46554747 and version in (2, 3)
    width = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
    kv = {}
    for _ in range(n_kv):
        key = text()
        (ty,) = take("I")
        if ty == 8:
            kv[key] = text()
        elif ty == 9:
            et, n = take("IQ")
            kv[key] = [text() for _ in range(n)] if et == 8 else list(take(width[et] * n))
        else:
            (kv[key],) = take(width[ty])
    infos = []
    for _ in range(n_t):
        name = text()
        (nd,) = take("I")
        dims = take("Q" * nd)
        ty, off = take("IQ")
        infos.append((name, dims, ty, off))
    align = kv.get("general.alignment", 32)
    data = (pos + align - 1) // align * align
    tensors = {}
    for name, dims, ty, off in infos:
        if ty != 0:
            continue
        n = int(np.prod(dims))
        arr = np.frombuffer(buf, np.float32, n, data + off).copy()
        tensors[name] = arr.reshape(tuple(reversed(dims)))
    return kv, tensors


def ops_golden():
    return read_gguf(os.path.join(GOLDEN, "ops.gguf"))


def kquant_golden():
    return dict(np.load(os.path.join(GOLDEN, "kquant_golden.npz")))


def vit_golden():
    return dict(np.load(os.path.join(GOLDEN, "vit_golden.npz")))


def vit_bench_golden():
    return dict(np.load(os.path.join(GOLDEN, "vit_bench_golden.npz")))


def check_close(got, want, atol, rtol, what=""):
    """The reference's op-test rule (tests/test_ops.c:53): fail only when
    BOTH the worst absolute and the worst relative error are exceeded."""
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    a = np.abs(got - want)
    scale = np.abs(want)
    r = np.where(scale > 1e-6, a / np.maximum(scale, 1e-300), 0.0)
    worst_abs, worst_rel = float(a.max(initial=0.0)), float(r.max(initial=0.0))
    assert not (worst_abs > atol and worst_rel > rtol), \
        f"{what}: abs {worst_abs:.3g} rel {worst_rel:.3g} [atol {atol} rtol {rtol}]"
    return worst_abs, worst_rel


def rel_inf(got, want):
    """max |got - want| / max |want| -- the parity measure of the ViT path."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))

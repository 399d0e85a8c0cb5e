"""The CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker or as the timed CPU
baseline. The product library never loads it.

Two libraries live here:
  * _build/liboracle.so -- the C restatement of roofline.c's path (oracle.h);
  * _ref/libtcref.so    -- roofline.c's own src/*.c compiled unmodified by
    `make -C oracle ref` (only where the reference tree is present; the .so
    then travels with the repository snapshot).
and, from `make -C oracle droptests`, the reference's own test programs
(_ref/test_{arena,gguf,ops}_tcg) compiled against include/ and linked with
the product library libtcg.so -- the drop-in check, run by tests/.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtcref.so")

F32, F16, Q4_K, Q6_K = 0, 1, 12, 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}

_fp = C.POINTER(C.c_float)


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def build(with_ref: bool = True, ref_dir: str | None = None) -> None:
    """Build the C restatement and, when `with_ref` and a reference source
    tree is named (`ref_dir`, else the TC_REFERENCE environment variable),
    the reference's own library."""
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    ref = ref_dir or os.environ.get("TC_REFERENCE")
    if with_ref and ref and os.path.isdir(os.path.join(ref, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + ref], check=True)
        # the reference's own test programs linked against libtcg.so (the
        # drop-in check), once the library is built
        if os.path.exists(os.path.join(os.path.dirname(HERE), "roofline.c_b200", "lib", "libtcg.so")):
            subprocess.run(["make", "-s", "-C", HERE, "droptests", "REF=" + ref], check=True)


_port = None


def port() -> C.CDLL:
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(with_ref=False)
        lib = C.CDLL(PORT_SO)
        vp, sz, i, f = C.c_void_p, C.c_size_t, C.c_int, C.c_float
        lib.orc_f16_to_f32.argtypes = [C.c_uint16]; lib.orc_f16_to_f32.restype = f
        lib.orc_dequant.argtypes = [vp, vp, sz, i]; lib.orc_dequant.restype = C.c_bool
        lib.orc_matvec_q.argtypes = [vp, vp, vp, i, i, i]; lib.orc_matvec_q.restype = C.c_bool
        lib.orc_gemm.argtypes = [vp, vp, vp, i, i, i, C.c_bool]
        lib.orc_linear.argtypes = [vp, vp, vp, vp, i, i, i]
        lib.orc_layernorm.argtypes = [vp, vp, vp, vp, i, i, f]
        lib.orc_gelu.argtypes = [vp, vp, sz]
        lib.orc_gelu_quick.argtypes = [vp, vp, sz]
        lib.orc_softmax_rows.argtypes = [vp, vp, i, i]
        lib.orc_mha.argtypes = [vp, vp, vp, vp, i, i, i]
        lib.orc_add.argtypes = [vp, vp, vp, sz]
        lib.orc_scale.argtypes = [vp, vp, f, sz]
        lib.orc_vit_forward.argtypes = [vp, vp, vp, vp, vp, vp, vp]
        lib.orc_vit_forward.restype = C.c_bool
        _port = lib
    return _port


def have_ref() -> bool:
    return os.path.exists(REF_SO)


# ------------------------------------------------------------ numpy wrappers

def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def dequant(raw: np.ndarray, n: int, qtype: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    raw = np.ascontiguousarray(raw)
    if not port().orc_dequant(_ptr(out), _ptr(raw), n, qtype):
        raise ValueError(f"oracle cannot dequantize type {qtype}")
    return out


def f16_to_f32_all() -> np.ndarray:
    h = np.arange(65536, dtype=np.uint16)
    return dequant(h, 65536, F16)


def matvec_q(raw: np.ndarray, x: np.ndarray, N: int, K: int, qtype: int) -> np.ndarray:
    y = np.empty(N, np.float32)
    x = f32(x)
    raw = np.ascontiguousarray(raw)
    if not port().orc_matvec_q(_ptr(y), _ptr(raw), _ptr(x), N, K, qtype):
        raise ValueError("oracle matvec failed")
    return y


def gemm(A, B, M, N, K, b_transposed=True):
    C_ = np.empty((M, N), np.float32)
    A, B = f32(A), f32(B)
    port().orc_gemm(_ptr(C_), _ptr(A), _ptr(B), M, N, K, b_transposed)
    return C_


def linear(x, W, b, M, N, K):
    y = np.empty((M, N), np.float32)
    x, W = f32(x), f32(W)
    b = f32(b) if b is not None else None
    port().orc_linear(_ptr(y), _ptr(x), _ptr(W), _ptr(b), M, N, K)
    return y


def layernorm(x, g, b, rows, cols, eps):
    out = np.empty((rows, cols), np.float32)
    x = f32(x)
    g = f32(g) if g is not None else None
    b = f32(b) if b is not None else None
    port().orc_layernorm(_ptr(out), _ptr(x), _ptr(g), _ptr(b), rows, cols, eps)
    return out


def gelu(x, quick=False):
    x = f32(x)
    out = np.empty_like(x)
    (port().orc_gelu_quick if quick else port().orc_gelu)(_ptr(out), _ptr(x), x.size)
    return out


def softmax_rows(x, rows, cols):
    x = f32(x)
    out = np.empty((rows, cols), np.float32)
    port().orc_softmax_rows(_ptr(out), _ptr(x), rows, cols)
    return out


def mha(q, k, v, T, H, HD):
    q, k, v = f32(q), f32(k), f32(v)
    out = np.empty((T, H * HD), np.float32)
    port().orc_mha(_ptr(out), _ptr(q), _ptr(k), _ptr(v), T, H, HD)
    return out


def add(a, b):
    a, b = f32(a), f32(b)
    out = np.empty_like(a)
    port().orc_add(_ptr(out), _ptr(a), _ptr(b), a.size)
    return out


def scale(x, s):
    x = f32(x)
    out = np.empty_like(x)
    port().orc_scale(_ptr(out), _ptr(x), s, x.size)
    return out


# ------------------------------------------------------------------ ViT

class _Block(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "ln1_g", "ln1_b", "qkv_w", "qkv_b", "out_w", "out_b",
        "ln2_g", "ln2_b", "up_w", "up_b", "down_w", "down_b")]


class _Vit(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("d_model", C.c_int), ("n_head", C.c_int),
                ("d_ffn", C.c_int), ("patch", C.c_int), ("image", C.c_int),
                ("d_out", C.c_int), ("ln_eps", C.c_float), ("quick_gelu", C.c_int)] + \
               [(n, C.c_void_p) for n in ("patch_embd", "cls_token", "pos_embd", "ln_pre_g",
                                          "ln_pre_b", "ln_post_g", "ln_post_b", "proj")] + \
               [("blocks", C.POINTER(_Block))]


class PortVit:
    """The oracle's ViT over numpy weights (the same dict a synthetic GGUF is
    written from)."""

    def __init__(self, cfg: dict, w: dict, quick_gelu: bool = False, eps: float = 1e-5):
        self.cfg, self.w = cfg, {k: f32(v) for k, v in w.items()}
        L = cfg["n_layer"]
        self._blocks = (_Block * L)()
        for i in range(L):
            p = f"v.blk.{i}."
            names = ["ln1.weight", "ln1.bias", "attn_qkv.weight", "attn_qkv.bias",
                     "attn_out.weight", "attn_out.bias", "ln2.weight", "ln2.bias",
                     "ffn_up.weight", "ffn_up.bias", "ffn_down.weight", "ffn_down.bias"]
            for field, n in zip(_Block._fields_, names):
                setattr(self._blocks[i], field[0], self.w[p + n].ctypes.data)
        m = _Vit()
        for k in ("n_layer", "d_model", "n_head", "d_ffn", "patch", "image", "d_out"):
            setattr(m, k, cfg[k])
        m.ln_eps, m.quick_gelu = eps, int(quick_gelu)
        for field, n in (("patch_embd", "v.patch_embd.weight"), ("cls_token", "v.cls_token"),
                         ("pos_embd", "v.pos_embd"), ("ln_pre_g", "v.ln_pre.weight"),
                         ("ln_pre_b", "v.ln_pre.bias"), ("ln_post_g", "v.ln_post.weight"),
                         ("ln_post_b", "v.ln_post.bias"), ("proj", "v.proj")):
            setattr(m, field, self.w[n].ctypes.data)
        m.blocks = self._blocks
        self._m = m

    def forward(self, pixels: np.ndarray, taps: bool = True) -> dict:
        cfg = self.cfg
        T, D = cfg["n_token"], cfg["d_model"]
        out = np.empty(cfg["d_out"], np.float32)
        tp = {k: np.empty((T, D), np.float32) for k in ("ln_pre", "blk0", "blk_last", "ln_post")} \
            if taps else {}
        px = f32(pixels)
        ok = port().orc_vit_forward(C.byref(self._m), _ptr(px), _ptr(out),
                                    *(_ptr(tp.get(k)) for k in ("ln_pre", "blk0", "blk_last", "ln_post")))
        if not ok:
            raise MemoryError("oracle ViT forward failed")
        tp["embedding"] = out
        return tp


# -------------------------------------------- the reference library itself

class RefLib:
    """roofline.c's unmodified C library (oracle/_ref/libtcref.so)."""

    TAP = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_int, C.c_int)

    def __init__(self):
        if not have_ref():
            raise FileNotFoundError(REF_SO)
        lib = C.CDLL(REF_SO)
        vp, sz, i = C.c_void_p, C.c_size_t, C.c_int
        lib.tc_ref_gemm.argtypes = [vp, vp, vp, i, i, i, C.c_bool]
        lib.tc_ref_linear.argtypes = [vp, vp, vp, vp, i, i, i]
        lib.tc_ref_layernorm.argtypes = [vp, vp, vp, vp, i, i, C.c_float]
        lib.tc_ref_gelu.argtypes = [vp, vp, sz]
        lib.tc_ref_gelu_quick.argtypes = [vp, vp, sz]
        lib.tc_ref_softmax_rows.argtypes = [vp, vp, i, i]
        lib.tc_ref_mha.argtypes = [vp, vp, vp, vp, i, i, i, vp]
        lib.tc_ref_add.argtypes = [vp, vp, vp, sz]
        lib.tc_ref_scale.argtypes = [vp, vp, C.c_float, sz]
        lib.tc_f16_to_f32.argtypes = [C.c_uint16]; lib.tc_f16_to_f32.restype = C.c_float
        lib.tc_dequant.argtypes = [vp, vp, sz, i]; lib.tc_dequant.restype = C.c_bool
        lib.arena_create.argtypes = [sz, C.c_char_p]
        lib.arena_create.restype = _Arena
        lib.arena_destroy.argtypes = [C.POINTER(_Arena)]
        lib.tc_vit_load.argtypes = [vp, C.c_char_p, C.POINTER(_Arena)]
        lib.tc_vit_load.restype = C.c_bool
        lib.tc_vit_encode.argtypes = [vp, vp, vp, C.POINTER(_Arena), vp, vp]
        lib.tc_vit_encode.restype = C.c_bool
        lib.tc_vit_free.argtypes = [vp]
        lib.tc_vit_scratch_bytes.argtypes = [vp]
        lib.tc_vit_scratch_bytes.restype = sz
        self.lib = lib


class _Arena(C.Structure):
    _fields_ = [("base", C.c_void_p), ("cap", C.c_size_t), ("used", C.c_size_t),
                ("peak", C.c_size_t), ("name", C.c_char_p)]


class RefVit:
    """tc_vit_load + tc_vit_encode of the reference, for one GGUF file. The
    model struct is kept as an opaque, generously sized byte buffer (its only
    field read here is the err string, at a fixed offset from the end is not
    assumed; errors are reported by the load's bool)."""

    def __init__(self, path: str, scratch_mb: int = 512):
        self.ref = RefLib()
        lib = self.ref.lib
        self._m = C.create_string_buffer(1 << 16)
        self._wa = lib.arena_create(1 << 30, b"weights")
        self._sa = lib.arena_create(scratch_mb << 20, b"scratch")
        if not lib.tc_vit_load(self._m, path.encode(), C.byref(self._wa)):
            raise RuntimeError(f"reference tc_vit_load failed for {path}")

    def encode(self, pixels: np.ndarray, d_out: int, taps: bool = False) -> dict:
        lib = self.ref.lib
        out = np.empty(d_out, np.float32)
        got = {}

        def cb(_ud, name, data, rows, cols):
            got[name.decode()] = np.ctypeslib.as_array(data, shape=(rows * cols,)).copy().reshape(rows, cols)

        tap = RefLib.TAP(cb) if taps else None
        px = f32(pixels)
        ok = lib.tc_vit_encode(self._m, _ptr(px), _ptr(out), C.byref(self._sa),
                               C.cast(tap, C.c_void_p) if tap else None, None)
        if not ok:
            raise RuntimeError("reference tc_vit_encode failed")
        got["embedding"] = out
        return got

    def close(self):
        lib = self.ref.lib
        lib.tc_vit_free(self._m)
        lib.arena_destroy(C.byref(self._wa))
        lib.arena_destroy(C.byref(self._sa))

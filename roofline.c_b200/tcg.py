"""ctypes binding of libtcg.so -- the Python mirror of the C ABI in include/.

The library is the product; this module only declares its signatures and
offers numpy conveniences. It never computes anything itself: if the shared
library is missing it raises, it does not fall back.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libtcg.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

F32, F16, Q4_K, Q6_K = 0, 1, 12, 14
QK_K = 256
BLOCK_BYTES = {F32: 4, F16: 2, Q4_K: 144, Q6_K: 210}
BLOCK_ELEMS = {F32: 1, F16: 1, Q4_K: 256, Q6_K: 256}

vp, sz, i32, f32, boolean = C.c_void_p, C.c_size_t, C.c_int, C.c_float, C.c_bool
TAP_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_int, C.c_int)


class TcgError(RuntimeError):
    pass


# ------------------------------------------------------------------ structs

class Arena(C.Structure):            # include/arena.h
    _fields_ = [("base", vp), ("cap", sz), ("used", sz), ("peak", sz), ("name", C.c_char_p)]


class GgufStr(C.Structure):          # include/gguf.h
    _fields_ = [("ptr", C.c_void_p), ("len", C.c_uint64)]

    def text(self) -> str:
        return C.string_at(self.ptr, self.len).decode() if self.ptr else ""


class GgufArr(C.Structure):
    _fields_ = [("type", C.c_int), ("len", C.c_uint64), ("data", vp), ("strs", C.POINTER(GgufStr))]


class GgufVal(C.Union):
    _fields_ = [("u8", C.c_uint8), ("i8", C.c_int8), ("u16", C.c_uint16), ("i16", C.c_int16),
                ("u32", C.c_uint32), ("i32", C.c_int32), ("f32", C.c_float), ("u64", C.c_uint64),
                ("i64", C.c_int64), ("f64", C.c_double), ("b", C.c_bool), ("str", GgufStr),
                ("arr", GgufArr)]


class GgufKV(C.Structure):
    _fields_ = [("key", GgufStr), ("type", C.c_int), ("v", GgufVal)]


class GgufTensor(C.Structure):
    _fields_ = [("name", GgufStr), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4), ("type", C.c_int),
                ("offset", C.c_uint64), ("data", vp), ("n_elem", C.c_uint64), ("nbytes", C.c_uint64)]


class Gguf(C.Structure):
    _fields_ = [("map", vp), ("map_size", sz), ("fd", C.c_int), ("version", C.c_uint32),
                ("alignment", C.c_uint32), ("n_kv", C.c_uint64), ("n_tensors", C.c_uint64),
                ("kv", C.POINTER(GgufKV)), ("tensors", C.POINTER(GgufTensor)), ("data", vp),
                ("data_size", sz), ("err", C.c_char * 256)]


class VitBlock(C.Structure):         # include/vit.h
    _fields_ = [(n, vp) for n in ("ln1_g", "ln1_b", "qkv_w", "qkv_b", "out_w", "out_b",
                                  "ln2_g", "ln2_b", "up_w", "up_b", "down_w", "down_b")]


class Vit(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "d_model", "n_head", "head_dim", "d_ffn", "patch",
                                       "image", "grid", "n_token", "d_out")] + \
               [("ln_eps", C.c_float), ("quick_gelu", C.c_bool), ("mean", C.c_float * 3),
                ("std", C.c_float * 3)] + \
               [(n, vp) for n in ("patch_embd", "cls_token", "pos_embd", "ln_pre_g", "ln_pre_b",
                                  "ln_post_g", "ln_post_b", "proj")] + \
               [("blocks", C.POINTER(VitBlock)), ("gguf", Gguf), ("weight_bytes", sz),
                ("err", C.c_char * 256), ("dev", vp)]


class Roofline(C.Structure):          # include/tcg.h tc_roofline_t
    _fields_ = [(n, C.c_double) for n in ("weight_bytes", "hbm_gbs", "tensor_tflops", "flops_per_unit",
                                          "mem_units_per_s", "compute_units_per_s", "ridge_batch")] + \
               [("encoder", C.c_bool)]


# (name, restype, argtypes) of every entry point the binding uses
_SIGS = [
    # arena.h
    ("arena_create", Arena, [sz, C.c_char_p]), ("arena_destroy", None, [C.POINTER(Arena)]),
    ("arena_ok", boolean, [C.POINTER(Arena)]), ("arena_alloc", vp, [C.POINTER(Arena), sz, sz]),
    ("arena_calloc", vp, [C.POINTER(Arena), sz, sz, sz]), ("arena_memdup", vp, [C.POINTER(Arena), vp, sz, sz]),
    ("arena_mark", sz, [C.POINTER(Arena)]), ("arena_release", None, [C.POINTER(Arena), sz]),
    ("arena_reset", None, [C.POINTER(Arena)]), ("arena_used", sz, [C.POINTER(Arena)]),
    ("arena_peak", sz, [C.POINTER(Arena)]), ("arena_avail", sz, [C.POINTER(Arena)]),
    ("arena_fmt_bytes", C.c_char_p, [C.c_char_p, sz, sz]),
    # gguf.h
    ("gguf_open", boolean, [C.POINTER(Gguf), C.c_char_p, C.POINTER(Arena)]),
    ("gguf_close", None, [C.POINTER(Gguf)]),
    ("gguf_find", C.POINTER(GgufKV), [C.POINTER(Gguf), C.c_char_p]),
    ("gguf_get_u64", boolean, [C.POINTER(Gguf), C.c_char_p, C.POINTER(C.c_uint64)]),
    ("gguf_get_i64", boolean, [C.POINTER(Gguf), C.c_char_p, C.POINTER(C.c_int64)]),
    ("gguf_get_f32", boolean, [C.POINTER(Gguf), C.c_char_p, C.POINTER(C.c_float)]),
    ("gguf_get_str", boolean, [C.POINTER(Gguf), C.c_char_p, C.POINTER(GgufStr)]),
    ("gguf_u64_or", C.c_uint64, [C.POINTER(Gguf), C.c_char_p, C.c_uint64]),
    ("gguf_f32_or", f32, [C.POINTER(Gguf), C.c_char_p, f32]),
    ("gguf_tensor", C.POINTER(GgufTensor), [C.POINTER(Gguf), C.c_char_p]),
    ("ggml_type_name", C.c_char_p, [C.c_int]), ("ggml_blck_size", C.c_uint32, [C.c_int]),
    ("ggml_type_size", sz, [C.c_int]), ("ggml_type_supported", boolean, [C.c_int]),
    ("gguf_type_name", C.c_char_p, [C.c_int]),
    ("gguf_str_cstr", C.c_char_p, [C.c_char_p, sz, GgufStr]), ("gguf_str_eq", boolean, [GgufStr, C.c_char_p]),
    # dequant.h
    ("tc_f16_to_f32", f32, [C.c_uint16]), ("tc_dequant", boolean, [vp, vp, sz, C.c_int]),
    ("tc_dequant_view", vp, [C.POINTER(GgufTensor), C.POINTER(Arena), C.POINTER(C.c_bool)]),
    # vit.h
    ("tc_vit_load", boolean, [C.POINTER(Vit), C.c_char_p, C.POINTER(Arena)]),
    ("tc_vit_free", None, [C.POINTER(Vit)]),
    ("tc_vit_encode", boolean, [C.POINTER(Vit), vp, vp, C.POINTER(Arena), vp, vp]),
    ("tc_vit_scratch_bytes", sz, [C.POINTER(Vit)]),
    # tcg.h
    ("tcg_last_error", C.c_char_p, []), ("tcg_version", C.c_char_p, []),
    ("tcg_init", boolean, [i32]), ("tcg_device_count", i32, []), ("tcg_sm_count", i32, []),
    ("tcg_sync", boolean, []), ("tcg_get_stream", vp, []), ("tcg_set_stream", boolean, [vp]),
    ("tcg_device_error", i32, []), ("tcg_clear_device_error", boolean, []),
    ("tcg_malloc", vp, [sz]), ("tcg_free", boolean, [vp]),
    ("tcg_host_alloc", vp, [sz]), ("tcg_host_free", boolean, [vp]),
    ("tcg_h2d", boolean, [vp, vp, sz]), ("tcg_d2h", boolean, [vp, vp, sz]),
    ("tcg_d2d", boolean, [vp, vp, sz]), ("tcg_memset", boolean, [vp, i32, sz]),
    ("tcg_read_ceiling", boolean, [vp, sz]), ("tcg_device_delay_us", boolean, [i32]),
    ("tcg_event_record", boolean, [i32]), ("tcg_event_elapsed_ms", f32, [i32, i32]),
    ("tcg_arena_create", Arena, [sz, C.c_char_p]), ("tcg_arena_destroy", None, [C.POINTER(Arena)]),
    ("tcg_arena_ok", boolean, [C.POINTER(Arena)]), ("tcg_arena_alloc", vp, [C.POINTER(Arena), sz, sz]),
    ("tcg_arena_mark", sz, [C.POINTER(Arena)]), ("tcg_arena_release", None, [C.POINTER(Arena), sz]),
    ("tcg_arena_reset", None, [C.POINTER(Arena)]),
    ("tcg_dequant", boolean, [vp, vp, sz, C.c_int]),
    ("tcg_dequant_view", vp, [C.POINTER(GgufTensor), C.POINTER(Arena), C.POINTER(C.c_bool)]),
    ("tcg_tensor_upload", vp, [C.POINTER(GgufTensor), C.POINTER(Arena)]),
    ("tcg_matvec_q", boolean, [vp, vp, vp, i32, i32, C.c_int]),
    ("tcg_gemm", boolean, [vp, vp, vp, i32, i32, i32, boolean]),
    ("tcg_linear", boolean, [vp, vp, vp, vp, i32, i32, i32]),
    ("tcg_linear_cfg", boolean, [vp, vp, vp, vp, i32, i32, i32, i32]),
    ("tcg_gemm_num_cfgs", i32, []), ("tcg_gemm_set_chunk_k", i32, [i32]), ("tcg_gemm_force_cfg", i32, [i32]),
    ("tcg_gemm_set_streamk", i32, [i32]), ("tcg_set_pdl", i32, [i32]),
    ("tcg_gemm_last_plan", None, [C.POINTER(C.c_int)]), ("tcg_gemm_set_tma_store", i32, [i32]),
    ("tcg_set_attention_variant", i32, [i32]), ("tcg_set_attention_short_kernel", i32, [i32]),
    ("tcg_matvec_last_kernel", i32, []), ("tcg_matvec_set_tc", i32, [i32]),
    ("tcg_matvec_set_mma", i32, [i32]), ("tcg_matvec_mma_segments", i32, [i32]),
    ("tcg_matvec_set_static_weights", i32, [i32]), ("tcg_matvec_mma_slots", i32, [i32]), ("tcg_gemm_set_f16_cfg", i32, [i32]), ("tcg_matvec_mma_direct", i32, [i32]),
    ("tcg_matvec_mma_split", i32, [i32]), ("tcg_matvec_mma_tiles", i32, [i32]),
    ("tcg_split_tf32", boolean, [vp, vp, vp, sz]),
    ("tcg_test_gemm_withhold_flags", boolean, [i32, C.c_double]), ("tcg_gemm_throughput_cfg", i32, []),
    ("tcg_op_scratch_bytes", sz, []),
    ("tcg_linear_noalloc", boolean, [vp, vp, vp, vp, i32, i32, i32]),
    ("tcg_linear_q", boolean, [vp, vp, vp, vp, i32, i32, i32, C.c_int]),
    ("tcg_linear_split", boolean, [vp, vp, vp, vp, vp, vp, i32, i32, i32]),
    ("tcg_linear_split_cfg", boolean, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]),
    ("tcg_layernorm", boolean, [vp, vp, vp, vp, i32, i32, f32]),
    ("tcg_gelu", boolean, [vp, vp, sz]), ("tcg_gelu_quick", boolean, [vp, vp, sz]),
    ("tcg_softmax_rows", boolean, [vp, vp, i32, i32]),
    ("tcg_mha", boolean, [vp, vp, vp, vp, i32, i32, i32]),
    ("tcg_mha_images", boolean, [vp, vp, vp, vp, i32, i32, i32, i32]),
    ("tcg_split_f16", boolean, [vp, vp, vp, vp, i32, i32, i32]),
    ("tcg_layernorm_f16", boolean, [vp, vp, vp, vp, vp, vp, vp, i32, i32, C.c_float]),
    ("tcg_weight_bounds", boolean, [vp, vp, i32, i32, vp]),
    ("tcg_linear_f16_split", boolean, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]),
    ("tcg_add", boolean, [vp, vp, vp, sz]), ("tcg_scale", boolean, [vp, vp, f32, sz]),
    ("tcg_vit_upload", vp, [C.POINTER(Vit), i32]), ("tcg_vit_release", None, [vp]),
    ("tcg_vit_max_batch", i32, [vp]), ("tcg_vit_device_bytes", sz, [vp]),
    ("tcg_vit_use_graphs", None, [vp, boolean]),
    ("tcg_vit_set_upload_mode", i32, [i32]), ("tcg_vit_set_packed_weights", i32, [i32]),
    ("tcg_vit_set_f16", i32, [i32]), ("tcg_vit_uses_f16", i32, [vp]),
    ("tcg_vit_gemm_weight_bytes", sz, [vp]), ("tcg_vit_set_jit_rows", C.c_long, [C.c_long]), ("tcg_vit_last_upload_ms", C.c_double, []),
    ("tcg_vit_upload_fallback", C.c_char_p, []),
    ("tcg_vit_encode_batch", boolean, [vp, vp, i32, vp, vp, vp]),
    ("tcg_vit_encode_device", boolean, [vp, vp, i32, vp]),
    ("tcg_vit_submit", boolean, [vp, vp, i32, vp, C.POINTER(C.c_int)]),
    ("tcg_vit_wait", boolean, [vp, i32]),
    ("tcg_vit_launches_per_forward", i32, [vp]), ("tcg_vit_profile_begin", None, []),
    ("tcg_vit_profile_end", boolean, [C.POINTER(C.c_float), C.POINTER(C.c_int)]),
    ("tcg_preprocess_rgb8", boolean, [vp, vp, i32, i32, i32, i32, C.POINTER(C.c_float), C.POINTER(C.c_float), i32]),
    ("tcg_vit_preprocess", boolean, [C.POINTER(Vit), vp, vp, i32, i32, i32]),
    ("tc_roofline_b200", boolean, [C.POINTER(Gguf), C.c_double, C.c_double, C.POINTER(Roofline)]),
    ("tcg_nccl_unique_id", boolean, [C.c_char_p]),
    ("tcg_vit_upload_bcast", vp, [C.POINTER(Vit), i32, i32, i32, C.c_char_p]),
]

_lib = None


def lib() -> C.CDLL:
    """The loaded libtcg.so. Raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise TcgError(f"{LIB_PATH} is missing: build it with `make -C roofline.c_b200` "
                           "(or __graft_entry__.build())")
        h = C.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            fn = getattr(h, name)
            fn.restype, fn.argtypes = res, args
        _lib = h
    return _lib


def header_functions() -> list:
    """Every function declared in include/*.h (name only)."""
    names = []
    for fn in sorted(os.listdir(INCLUDE)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"#define[^\n]*", "", text)
        text = re.sub(r"typedef[^;]*;", "", text)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", text):
            name = m.group(1)
            if name not in ("sizeof", "__attribute__") and not name.startswith("_"):
                names.append(name)
    return sorted(set(names))


def err() -> str:
    return (lib().tcg_last_error() or b"").decode()


def check(ok, what="libtcg call"):
    if not ok:
        raise TcgError(f"{what}: {err()}")
    return ok


# ------------------------------------------------------------------ device

def init(device: int = 0) -> None:
    check(lib().tcg_init(device), "tcg_init")


def sync() -> None:
    check(lib().tcg_sync(), "tcg_sync")


class DeviceBuffer:
    """A raw device allocation (tcg_malloc), freed on close()."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        self.ptr = lib().tcg_malloc(max(self.nbytes, 1))
        if not self.ptr:
            raise TcgError(f"tcg_malloc({nbytes}): {err()}")

    @classmethod
    def from_array(cls, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        b.upload(a)
        return b

    def upload(self, a: np.ndarray, offset: int = 0) -> None:
        a = np.ascontiguousarray(a)
        check(lib().tcg_h2d(self.ptr + offset, a.ctypes.data, a.nbytes), "tcg_h2d")
        sync()

    def download(self, shape, dtype=np.float32, offset: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype)
        check(lib().tcg_d2h(out.ctypes.data, self.ptr + offset, out.nbytes), "tcg_d2h")
        sync()
        return out

    def close(self) -> None:
        if self.ptr:
            lib().tcg_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class HostBuffer:
    """Page-locked host memory (tcg_host_alloc) viewed as a numpy array."""

    def __init__(self, shape, dtype=np.float32):
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        self.ptr = lib().tcg_host_alloc(max(n, 1))
        if not self.ptr:
            raise TcgError(f"tcg_host_alloc({n}): {err()}")
        self.array = np.ctypeslib.as_array((C.c_byte * n).from_address(self.ptr)).view(dtype).reshape(shape)

    def close(self):
        if self.ptr:
            self.array = None
            lib().tcg_host_free(self.ptr)
            self.ptr = None


def time_ms(fn, slot_a: int = 0, slot_b: int = 1) -> float:
    """Device time of fn()'s work on the library stream (CUDA events)."""
    check(lib().tcg_event_record(slot_a), "tcg_event_record")
    fn()
    check(lib().tcg_event_record(slot_b), "tcg_event_record")
    return float(lib().tcg_event_elapsed_ms(slot_a, slot_b))


# ------------------------------------------------------------------ ViT

class VitModel:
    """tc_vit_load'ed model plus (optionally) its batched device copy."""

    def __init__(self, path: str, arena_bytes: int = 1 << 30):
        self.arena = lib().arena_create(arena_bytes, b"weights")
        if not self.arena.base:
            raise TcgError("arena_create failed")
        self.m = Vit()
        if not lib().tc_vit_load(C.byref(self.m), path.encode(), C.byref(self.arena)):
            msg = self.m.err.decode()
            lib().arena_destroy(C.byref(self.arena))
            raise TcgError(f"tc_vit_load({path}): {msg}")
        self.dev = None

    @property
    def cfg(self) -> dict:
        m = self.m
        return dict(n_layer=m.n_layer, d_model=m.d_model, n_head=m.n_head, d_ffn=m.d_ffn, patch=m.patch,
                    image=m.image, d_out=m.d_out, n_token=m.n_token)

    def upload(self, max_batch: int) -> None:
        self.dev = lib().tcg_vit_upload(C.byref(self.m), max_batch)
        if not self.dev:
            raise TcgError(f"tcg_vit_upload: {err()}")

    def upload_bcast(self, max_batch: int, rank: int, nranks: int, uid: bytes) -> None:
        self.dev = lib().tcg_vit_upload_bcast(C.byref(self.m), max_batch, rank, nranks, uid)
        if not self.dev:
            raise TcgError(f"tcg_vit_upload_bcast: {err()}")

    def encode(self, pixels: np.ndarray, taps: bool = False):
        """Batched host-buffer encode; returns (out [n, d_out], {tap: [n, rows, cols]})."""
        px = np.ascontiguousarray(pixels, np.float32)
        n = px.shape[0]
        out = np.empty((n, self.m.d_out), np.float32)
        got: dict = {}

        def cb(_ud, name, data, rows, cols):
            got.setdefault(name.decode(), []).append(
                np.ctypeslib.as_array(data, shape=(rows * cols,)).copy().reshape(rows, cols))

        tap = TAP_FN(cb) if taps else None
        check(lib().tcg_vit_encode_batch(self.dev, px.ctypes.data, n, out.ctypes.data,
                                         C.cast(tap, C.c_void_p) if tap else None, None),
              "tcg_vit_encode_batch")
        return out, {k: np.stack(v) for k, v in got.items()}

    def encode_single(self, pixels: np.ndarray, taps: bool = True):
        """The reference-shaped entry point tc_vit_encode (one image)."""
        px = np.ascontiguousarray(pixels, np.float32)
        out = np.empty(self.m.d_out, np.float32)
        scratch = lib().arena_create(lib().tc_vit_scratch_bytes(C.byref(self.m)) + (1 << 20), b"scratch")
        got: dict = {}

        def cb(_ud, name, data, rows, cols):
            got[name.decode()] = np.ctypeslib.as_array(data, shape=(rows * cols,)).copy().reshape(rows, cols)

        tap = TAP_FN(cb) if taps else None
        try:
            ok = lib().tc_vit_encode(C.byref(self.m), px.ctypes.data, out.ctypes.data, C.byref(scratch),
                                     C.cast(tap, C.c_void_p) if tap else None, None)
            if not ok:
                raise TcgError(f"tc_vit_encode: {self.m.err.decode()}")
        finally:
            lib().arena_destroy(C.byref(scratch))
        return out, got

    def close(self) -> None:
        if self.dev:
            lib().tcg_vit_release(self.dev)
            self.dev = None
        if self.m.dev:
            pass  # released by tc_vit_free
        lib().tc_vit_free(C.byref(self.m))
        lib().arena_destroy(C.byref(self.arena))

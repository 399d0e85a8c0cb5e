"""The host C layer of libtcg.so (arena.h, gguf.h, the tc_vit_load refusals),
checked on the CPU the way the reference checks its own (tests/test_arena.c,
tests/test_gguf.c, src/vit.c:135-261). These entry points touch no GPU."""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import tcg
import tcg_gguf as G

SIZE_MAX = (1 << 64) - 1


@pytest.fixture()
def L():
    return tcg.lib()


# ------------------------------------------------------------------ arena

def test_arena_contract(L):                      # tests/test_arena.c:6-83
    a = L.arena_create(1 << 20, b"test")
    pa = C.byref(a)
    assert L.arena_ok(pa) and a.cap >= 1 << 20 and L.arena_used(pa) == 0
    align = 1
    while align <= 4096:
        p = L.arena_alloc(pa, 1, align)
        assert p and p % align == 0
        align *= 2
    assert not L.arena_alloc(pa, 8, 3)
    mark = L.arena_mark(pa)
    assert L.arena_alloc(pa, 4096, 64) and L.arena_used(pa) > mark
    L.arena_release(pa, mark)
    assert L.arena_used(pa) == mark
    L.arena_release(pa, L.arena_used(pa) + 999999)
    assert L.arena_used(pa) == mark
    assert L.arena_peak(pa) > mark
    msg = b"grouped-query attention\0"
    cp = L.arena_memdup(pa, msg, len(msg), 1)
    assert C.string_at(cp) == msg[:-1]
    C.memset(cp, 0xAB, len(msg))
    L.arena_release(pa, mark)
    z = L.arena_calloc(pa, 64, 1, 64)
    assert C.string_at(z, 64) == b"\0" * 64
    assert not L.arena_alloc(pa, a.cap + 1, 64)
    assert not L.arena_alloc(pa, SIZE_MAX, 64)
    assert not L.arena_alloc(pa, SIZE_MAX - 16, 64)
    assert L.arena_alloc(pa, 128, 64)
    assert not L.arena_calloc(pa, SIZE_MAX // 2, 4, 64)
    L.arena_reset(pa)
    assert L.arena_used(pa) == 0 and L.arena_peak(pa) > 0
    nil = L.arena_create(0, b"nil")
    assert not L.arena_ok(C.byref(nil)) and not L.arena_alloc(C.byref(nil), 1, 1)
    L.arena_destroy(C.byref(nil))
    buf = C.create_string_buffer(32)
    for n, s in ((512, b"512 B"), (1024, b"1.00 KiB"), (1536, b"1.50 KiB"), (1 << 30, b"1.00 GiB")):
        assert L.arena_fmt_bytes(buf, 32, n) == s
    L.arena_destroy(pa)
    assert not L.arena_ok(pa)


# ------------------------------------------------------------------ gguf

def _s(t: bytes) -> bytes:
    return struct.pack("<Q", len(t)) + t


def build_good() -> bytearray:                   # tests/test_gguf.c:54-102
    b = bytearray(struct.pack("<IIQQ", 0x46554747, 3, 2, 7))
    b += _s(b"general.architecture") + struct.pack("<I", 8) + _s(b"llama")
    b += _s(b"general.alignment") + struct.pack("<II", 4, 32)
    b += _s(b"llama.block_count") + struct.pack("<II", 4, 4)
    b += _s(b"llama.attention.layer_norm_rms_epsilon") + struct.pack("<If", 6, 1e-5)
    b += _s(b"test.bool") + struct.pack("<IB", 7, 1)
    b += _s(b"test.i32_array") + struct.pack("<IIQiii", 9, 5, 3, 10, 20, 30)
    b += _s(b"tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, 3) + _s(b"<s>") + _s(b"hello") + _s(b"world")
    b += _s(b"token_embd.weight") + struct.pack("<IQQIQ", 2, 4, 8, 0, 0)
    b += _s(b"blk.0.attn_q.weight") + struct.pack("<IQQIQ", 2, 32, 2, 2, 128)
    b += b"\0" * ((-len(b)) % 32)
    b += struct.pack("<32f", *[i * 0.5 for i in range(32)])
    b += bytes(range(36))
    return b


def open_bytes(L, tmp_path, data, arena):
    p = tmp_path / "t.gguf"
    p.write_bytes(bytes(data))
    g = tcg.Gguf()
    ok = L.gguf_open(C.byref(g), str(p).encode(), C.byref(arena))
    return ok, g


def test_gguf_happy_path(L, tmp_path):           # tests/test_gguf.c:131-214
    a = L.arena_create(8 << 20, b"test-gguf")
    ok, g = open_bytes(L, tmp_path, build_good(), a)
    assert ok, g.err
    assert (g.version, g.alignment, g.n_kv, g.n_tensors, g.data_size) == (3, 32, 7, 2, 164)
    s = tcg.GgufStr()
    assert L.gguf_get_str(C.byref(g), b"general.architecture", C.byref(s))
    assert L.gguf_str_eq(s, b"llama") and not L.gguf_str_eq(s, b"llam") and not L.gguf_str_eq(s, b"llamaa")
    assert g.map <= s.ptr < g.map + g.map_size
    buf = C.create_string_buffer(8)
    assert L.gguf_str_cstr(buf, 8, s) == b"llama"
    assert L.gguf_str_cstr(buf, 4, s) == b"lla"
    assert L.gguf_u64_or(C.byref(g), b"llama.block_count", 999) == 4
    assert L.gguf_u64_or(C.byref(g), b"does.not.exist", 999) == 999
    assert abs(L.gguf_f32_or(C.byref(g), b"llama.attention.layer_norm_rms_epsilon", 0.0) - 1e-5) < 1e-7
    kb = L.gguf_find(C.byref(g), b"test.bool")
    assert kb and kb.contents.type == 7 and kb.contents.v.b
    ka = L.gguf_find(C.byref(g), b"test.i32_array").contents
    assert ka.type == 9 and ka.v.arr.len == 3 and ka.v.arr.type == 5
    assert struct.unpack("<i", C.string_at(ka.v.arr.data + 8, 4))[0] == 30
    kt = L.gguf_find(C.byref(g), b"tokenizer.ggml.tokens").contents
    assert kt.v.arr.len == 3 and [kt.v.arr.strs[i].text() for i in range(3)] == ["<s>", "hello", "world"]
    t0 = L.gguf_tensor(C.byref(g), b"token_embd.weight").contents
    assert (t0.n_dims, t0.dims[0], t0.dims[1], t0.n_elem, t0.type, t0.nbytes) == (2, 4, 8, 32, 0, 128)
    vals = np.frombuffer(C.string_at(t0.data, 128), np.float32)
    assert vals[0] == 0.0 and vals[7] == 3.5 and vals[31] == 15.5
    t1 = L.gguf_tensor(C.byref(g), b"blk.0.attn_q.weight").contents
    assert (t1.n_elem, t1.type, t1.nbytes, t1.offset) == (64, 2, 36, 128)
    raw = C.string_at(t1.data, 36)
    assert raw[0] == 0 and raw[35] == 35
    assert not L.gguf_tensor(C.byref(g), b"nope")
    L.gguf_close(C.byref(g))
    L.arena_destroy(C.byref(a))


def test_ggml_block_table(L):                    # tests/test_gguf.c:216-225
    assert L.ggml_blck_size(12) == 256 and L.ggml_type_size(12) == 144
    assert L.ggml_type_size(14) == 210 and L.ggml_type_size(8) == 34
    assert L.ggml_type_supported(12)
    assert not L.ggml_type_supported(16) and L.ggml_type_name(16) == b"UNSUPPORTED"
    assert not L.ggml_type_supported(9999)


@pytest.mark.parametrize("mutate,needle", [
    (lambda b: b.__setitem__(0, ord("X")), b"not a GGUF"),
    (lambda b: b.__setitem__(slice(0, 4), struct.pack("<I", 0x47475546)), b"big-endian"),
    (lambda b: b.__setitem__(slice(4, 8), struct.pack("<I", 1)), b"version"),
    (lambda b: b.__delitem__(slice(40, None)), None),
    (lambda b: b.__delitem__(slice(len(b) - 8, None)), b"overruns"),
    (lambda b: b.__setitem__(slice(8, 16), struct.pack("<Q", (1 << 64) - 1)), b"impossible"),
    (lambda b: b.__delitem__(slice(16, None)), b"too small"),
])
def test_gguf_corrupt_files(L, tmp_path, mutate, needle):    # tests/test_gguf.c:227-280
    a = L.arena_create(8 << 20, b"test-gguf")
    b = build_good()
    mutate(b)
    ok, g = open_bytes(L, tmp_path, b, a)
    assert not ok
    if needle:
        assert needle in g.err
    L.arena_destroy(C.byref(a))


def test_gguf_missing_file(L):
    a = L.arena_create(1 << 20, b"x")
    g = tcg.Gguf()
    assert not L.gguf_open(C.byref(g), b"/nonexistent/model.gguf", C.byref(a))
    assert b"cannot open" in g.err
    L.arena_destroy(C.byref(a))


def test_kquant_tensor_must_be_whole_superblocks(L, tmp_path):
    # a Q4_K tensor of 300 elements: rejected at parse time (src/gguf.c:282-285)
    raw = np.zeros(144 * 2, np.uint8)
    path = str(tmp_path / "bad.gguf")
    G.write_gguf(path, {"general.architecture": "x"}, [("w", raw, G.Q4_K, (300,))])
    a = L.arena_create(1 << 20, b"x")
    g = tcg.Gguf()
    assert not L.gguf_open(C.byref(g), path.encode(), C.byref(a))
    assert b"not a multiple of the Q4_K block size 256" in g.err
    L.arena_destroy(C.byref(a))


def test_kquant_tensor_descriptor(L, tmp_path):
    raw = G.make_kquant(G.Q6_K, 4, 512, seed=1)
    path = str(tmp_path / "q.gguf")
    G.write_gguf(path, {"general.architecture": "x"}, [("w", raw, G.Q6_K, (4, 512))])
    a = L.arena_create(1 << 20, b"x")
    g = tcg.Gguf()
    assert L.gguf_open(C.byref(g), path.encode(), C.byref(a)), g.err
    t = L.gguf_tensor(C.byref(g), b"w").contents
    assert (t.n_elem, t.nbytes, t.dims[0], t.dims[1]) == (2048, 8 * 210, 512, 4)
    assert C.string_at(t.data, t.nbytes) == raw.tobytes()
    L.gguf_close(C.byref(g))
    L.arena_destroy(C.byref(a))


# ------------------------------------------------------ tc_vit_load refusals

def _vit_file(tmp_path, name="m.gguf", drop=None, **meta):
    cfg = G.vit_config("vit-b32", n_layer=1, d_model=64, n_head=4, d_ffn=128, patch=16, image=32, d_out=16)
    w = G.make_vit_weights(cfg, 0)
    if drop:
        w.pop(drop)
    kv = G.vit_metadata(cfg)
    for k, v in meta.items():
        key = "clip-vit." + k.replace("__", ".")
        if v is None:
            kv.pop(key, None)
        else:
            kv[key] = v
    path = str(tmp_path / name)
    G.write_gguf(path, kv, [(n, a, G.F32, a.shape) for n, a in w.items()])
    return path, cfg


def test_vit_load_ok_zero_copy(L, tmp_path):
    path, cfg = _vit_file(tmp_path)
    m = tcg.VitModel(path)
    assert m.cfg["n_token"] == cfg["n_token"] == 5 and m.m.head_dim == 16 and not m.m.quick_gelu
    assert m.m.weight_bytes == 0                       # F32: pointers into the mapping
    assert m.m.gguf.map <= m.m.patch_embd < m.m.gguf.map + m.m.gguf.map_size
    assert L.tc_vit_scratch_bytes(C.byref(m.m)) == (6 * 5 * 64 + 5 * 128 + 5) * 4 + 8 * 64
    m.close()


@pytest.mark.parametrize("meta,needle", [
    (dict(activation=None), "GELU form must not be guessed"),
    (dict(activation="relu"), "unsupported activation 'relu'"),
    (dict(pooling="mean"), "pooling 'mean' not implemented"),
    (dict(context_length=7), "context_length 7 but grid implies 5 tokens"),
    (dict(block_count=None), "incomplete architecture metadata"),
    (dict(attention__head_count=3), "not divisible by 3 heads"),
])
def test_vit_load_refusals(tmp_path, meta, needle):
    path, _ = _vit_file(tmp_path, **meta)
    with pytest.raises(tcg.TcgError, match=needle):
        tcg.VitModel(path)


def test_vit_load_missing_tensor(tmp_path):
    path, _ = _vit_file(tmp_path, drop="v.blk.0.ffn_up.bias")
    with pytest.raises(tcg.TcgError, match="missing tensor 'v.blk.0.ffn_up.bias'"):
        tcg.VitModel(path)


def test_vit_load_quick_gelu(tmp_path):
    path, _ = _vit_file(tmp_path, activation="gelu_quick")
    m = tcg.VitModel(path)
    assert m.m.quick_gelu
    m.close()

"""K-quant dequant and fused dequant-matvec on the GPU against the oracle.

Dequant is integer unpacking plus fp32 scaling in the restatement's exact
rounding order, so the bar is bit-exact. The matvec sums in a different
order from the reference's sequential dot product, so its bar is
max|y - y_ref| <= 1e-4 * max|y_ref|.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
import tcg
import tcg_gguf as G
from fixtures_io import kquant_golden

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def dev_dequant(raw: np.ndarray, n: int, qtype: int, src_offset: int = 0) -> np.ndarray:
    L = tcg.lib()
    with tcg.DeviceBuffer(raw.nbytes + 64) as src, tcg.DeviceBuffer(n * 4) as dst:
        src.upload(raw, offset=src_offset)
        tcg.check(L.tcg_dequant(dst.ptr, src.ptr + src_offset, n, qtype), "tcg_dequant")
        return dst.download(n)


def test_f16_every_input_bit_exact(gpu):
    h = np.arange(65536, dtype=np.uint16)
    got = dev_dequant(h.view(np.uint8), 65536, G.F16)
    assert np.array_equal(bits(got), bits(oracle.f16_to_f32_all()))


@pytest.mark.parametrize("tag,qt", [("q4k", G.Q4_K), ("q6k", G.Q6_K)])
def test_golden_blocks_bit_exact(gpu, tag, qt):
    g = kquant_golden()
    got = dev_dequant(g[f"{tag}_blocks"].reshape(-1), g[f"{tag}_values"].size, qt)
    assert np.array_equal(bits(got), bits(g[f"{tag}_values"]))


@pytest.mark.parametrize("qt", [G.Q4_K, G.Q6_K])
def test_full_size_bit_exact(gpu, qt):
    # the 14336 x 4096 tensor of the dequant benchmark, seeded as there
    raw = G.make_kquant(qt, 14336, 4096, seed=2)
    n = 14336 * 4096
    got = dev_dequant(raw, n, qt)
    assert np.array_equal(bits(got), bits(oracle.dequant(raw, n, qt)))


@pytest.mark.parametrize("qt", [G.Q4_K, G.Q6_K])
@pytest.mark.parametrize("nblocks", [1, 7, 8, 9, 13, 1001])
@pytest.mark.parametrize("offset", [0, 2, 1])
def test_ragged_counts_and_alignment(gpu, qt, nblocks, offset):
    raw = G.make_kquant(qt, nblocks, 256, seed=nblocks + 17 * offset)
    got = dev_dequant(raw, nblocks * 256, qt, src_offset=offset)
    assert np.array_equal(bits(got), bits(oracle.dequant(raw, nblocks * 256, qt)))


def test_rejections(gpu):
    L = tcg.lib()
    with tcg.DeviceBuffer(4096) as b:
        assert not L.tcg_dequant(b.ptr, b.ptr, 300, G.Q4_K)
        assert b"superblocks" in L.tcg_last_error()
        assert not L.tcg_dequant(b.ptr, b.ptr, 256, 13)
        assert not L.tcg_dequant(b.ptr + 4, b.ptr, 256, G.Q4_K)     # dst not 16-byte aligned
        assert L.tcg_dequant(b.ptr, b.ptr, 0, G.Q4_K)              # empty is fine


@pytest.mark.parametrize("qt", [G.F16, G.Q4_K, G.Q6_K])
def test_host_seam_tc_dequant(gpu, qt):
    L = tcg.lib()
    if qt == G.F16:
        raw = np.random.default_rng(4).integers(0, 65536, 4096, dtype=np.uint16).view(np.uint8)
        n = 4096
    else:
        raw = G.make_kquant(qt, 37, 256, seed=9)
        n = 37 * 256
    out = np.empty(n, np.float32)
    assert L.tc_dequant(out.ctypes.data, raw.ctypes.data, n, qt), tcg.err()
    want = oracle.dequant(raw, n, qt)
    same = (bits(out) == bits(want)) | (np.isnan(out) & np.isnan(want))
    assert same.all()


def test_dequant_view_from_gguf(gpu, tmp_path):
    L = tcg.lib()
    raw = G.make_kquant(G.Q4_K, 8, 1024, seed=5)
    path = str(tmp_path / "q.gguf")
    G.write_gguf(path, {"general.architecture": "x"}, [("w", raw, G.Q4_K, (8, 1024))])
    a = L.arena_create(1 << 20, b"x")
    g = tcg.Gguf()
    assert L.gguf_open(C.byref(g), path.encode(), C.byref(a))
    t = L.gguf_tensor(C.byref(g), b"w")
    da = L.tcg_arena_create(1 << 22, b"dev")
    conv = C.c_bool(False)
    p = L.tcg_dequant_view(t, C.byref(da), C.byref(conv))
    assert p and conv.value
    got = np.empty(8192, np.float32)
    assert L.tcg_d2h(got.ctypes.data, p, got.nbytes) and L.tcg_sync()
    assert np.array_equal(bits(got), bits(oracle.dequant(raw, 8192, G.Q4_K)))
    # host view through the reference-named seam
    hv = L.tc_dequant_view(t, C.byref(a), C.byref(conv))
    assert hv and conv.value
    assert np.array_equal(np.frombuffer(C.string_at(hv, 8192 * 4), np.uint32), bits(got))
    L.tcg_arena_destroy(C.byref(da))
    L.gguf_close(C.byref(g))
    L.arena_destroy(C.byref(a))


def dev_matvec(raw, x, N, K, qt, repeat=1):
    """y of the device matvec; with repeat > 1 every launch must give the
    same bits (the K-segment reduction resets its counters itself)."""
    L = tcg.lib()
    with tcg.DeviceBuffer.from_array(raw) as w, tcg.DeviceBuffer.from_array(x) as xb, \
            tcg.DeviceBuffer(N * 4) as y:
        first = None
        for _ in range(repeat):
            tcg.check(L.tcg_matvec_q(y.ptr, w.ptr, xb.ptr, N, K, qt), "tcg_matvec_q")
            got = y.download(N)
            if first is None:
                first = got
            else:
                assert np.array_equal(got, first)
        assert L.tcg_device_error() == 0
        return first


@pytest.mark.parametrize("qt,N,K,seed", [
    (G.Q4_K, 4096, 14336, 3),      # the decode matvec
    (G.Q6_K, 128256, 4096, 5),     # the output head
    (G.Q4_K, 1, 256, 7), (G.Q6_K, 3, 768, 8), (G.Q4_K, 100, 2304, 9),
    (G.Q6_K, 5000, 512, 10), (G.Q4_K, 70, 4096, 11),
    (G.Q4_K, 4095, 14336, 12),     # odd row count, a partial last CTA iteration
    (G.Q4_K, 9473, 14336, 13),     # long rows, many of them: row pairs, the last pair one row
    (G.Q6_K, 9473, 14336, 14),     # long rows of 210-byte superblocks
])
def test_matvec_vs_dequant_then_linear(gpu, qt, N, K, seed):
    raw = G.make_kquant(qt, N, K, seed=seed)
    x = np.random.default_rng(seed + 100).standard_normal(K).astype(np.float32)
    got = dev_matvec(raw, x, N, K, qt, repeat=3)
    kernel = tcg.lib().tcg_matvec_last_kernel()
    # Q4_K runs the integer mma.sync kernel, Q6_K too where a row is whole
    # 8-superblock (1680-byte) segments, else the streaming or the staged one
    if qt == G.Q4_K:
        assert kernel == 5, kernel
    else:
        assert kernel == 6 if K % 2048 == 0 else kernel in (2, 3), kernel
    want = oracle.matvec_q(raw, x, N, K, qt)
    err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert err <= MATVEC_TOL, err


def _x_cases(K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(K).astype(np.float32)
    wide = x * np.float32(2.0) ** rng.integers(-30, 30, K).astype(np.float32)   # 60 binades within sub-blocks
    zeros = x.copy()
    zeros[32:96] = 0.0                                                          # whole zero sub-blocks
    zeros[300:301] = 0.0
    tiny = (x * np.float32(1e-30)).astype(np.float32)
    return {"normal": x, "wide": wide.astype(np.float32), "zeros": zeros, "tiny": tiny}


@pytest.mark.parametrize("N,K", [
    (4096, 14336),      # the decode matvec: ~12 units per CTA, tiles shared by several CTAs
    (100, 2304),        # one ragged tile split over 9 CTAs
    (129, 256),         # two tiles, one row in the second
    (37888, 256),       # 296 tiles of one superblock, two per CTA, written directly
    (1, 256), (70, 4096), (300, 768),
])
def test_matvec_q4k_tensor_cores(gpu, N, K):
    """The opt-in Q4_K matvec on tcgen05 (int8 nibbles x int8 pieces of x,
    exact integer sums per sub-block) against the oracle and against the
    CUDA-core kernel, on x with wide dynamic range, zero sub-blocks and tiny
    values; repeated launches give the same bits (tile counters reset
    themselves)."""
    L = tcg.lib()
    raw = G.make_kquant(G.Q4_K, N, K, seed=N + K)
    for name, x in _x_cases(K, N * 7 + K).items():
        old = L.tcg_matvec_set_tc(1)
        try:
            got = dev_matvec(raw, x, N, K, G.Q4_K, repeat=3)
            assert L.tcg_matvec_last_kernel() == 4
        finally:
            L.tcg_matvec_set_tc(old)
        want = oracle.matvec_q(raw, x, N, K, G.Q4_K).astype(np.float64)
        scale = np.abs(want).max()
        assert scale > 0, name
        err = np.abs(got.astype(np.float64) - want).max() / scale
        assert err <= MATVEC_TOL, (name, err)
        old = L.tcg_matvec_set_mma(0)
        try:
            cuda_cores = dev_matvec(raw, x, N, K, G.Q4_K)
            assert L.tcg_matvec_last_kernel() in (2, 3)
        finally:
            L.tcg_matvec_set_mma(old)
        assert np.abs(cuda_cores.astype(np.float64) - want).max() / scale <= MATVEC_TOL, name


@pytest.mark.parametrize("case", ["normal", "wide", "zeros", "tiny"])
def test_matvec_q4k_row_pairs_x_cases(gpu, case):
    """Q4_K rows are taken in pairs that share every x load; an odd row
    count leaves the last pair one row (they run where the rows are too long
    for the one-row rings). x with 60 binades, zero sub-blocks and 1e-30
    values."""
    N, K = 9473, 14336
    raw = G.make_kquant(G.Q4_K, N, K, seed=21)
    x = _x_cases(K, 22)[case]
    L = tcg.lib()
    old = L.tcg_matvec_set_mma(0)
    try:
        got = dev_matvec(raw, x, N, K, G.Q4_K, repeat=2)
        assert L.tcg_matvec_last_kernel() == 2
    finally:
        L.tcg_matvec_set_mma(old)
    want = oracle.matvec_q(raw, x, N, K, G.Q4_K).astype(np.float64)
    err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert err <= MATVEC_TOL, err


@pytest.mark.parametrize("N,K", [
    (4096, 14336),      # the decode matvec: 16-row tiles split in 8 K segments, summed by the last warp
    (14336, 4096),      # many tiles, split in 16
    (4095, 14336),      # a ragged last tile
    (9473, 14336),      # long rows, many of them
    (100, 2304), (129, 256), (1, 256), (17, 512), (70, 4096), (37888, 256), (300, 768),
    (4096, 11008), (300, 11008),   # 43 superblocks a row: the last segment of a row is short
])
def test_matvec_q4k_mma(gpu, N, K):
    """The default Q4_K matvec: integer mma.sync over the raw nibbles and
    exact int8 pieces of x, against the oracle (dequantise, then the
    reference's linear) and the CUDA-core kernel, on x with wide dynamic
    range, zero sub-blocks and tiny values; repeated launches give the same
    bits (the per-tile counters reset themselves)."""
    L = tcg.lib()
    raw = G.make_kquant(G.Q4_K, N, K, seed=N + 3 * K)
    for name, x in _x_cases(K, N * 5 + K).items():
        got = dev_matvec(raw, x, N, K, G.Q4_K, repeat=3)
        assert L.tcg_matvec_last_kernel() == 5
        want = oracle.matvec_q(raw, x, N, K, G.Q4_K).astype(np.float64)
        scale = np.abs(want).max()
        assert scale > 0, name
        err = np.abs(got.astype(np.float64) - want).max() / scale
        assert err <= MATVEC_TOL, (name, err)
        old = L.tcg_matvec_set_mma(0)
        try:
            cuda_cores = dev_matvec(raw, x, N, K, G.Q4_K)
        finally:
            L.tcg_matvec_set_mma(old)
        assert np.abs(cuda_cores.astype(np.float64) - got).max() / scale <= 2 * MATVEC_TOL, name


@pytest.mark.parametrize("segs", [2, 4, 5, 7, 8, 9, 14])
def test_matvec_q4k_mma_segments(gpu, segs):
    """K splits of the 4096 x 14336 decode matvec: units of 16 rows x
    ceil(56/segs) superblocks (5 and 9 segments leave a short last one) stream through a ring of shared-memory slots that is
    refilled (more units per CTA than slots for the long units), and split
    tiles are summed by the last segment to arrive; each against the oracle,
    three calls giving the same bits."""
    N, K = 4096, 14336
    L = tcg.lib()
    raw = G.make_kquant(G.Q4_K, N, K, seed=31)
    x = _x_cases(K, 32)["wide"]
    old = L.tcg_matvec_mma_segments(segs)
    try:
        got = dev_matvec(raw, x, N, K, G.Q4_K, repeat=3)
        assert L.tcg_matvec_last_kernel() == 5
    finally:
        L.tcg_matvec_mma_segments(old)
    want = oracle.matvec_q(raw, x, N, K, G.Q4_K).astype(np.float64)
    assert np.abs(got.astype(np.float64) - want).max() / np.abs(want).max() <= MATVEC_TOL


@pytest.mark.parametrize("N,K", [
    (128256, 4096),     # the output head: 2 segments a row, ~108 units per CTA through 7 slots
    (4096, 14336),      # 7 segments a row
    (14336, 4096),
    (4095, 14336),      # a ragged last tile
    (1, 2048), (17, 2048), (100, 8192), (300, 6144),
])
def test_matvec_q6k_mma(gpu, N, K):
    """The default Q6_K matvec where rows are whole 1680-byte segments:
    integer mma.sync over the 6-bit q (nibble and high bits merged in
    registers; odd superblocks 2 bytes off a word boundary), -32 folded into
    the accumulator input; against the oracle (dequantise, then the
    reference's linear) and the CUDA-core kernel, on x with wide dynamic
    range, zero sub-blocks and tiny values; three calls give the same bits."""
    L = tcg.lib()
    raw = G.make_kquant(G.Q6_K, N, K, seed=N + 5 * K)
    cases = _x_cases(K, N * 7 + K)
    if N * K > 1 << 28:
        cases = {"wide": cases["wide"]}
    for name, x in cases.items():
        got = dev_matvec(raw, x, N, K, G.Q6_K, repeat=3)
        assert L.tcg_matvec_last_kernel() == 6
        want = oracle.matvec_q(raw, x, N, K, G.Q6_K).astype(np.float64)
        scale = np.abs(want).max()
        assert scale > 0, name
        err = np.abs(got.astype(np.float64) - want).max() / scale
        assert err <= MATVEC_TOL, (name, err)
        old = L.tcg_matvec_set_mma(0)
        try:
            cuda_cores = dev_matvec(raw, x, N, K, G.Q6_K)
            assert L.tcg_matvec_last_kernel() in (2, 3)
        finally:
            L.tcg_matvec_set_mma(old)
        assert np.abs(cuda_cores.astype(np.float64) - got).max() / scale <= 2 * MATVEC_TOL, name


@pytest.mark.parametrize("split", [0, 1])
@pytest.mark.parametrize("N,K", [(14336, 4096), (1000, 16384)])
def test_matvec_q6k_mma_split(gpu, split, N, K):
    """Q6_K units read by one warp, or by two warps (four superblocks each,
    two partial sums per segment): the same result within rounding, each
    against the oracle, three calls giving the same bits."""
    L = tcg.lib()
    raw = G.make_kquant(G.Q6_K, N, K, seed=41 + N)
    x = _x_cases(K, 77)["wide"]
    old = L.tcg_matvec_mma_split(split)
    try:
        got = dev_matvec(raw, x, N, K, G.Q6_K, repeat=3)
        assert L.tcg_matvec_last_kernel() == 6
    finally:
        L.tcg_matvec_mma_split(old)
    want = oracle.matvec_q(raw, x, N, K, G.Q6_K).astype(np.float64)
    assert np.abs(got.astype(np.float64) - want).max() / np.abs(want).max() <= MATVEC_TOL


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("qt,N,K", [(G.Q4_K, 4096, 14336), (G.Q4_K, 4095, 11008), (G.Q4_K, 14336, 4096),
                                    (G.Q6_K, 4096, 14336), (G.Q6_K, 300, 6144)])
def test_matvec_mma_tile_modes(gpu, mode, qt, N, K):
    """Units in segment-major ranges (split tiles summed through global
    memory by the last segment to arrive) or whole tiles per CTA (a tile's
    segments summed in shared memory): each against the oracle, three calls
    giving the same bits."""
    L = tcg.lib()
    raw = G.make_kquant(qt, N, K, seed=13 + N + qt)
    x = _x_cases(K, 5)["wide"]
    old = L.tcg_matvec_mma_tiles(mode)
    try:
        got = dev_matvec(raw, x, N, K, qt, repeat=3)
        assert L.tcg_matvec_last_kernel() == (5 if qt == G.Q4_K else 6)
    finally:
        L.tcg_matvec_mma_tiles(old)
    want = oracle.matvec_q(raw, x, N, K, qt).astype(np.float64)
    assert np.abs(got.astype(np.float64) - want).max() / np.abs(want).max() <= MATVEC_TOL


def _q4k_vs_oracle(N, K, seed, hook, mode):
    L = tcg.lib()
    raw = G.make_kquant(G.Q4_K, N, K, seed=seed)
    x = _x_cases(K, seed + 1)["wide"]
    old = hook(mode)
    try:
        got = dev_matvec(raw, x, N, K, G.Q4_K, repeat=3)
        assert L.tcg_matvec_last_kernel() == 5
    finally:
        hook(old)
    want = oracle.matvec_q(raw, x, N, K, G.Q4_K).astype(np.float64)
    assert np.abs(got.astype(np.float64) - want).max() / np.abs(want).max() <= MATVEC_TOL


@pytest.mark.parametrize("direct", [0, 1])
@pytest.mark.parametrize("N,K", [(4096, 14336), (4090, 14336), (14336, 4096), (14330, 4096)])
def test_matvec_q4k_direct_units(gpu, direct, N, K):
    """The few units past a CTA's slots read from global memory by the idle
    consumer warps (after L2 and L1 prefetches), or the slots refilled:
    segment-major (4096 x 14336) and tile-major (14336 x 4096) ranges, ragged
    last tiles; each against the oracle, three calls giving the same bits."""
    _q4k_vs_oracle(N, K, 21 + N, tcg.lib().tcg_matvec_mma_direct, direct)


@pytest.mark.parametrize("static", [0, 1])
@pytest.mark.parametrize("N,K", [(4096, 14336), (4090, 14336)])
def test_matvec_q4k_static_grid(gpu, static, N, K):
    """With the static-weights promise the Q4_K matvec runs one CTA fewer
    than SMs (other unit ranges, direct units): against the oracle."""
    _q4k_vs_oracle(N, K, 41 + N, tcg.lib().tcg_matvec_set_static_weights, static)


@pytest.mark.parametrize("split", [2, 4])
@pytest.mark.parametrize("N,K", [(4096, 14336), (14336, 4096), (4095, 11008)])
def test_matvec_q4k_parts(gpu, split, N, K):
    """Two or four warps per Q4_K unit (their sums met in shared memory)."""
    _q4k_vs_oracle(N, K, 31 + N, tcg.lib().tcg_matvec_mma_split, split)


@pytest.mark.parametrize("static", [0, 1])
def test_matvec_decode_chain(gpu, static):
    """A decode-like chain on one stream, each matvec reading the one before
    it's output: y1 = W1 x, y2 = W2 y1, y3 = W3 y2 (Q4_K, Q6_K, Q4_K), queued
    behind a device delay so that they run back to back. With the
    static-weights promise the kernels overlap (each fetches its weights while
    the one before it finishes); x must still be read only after it is
    written. Each output against the oracle on the device's own input."""
    L = tcg.lib()
    n = 4096
    qts = [G.Q4_K, G.Q6_K, G.Q4_K]
    raws = [G.make_kquant(qt, n, n, seed=40 + i) for i, qt in enumerate(qts)]
    x = np.random.default_rng(44).standard_normal(n).astype(np.float32)
    ws = [tcg.DeviceBuffer.from_array(r) for r in raws]
    ys = [tcg.DeviceBuffer.from_array(x)] + [tcg.DeviceBuffer(n * 4) for _ in qts]
    old = L.tcg_matvec_set_static_weights(static)
    try:
        for rep in range(3):
            for b in ys[1:]:
                tcg.check(L.tcg_memset(b.ptr, 0xFF, n * 4))           # NaN: a read before the write shows
            tcg.check(L.tcg_device_delay_us(300))
            for i, qt in enumerate(qts):
                tcg.check(L.tcg_matvec_q(ys[i + 1].ptr, ws[i].ptr, ys[i].ptr, n, n, qt), "tcg_matvec_q")
            outs = [b.download(n) for b in ys]
            assert L.tcg_device_error() == 0
            for i, qt in enumerate(qts):
                want = oracle.matvec_q(raws[i], outs[i], n, n, qt).astype(np.float64)
                got = outs[i + 1].astype(np.float64)
                assert np.isfinite(got).all()
                assert np.abs(got - want).max() / np.abs(want).max() <= MATVEC_TOL
    finally:
        L.tcg_matvec_set_static_weights(old)
        for b in ws + ys:
            b.close()


def test_device_delay(gpu):
    """The queue delay holds the stream for about the time asked, and refuses
    more than 20 ms."""
    L = tcg.lib()
    ms = tcg.time_ms(lambda: tcg.check(L.tcg_device_delay_us(400)), 2, 3)
    assert 0.3 <= ms <= 5.0
    assert not L.tcg_device_delay_us(20001)
    assert b"20 ms" in L.tcg_last_error()
    assert L.tcg_device_delay_us(0)


def test_matvec_rejections(gpu):
    L = tcg.lib()
    assert not L.tcg_matvec_q(None, None, None, 4, 300, G.Q4_K)
    assert b"multiple of 256" in L.tcg_last_error()
    assert not L.tcg_matvec_q(None, None, None, 4, 256, G.F16)

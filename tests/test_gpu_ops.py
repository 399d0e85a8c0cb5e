"""Op-level parity of the device kernels (tcg_* in include/tcg.h).

* the reference's golden vectors (tests/fixtures/ops.gguf) with the
  reference's own per-op tolerances (tests/test_ops.c:74-148);
* LayerNorm against the oracle on ViT-width rows (one offset by 1e4);
* the 3xTF32 tcgen05 GEMM in every tile configuration on ragged shapes,
  against the oracle's sequential fp32 GEMM: max|err| <= 1e-5 * max|y|;
* the stream-K split of a GEMM's last, partial wave of tiles (less than one
  wave, one wave and a part, a K of 12 chunks): deterministic, and within the
  same bound of a float64 product as the whole-tile schedule.
"""
import numpy as np
import pytest

import oracle
import tcg
from fixtures_io import check_close, ops_golden

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-5


class Dev:
    """Upload numpy arrays, run, download."""

    def __init__(self):
        self.bufs = []

    def put(self, a):
        b = tcg.DeviceBuffer.from_array(np.ascontiguousarray(a, np.float32))
        self.bufs.append(b)
        return b.ptr

    def empty(self, n):
        b = tcg.DeviceBuffer(int(n) * 4)
        self.bufs.append(b)
        return b

    def close(self):
        for b in self.bufs:
            b.close()


@pytest.fixture()
def dev(gpu):
    d = Dev()
    yield d
    d.close()


def test_golden_vectors(dev):
    L = tcg.lib()
    kv, t = ops_golden()
    for tag in ("small", "wide"):
        M, N, K = kv[f"gemm.{tag}.M"], kv[f"gemm.{tag}.N"], kv[f"gemm.{tag}.K"]
        y = dev.empty(M * N)
        tcg.check(L.tcg_gemm(y.ptr, dev.put(t[f"gemm.{tag}.A"]), dev.put(t[f"gemm.{tag}.B"]), M, N, K, True))
        check_close(y.download(M * N), t[f"gemm.{tag}.C"], 2e-4, 1e-5, f"gemm {tag}")
    M, N, K = kv["linear.M"], kv["linear.N"], kv["linear.K"]
    y = dev.empty(M * N)
    tcg.check(L.tcg_linear(y.ptr, dev.put(t["linear.x"]), dev.put(t["linear.W"]), dev.put(t["linear.b"]), M, N, K))
    check_close(y.download(M * N), t["linear.y"], 1e-5, 1e-5, "linear")
    rows, cols = kv["ln.rows"], kv["ln.cols"]
    y = dev.empty(rows * cols)
    tcg.check(L.tcg_layernorm(y.ptr, dev.put(t["ln.x"]), dev.put(t["ln.gamma"]), dev.put(t["ln.beta"]),
                              rows, cols, kv["ln.eps"]))
    check_close(y.download(rows * cols), t["ln.out"], 1e-4, 1e-4, "layernorm")
    n = t["gelu.x"].size
    y, q = dev.empty(n), dev.empty(n)
    gx = dev.put(t["gelu.x"])
    tcg.check(L.tcg_gelu(y.ptr, gx, n))
    tcg.check(L.tcg_gelu_quick(q.ptr, gx, n))
    ge, gq = y.download(n), q.download(n)
    check_close(ge, t["gelu.exact"], 1e-6, 1e-6, "gelu")
    check_close(gq, t["gelu.quick"], 1e-6, 1e-6, "gelu quick")
    assert np.abs(ge - gq).max() > 0.01
    rows, cols = kv["softmax.rows"], kv["softmax.cols"]
    y = dev.empty(rows * cols)
    tcg.check(L.tcg_softmax_rows(y.ptr, dev.put(t["softmax.x"]), rows, cols))
    sm = y.download((rows, cols))
    check_close(sm, t["softmax.out"], 1e-6, 1e-5, "softmax")
    assert np.all(np.abs(sm.astype(np.float64).sum(1) - 1.0) < 1e-5)
    T, H, HD = kv["mha.T"], kv["mha.n_head"], kv["mha.head_dim"]
    y = dev.empty(T * H * HD)
    tcg.check(L.tcg_mha(y.ptr, dev.put(t["mha.q"]), dev.put(t["mha.k"]), dev.put(t["mha.v"]), T, H, HD))
    check_close(y.download(T * H * HD), t["mha.out"], 1e-5, 1e-5, "mha")


def test_add_and_scale(dev):
    L = tcg.lib()
    rng = np.random.default_rng(1)
    a, b = rng.standard_normal(1000).astype(np.float32), rng.standard_normal(1000).astype(np.float32)
    y = dev.empty(1000)
    tcg.check(L.tcg_add(y.ptr, dev.put(a), dev.put(b), 1000))
    assert np.array_equal(y.download(1000), oracle.add(a, b))
    tcg.check(L.tcg_scale(y.ptr, dev.put(a), 0.37, 1000))
    assert np.array_equal(y.download(1000), oracle.scale(a, np.float32(0.37)))


@pytest.mark.parametrize("rows,cols", [(300, 768), (17, 1024), (5, 64), (3, 100)])
def test_layernorm_vs_oracle(dev, rows, cols):
    L = tcg.lib()
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[rows // 2] += 1e4
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    y = dev.empty(rows * cols)
    tcg.check(L.tcg_layernorm(y.ptr, dev.put(x), dev.put(g), dev.put(b), rows, cols, 1e-5))
    got, want = y.download((rows, cols)), oracle.layernorm(x, g, b, rows, cols, 1e-5)
    # double statistics summed in another order: identical but for rare 1-ulp ties
    ulp = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
    assert ulp.max() <= 2 and (ulp == 0).mean() > 0.999


def _pieces(hi, lo, ex, rows, cols, blk):
    """fp16 pieces back to values: (hi + lo) * 2^-e per (row, blk-column block)."""
    h = hi.view(np.float16).astype(np.float64).reshape(rows, cols)
    l = lo.view(np.float16).astype(np.float64).reshape(rows, cols)
    e = ex.view(np.int8)[: rows * (cols // blk)].reshape(cols // blk, rows).T.astype(np.float64)
    return (h + l) * np.repeat(2.0 ** -e, blk, axis=1)


@pytest.mark.parametrize("rows,cols", [(300, 768), (17, 1024), (5, 256)])
def test_layernorm_f16_pieces(dev, rows, cols):
    """LayerNorm written as fp16 pieces: per 256-column block the largest
    value scaled into [2^14, 2^15), hi + lo within 2^-21 of the block's
    largest of the oracle's output; the row norms of that output."""
    L = tcg.lib()
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[rows // 2] += 1e4
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    g[:256] *= np.float32(1e-3)                        # one block far smaller than the others
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    hi, lo, ex, rn = dev.empty(rows * cols // 2), dev.empty(rows * cols // 2), dev.empty(rows * cols // 1024 + 1), dev.empty(rows)
    tcg.check(L.tcg_layernorm_f16(hi.ptr, lo.ptr, ex.ptr, rn.ptr, dev.put(x), dev.put(g), dev.put(b), rows, cols, 1e-5))
    want = oracle.layernorm(x, g, b, rows, cols, 1e-5).astype(np.float64)
    got = _pieces(hi.download(rows * cols // 2, np.uint32), lo.download(rows * cols // 2, np.uint32),
                  ex.download(rows * cols // 1024 + 1, np.uint32), rows, cols, 256)
    for c in range(0, cols, 256):
        w, gv = want[:, c:c + 256], got[:, c:c + 256]
        assert np.all(np.abs(gv - w) <= 2.0 ** -21 * np.abs(w).max(axis=1, keepdims=True)), c
    assert np.allclose(rn.download(rows), np.linalg.norm(want, axis=1), rtol=1e-5)


def test_weight_bounds(dev):
    L = tcg.lib()
    rng = np.random.default_rng(3)
    W = rng.standard_normal((1000, 768)).astype(np.float32)
    W[417] *= 3
    bias = rng.standard_normal(1000).astype(np.float32)
    out = dev.empty(2)
    tcg.check(L.tcg_weight_bounds(out.ptr, dev.put(W), 1000, 768, dev.put(bias)))
    got = out.download(2)
    assert np.isclose(got[0], np.linalg.norm(W.astype(np.float64), axis=1).max(), rtol=1e-5)
    assert got[1] == np.abs(bias).max()


@pytest.mark.parametrize("T,H,HD", [(50, 12, 64), (56, 3, 64), (57, 2, 64), (64, 2, 64), (1, 3, 64), (5, 2, 64), (257, 16, 64), (17, 4, 16), (33, 2, 96)])
def test_mha_vs_oracle(dev, T, H, HD):
    L = tcg.lib()
    rng = np.random.default_rng(T)
    q, k, v = (rng.standard_normal((T, H * HD)).astype(np.float32) for _ in range(3))
    y = dev.empty(T * H * HD)
    tcg.check(L.tcg_mha(y.ptr, dev.put(q), dev.put(k), dev.put(v), T, H, HD))
    got, want = y.download((T, H * HD)), oracle.mha(q, k, v, T, H, HD)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


def _mha_short(L, dev, q, k, v, T, H, kernel):
    y = dev.empty(T * H * 64)
    old = L.tcg_set_attention_short_kernel(kernel)
    try:
        tcg.check(L.tcg_mha(y.ptr, dev.put(q), dev.put(k), dev.put(v), T, H, 64), f"kernel {kernel}")
    finally:
        L.tcg_set_attention_short_kernel(old)
    return y.download((T, H * 64))


@pytest.mark.parametrize("T", [1, 2, 5, 8, 15, 16, 17, 33, 48, 49, 50, 56, 63, 64])
def test_mha_short_kernels(dev, T):
    """head_dim 64, T <= 64: the fp16 hi/lo tensor-core kernel (the default)
    and the fp32 FMA kernel, each within the oracle's bound. One query row is
    50x the others (a peaked softmax), one key row 1e-6x, and head 1's V is
    1e4x larger than head 0's: every scale of the split is exercised."""
    L = tcg.lib()
    H = 3
    rng = np.random.default_rng(1000 + T)
    q, k, v = (rng.standard_normal((T, H * 64)).astype(np.float32) for _ in range(3))
    q[T // 2] *= 50
    k[(T - 1) // 3] *= 1e-6
    v[:, 64:128] *= 1e4
    want = oracle.mha(q, k, v, T, H, 64)
    for kernel in (1, 0):
        got = _mha_short(L, dev, q, k, v, T, H, kernel)
        for h in range(H):          # each head against its own magnitude
            w, g = want[:, 64 * h:64 * h + 64], got[:, 64 * h:64 * h + 64]
            assert np.abs(g - w).max() <= 1e-5 * np.abs(w).max(), (kernel, h)
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("scale", [1e-30, 1e-8, 1e3, 1e12, 1e30])
def test_mha_short_magnitudes(dev, scale):
    """The power-of-two scales of the fp16 split keep the operands inside
    fp16's range whatever the magnitude of q, k and v (scores stay finite:
    q is scaled by 1/scale where k is scaled by scale)."""
    L = tcg.lib()
    T, H = 50, 2
    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((T, H * 64)).astype(np.float32) for _ in range(3))
    q = (q / np.float32(scale)).astype(np.float32)
    k = (k * np.float32(scale)).astype(np.float32)
    v = (v * np.float32(scale)).astype(np.float32)
    want = oracle.mha(q, k, v, T, H, 64)
    got = _mha_short(L, dev, q, k, v, T, H, 1)
    assert np.all(np.isfinite(got))
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.parametrize("T,H,n_img", [(50, 12, 5), (64, 2, 3), (17, 4, 2), (100, 2, 2)])
def test_mha_images_fused_qkv(dev, T, H, n_img):
    """tcg_mha_images: n_img images whose q, k, v share one fused row of width
    3D, written as fp32 and as the tf32 hi/lo pair in one call; hi has tf32's
    10 mantissa bits and hi + lo is the fp32 output to 21 bits."""
    L = tcg.lib()
    D = H * 64
    rng = np.random.default_rng(T * n_img)
    qkv = rng.standard_normal((n_img * T, 3 * D)).astype(np.float32)
    y, hi, lo = dev.empty(n_img * T * D), dev.empty(n_img * T * D), dev.empty(n_img * T * D)
    tcg.check(L.tcg_mha_images(y.ptr, hi.ptr, lo.ptr, dev.put(qkv), T, H, 64, n_img))
    got = y.download((n_img * T, D))
    h, l = hi.download((n_img * T, D)), lo.download((n_img * T, D))
    assert np.all(np.abs((h.astype(np.float64) + l) - got) <= np.abs(got) * 2.0 ** -21)
    assert np.all((h.view(np.uint32) & 0x1FFF) == 0)
    for i in range(n_img):
        r = qkv[i * T:(i + 1) * T]
        want = oracle.mha(r[:, :D].copy(), r[:, D:2 * D].copy(), r[:, 2 * D:].copy(), T, H, 64)
        assert np.abs(got[i * T:(i + 1) * T] - want).max() <= 1e-5 * np.abs(want).max(), i
    assert not L.tcg_mha_images(None, hi.ptr, None, dev.put(qkv), T, H, 64, n_img)


@pytest.mark.parametrize("T,H", [(65, 2), (100, 3), (257, 2), (300, 1), (577, 2)])
def test_mha_long_sequence_kernels_agree(dev, T, H):
    """head_dim 64, T > 64. The streamed-K/V kernel (64- or 48-query blocks)
    performs the whole-K/V kernel's operations in the same order: identical
    bits where both apply (T = 577 fits only the streamed one; the others
    would need 318 KB of shared memory and the call is refused). The default
    (variant 1) is that kernel below T = 128 and the tensor cores from 128 on;
    every variant within the oracle's bound."""
    L = tcg.lib()
    rng = np.random.default_rng(T + 100 * H)
    q, k, v = (rng.standard_normal((T, H * 64)).astype(np.float32) for _ in range(3))
    qp, kp, vp = dev.put(q), dev.put(k), dev.put(v)
    got = {}
    for variant in ((0, 1, 2) if T <= 300 else (1, 2)):
        y = dev.empty(T * H * 64)
        old = L.tcg_set_attention_variant(variant)
        try:
            tcg.check(L.tcg_mha(y.ptr, qp, kp, vp, T, H, 64), f"variant {variant}")
        finally:
            L.tcg_set_attention_variant(old)
        got[variant] = y.download((T, H * 64))
    if T <= 300:
        assert np.array_equal(got[0], got[2])
    if T < 128:
        assert np.array_equal(got[1], got[2])
    want = oracle.mha(q, k, v, T, H, 64)
    for variant, g in got.items():
        assert np.abs(g - want).max() <= 1e-5 * np.abs(want).max(), variant
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("T,H", [(128, 2), (129, 3), (200, 2), (257, 4), (300, 1), (577, 2)])
def test_mha_tensor_core_long(dev, T, H):
    """head_dim 64, 128 <= T: whole blocks of 128 queries on tcgen05 (3xTF32,
    running-maximum softmax), the remaining rows one warp per row; within the
    oracle's bound."""
    L = tcg.lib()
    rng = np.random.default_rng(T + 7 * H)
    q, k, v = (rng.standard_normal((T, H * 64)).astype(np.float32) for _ in range(3))
    y = dev.empty(T * H * 64)
    old = L.tcg_set_attention_variant(3)
    try:
        tcg.check(L.tcg_mha(y.ptr, dev.put(q), dev.put(k), dev.put(v), T, H, 64), "tensor-core attention")
    finally:
        L.tcg_set_attention_variant(old)
    got, want = y.download((T, H * 64)), oracle.mha(q, k, v, T, H, 64)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("cfg", [16, 17, 18, 19, 20])
@pytest.mark.parametrize("blk", [128, 256])
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (300, 768, 768), (1600, 768, 768), (257, 3072, 768),
                                   (513, 768, 3072), (12800, 768, 768)])
def test_linear_f16_pieces(dev, M, N, K, blk, cfg):
    """kind::f16 GEMM on fp16-piece operands (tcg_split_f16: power-of-two
    scales per (row, 128-element K-block) of x and per row of W, two pieces of
    11 bits): within
    the tf32-pair GEMM's bound of the oracle, on rows spanning 1e-12 .. 1e12,
    a weight row of 1e9 and a zero K-block (blocks are exact for largest
    magnitudes in [2^-49, 2^77))."""
    L = tcg.lib()
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[: M // 4] *= np.float32(1e-12)
    x[M // 4: M // 2] *= np.float32(1e12)
    x[:, :blk] *= 0
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[N // 3] *= np.float32(1e9)
    b = rng.standard_normal(N).astype(np.float32)
    xd, Wd, bd = dev.put(x), dev.put(W), dev.put(b)
    f = [dev.empty(n) for n in (M * K // 2, M * K // 2, M * K // 512 + 1, N * K // 2, N * K // 2, N * K // 512 + 1)]
    tcg.check(L.tcg_split_f16(f[0].ptr, f[1].ptr, f[2].ptr, xd, M, K, 0 if blk == 128 else 2))
    tcg.check(L.tcg_split_f16(f[3].ptr, f[4].ptr, f[5].ptr, Wd, N, K, 1))
    y = dev.empty(M * N)
    old = L.tcg_gemm_set_f16_cfg(cfg)           # 16: 3 stages of 64, 17: 6 of 32, 18/19: CTA pairs
    try:
        tcg.check(L.tcg_linear_f16_split(y.ptr, f[0].ptr, f[1].ptr, f[2].ptr, f[3].ptr, f[4].ptr, f[5].ptr, bd,
                                         M, N, K, blk))
    finally:
        L.tcg_gemm_set_f16_cfg(old)
    got = y.download((M, N)).astype(np.float64)
    want = x.astype(np.float64) @ W.astype(np.float64).T + b
    # each row band against its own magnitude (the rows differ by 24 decades)
    for lo, hi in ((0, M // 4), (M // 4, M // 2), (M // 2, M)):
        if hi > lo:
            g, w = got[lo:hi], want[lo:hi]
            assert np.abs(g - w).max() <= GEMM_TOL * np.abs(w).max(), (lo, hi)
    assert L.tcg_device_error() == 0


SHAPES = [(1, 64, 4), (127, 100, 12), (129, 200, 588), (300, 768, 768), (50, 2304, 768), (261, 130, 3072)]


@pytest.mark.parametrize("cfg", [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, -2])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_every_config(dev, cfg, M, N, K):
    L = tcg.lib()
    rng = np.random.default_rng(M * 7 + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y = dev.empty(M * N)
    tcg.check(L.tcg_linear_cfg(y.ptr, dev.put(x), dev.put(W), dev.put(b), M, N, K, cfg), f"cfg {cfg}")
    got, want = y.download((M, N)), oracle.linear(x, W, b, M, N, K)
    err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert err <= GEMM_TOL, (cfg, err)
    assert tcg.lib().tcg_device_error() == 0


def test_gemm_untransposed_and_odd_k(dev):
    L = tcg.lib()
    rng = np.random.default_rng(2)
    A = rng.standard_normal((9, 11)).astype(np.float32)
    B = rng.standard_normal((11, 7)).astype(np.float32)
    y = dev.empty(63)
    tcg.check(L.tcg_gemm(y.ptr, dev.put(A), dev.put(B), 9, 7, 11, False))
    want = oracle.gemm(A, B, 9, 7, 11, b_transposed=False)
    assert np.abs(y.download((9, 7)) - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.parametrize("cfg", [-1, 13, 14, 1, 6])
@pytest.mark.parametrize("M,N,K", [(1, 64, 4), (127, 100, 12), (300, 768, 768), (261, 130, 3072), (1600, 2304, 768)])
def test_bulk_store_epilogue(dev, cfg, M, N, K):
    """Bulk tensor stores (N a multiple of 4) and plain stores give the same
    bits; partial 8-column units and row tiles past M are clipped."""
    import ctypes
    L = tcg.lib()
    rng = np.random.default_rng(M + 3 * N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    xp, wp, bp = dev.put(x), dev.put(W), dev.put(b)
    got = {}
    for t in (0, 1):
        y = dev.empty(M * N + 64)
        tcg.check(L.tcg_memset(y.ptr, 0x7f, (M * N + 64) * 4))
        old = L.tcg_gemm_set_tma_store(t)
        try:
            tcg.check(L.tcg_linear_cfg(y.ptr, xp, wp, bp, M, N, K, cfg), f"cfg {cfg} tma {t}")
        finally:
            L.tcg_gemm_set_tma_store(old)
        plan = (ctypes.c_int * 4)()
        L.tcg_gemm_last_plan(plan)
        assert plan[3] == (1 if t and N % 4 == 0 else 0)
        full = y.download((M * N + 64,))
        assert np.all(full[M * N:].view(np.uint32) == 0x7f7f7f7f)      # nothing written past the matrix
        got[t] = full[:M * N].reshape(M, N)
    assert np.array_equal(got[0], got[1])
    want = oracle.linear(x, W, b, M, N, K)
    assert np.abs(got[1].astype(np.float64) - want).max() <= GEMM_TOL * np.abs(want).max()
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(700, 512, 768), (2000, 2304, 768), (1600, 768, 3072)])
def test_streamk_split(dev, M, N, K):
    L = tcg.lib()
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    want = x.astype(np.float64) @ W.astype(np.float64).T + b
    xp, wp, bp = dev.put(x), dev.put(W), dev.put(b)
    y = dev.empty(M * N)
    got = {}
    for sk in (1, 1, 0):
        old = L.tcg_gemm_set_streamk(sk)
        try:
            tcg.check(L.tcg_linear_cfg(y.ptr, xp, wp, bp, M, N, K, 9), f"streamk {sk}")
        finally:
            L.tcg_gemm_set_streamk(old)
        r = y.download((M, N))
        if sk in got:
            assert np.array_equal(r, got[sk])            # the split is deterministic
        got[sk] = r
    for sk, r in got.items():
        err = np.abs(r.astype(np.float64) - want).max() / np.abs(want).max()
        assert err <= GEMM_TOL, (sk, err)
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(300, 768, 768), (1600, 768, 3072), (129, 200, 512), (1, 64, 256),
                                   (12800, 2304, 768), (777, 3072, 768)])
def test_linear_q4k_packed(dev, M, N, K):
    """tcg_linear_q: the GEMM reads W as Q4_K blocks and dequantises each
    tile in shared memory. Against the oracle (dequantise, then the
    reference's linear) within the GEMM bound, and bit-identical to the
    dequantise -> split -> tensor-core GEMM path with the same tile shape."""
    import tcg_gguf as G
    L = tcg.lib()
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    raw = G.make_kquant_like(G.Q4_K, N, K, M + K, 4e-4)
    W = oracle.dequant(raw, N * K, G.Q4_K).reshape(N, K)
    b = rng.standard_normal(N).astype(np.float32)
    xp, bp = dev.put(x), dev.put(b)
    wq = tcg.DeviceBuffer.from_array(raw)
    dev.bufs.append(wq)
    y = dev.empty(M * N)
    for _ in range(2):
        tcg.check(L.tcg_linear_q(y.ptr, xp, wq.ptr, bp, M, N, K, G.Q4_K), "tcg_linear_q")
    got = y.download((M, N))
    want = oracle.linear(x, W, b, M, N, K)
    err = np.abs(got.astype(np.float64) - want).max() / np.abs(want).max()
    assert err <= GEMM_TOL, err
    # the same GEMM on the split fp32 weights, tile shape 14 (the packed one's twin)
    wp = dev.put(W)
    xh, xl, wh, wl = dev.empty(M * K), dev.empty(M * K), dev.empty(N * K), dev.empty(N * K)
    tcg.check(L.tcg_split_tf32(xh.ptr, xl.ptr, xp, M * K))
    tcg.check(L.tcg_split_tf32(wh.ptr, wl.ptr, wp, N * K))
    y2 = dev.empty(M * N)
    tcg.check(L.tcg_linear_split_cfg(y2.ptr, xh.ptr, xl.ptr, wh.ptr, wl.ptr, bp, M, N, K, 14), "cfg 14")
    assert np.array_equal(got, y2.download((M, N)))
    assert L.tcg_device_error() == 0


def test_linear_q_refusals(dev):
    import tcg_gguf as G
    L = tcg.lib()
    d = dev.empty(64)
    assert not L.tcg_linear_q(d.ptr, d.ptr, d.ptr, None, 4, 4, 300, G.Q4_K)
    assert b"multiple of 256" in L.tcg_last_error()
    assert not L.tcg_linear_q(d.ptr, d.ptr, d.ptr, None, 4, 4, 256, G.Q6_K)
    assert b"Q4_K only" in L.tcg_last_error()

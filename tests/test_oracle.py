"""The oracle is pinned before anything is compared against it.

* K-quant arms: bit-exact against gguf 0.19.0's dequantize on the committed
  golden blocks (edge cases included).
* binary16 conversion: every one of the 65,536 inputs against the
  reference's own tc_f16_to_f32 (when oracle/_ref is built).
* ops: the reference's golden vectors (tests/fixtures/ops.gguf) within the
  reference's own tolerances (tests/test_ops.c:74-148), and bit-identical to
  the reference C when it is available.
* ViT: the reference's tc_vit_encode outputs committed in vit_golden.npz.
"""
import numpy as np
import pytest

import oracle
from fixtures_io import check_close, kquant_golden, ops_golden, rel_inf, vit_golden

import tcg_gguf as G


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("tag,qt", [("q4k", oracle.Q4_K), ("q6k", oracle.Q6_K)])
def test_kquant_matches_gguf_package_golden(tag, qt):
    g = kquant_golden()
    blocks, want = g[f"{tag}_blocks"], g[f"{tag}_values"]
    got = oracle.dequant(blocks.reshape(-1), want.size, qt)
    assert np.array_equal(bits(got), bits(want))


def test_kquant_rejects_partial_superblocks():
    raw = np.zeros(144, np.uint8)
    with pytest.raises(ValueError):
        oracle.dequant(raw, 255, oracle.Q4_K)
    with pytest.raises(ValueError):
        oracle.dequant(raw, 256, 13)          # Q5_K: no conversion, as the reference


def test_f16_all_inputs_match_reference():
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    ref = oracle.RefLib().lib
    h = np.arange(65536, dtype=np.uint16)
    want = np.empty(65536, np.float32)
    assert ref.tc_dequant(want.ctypes.data, h.ctypes.data, 65536, oracle.F16)
    assert np.array_equal(bits(oracle.f16_to_f32_all()), bits(want))


def test_f16_subnormal_and_specials():
    v = oracle.f16_to_f32_all()
    assert v[0x0001] == np.float32(2.0 ** -24)
    assert v[0x03FF] == np.float32(1023 * 2.0 ** -24)
    assert v[0x3C00] == 1.0 and v[0xBC00] == -1.0
    assert np.isinf(v[0x7C00]) and v[0x7C00] > 0
    assert bits(v)[0x7E01] == 0x7FC02000          # payload kept
    assert bits(v)[0x8000] == 0x80000000


def test_ops_golden_vectors():
    kv, t = ops_golden()
    for tag in ("small", "wide"):
        M, N, K = kv[f"gemm.{tag}.M"], kv[f"gemm.{tag}.N"], kv[f"gemm.{tag}.K"]
        got = oracle.gemm(t[f"gemm.{tag}.A"], t[f"gemm.{tag}.B"], M, N, K)
        check_close(got, t[f"gemm.{tag}.C"], 2e-4, 1e-5, f"gemm {tag}")
    M, N, K = kv["linear.M"], kv["linear.N"], kv["linear.K"]
    check_close(oracle.linear(t["linear.x"], t["linear.W"], t["linear.b"], M, N, K), t["linear.y"], 1e-5, 1e-5)
    got = oracle.layernorm(t["ln.x"], t["ln.gamma"], t["ln.beta"], kv["ln.rows"], kv["ln.cols"], kv["ln.eps"])
    check_close(got, t["ln.out"], 1e-4, 1e-4, "layernorm")
    check_close(oracle.gelu(t["gelu.x"]), t["gelu.exact"], 1e-6, 1e-6, "gelu")
    check_close(oracle.gelu(t["gelu.x"], quick=True), t["gelu.quick"], 1e-6, 1e-6, "gelu quick")
    assert np.abs(oracle.gelu(t["gelu.x"]) - oracle.gelu(t["gelu.x"], quick=True)).max() > 0.01
    sm = oracle.softmax_rows(t["softmax.x"], kv["softmax.rows"], kv["softmax.cols"])
    check_close(sm, t["softmax.out"], 1e-6, 1e-5, "softmax")
    assert np.all(np.abs(sm.astype(np.float64).sum(1) - 1.0) < 1e-5)
    got = oracle.mha(t["mha.q"], t["mha.k"], t["mha.v"], kv["mha.T"], kv["mha.n_head"], kv["mha.head_dim"])
    check_close(got, t["mha.out"], 1e-5, 1e-5, "mha")


def test_ops_port_bit_identical_to_reference():
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    ref = oracle.RefLib().lib
    kv, t = ops_golden()
    rng = np.random.default_rng(5)
    x = rng.standard_normal((9, 77)).astype(np.float32)
    W = rng.standard_normal((13, 77)).astype(np.float32)
    b = rng.standard_normal(13).astype(np.float32)
    want = np.empty((9, 13), np.float32)
    ref.tc_ref_linear(want.ctypes.data, x.ctypes.data, W.ctypes.data, b.ctypes.data, 9, 13, 77)
    assert np.array_equal(bits(oracle.linear(x, W, b, 9, 13, 77)), bits(want))
    q, k, v = (t["mha.q"], t["mha.k"], t["mha.v"])
    T, H, HD = kv["mha.T"], kv["mha.n_head"], kv["mha.head_dim"]
    want = np.empty((T, H * HD), np.float32)
    scratch = np.empty(T, np.float32)
    ref.tc_ref_mha(want.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data, T, H, HD, scratch.ctypes.data)
    assert np.array_equal(bits(oracle.mha(q, k, v, T, H, HD)), bits(want))
    want = np.empty((kv["ln.rows"], kv["ln.cols"]), np.float32)
    ref.tc_ref_layernorm(want.ctypes.data, t["ln.x"].ctypes.data, t["ln.gamma"].ctypes.data,
                         t["ln.beta"].ctypes.data, kv["ln.rows"], kv["ln.cols"], np.float32(kv["ln.eps"]))
    got = oracle.layernorm(t["ln.x"], t["ln.gamma"], t["ln.beta"], kv["ln.rows"], kv["ln.cols"], kv["ln.eps"])
    assert np.array_equal(bits(got), bits(want))


CASES = {"b32x2": ("vit-b32", dict(n_layer=2)), "l14x1": ("vit-l14", dict(n_layer=1))}


@pytest.mark.parametrize("tag", sorted(CASES))
def test_vit_port_matches_reference_golden(tag):
    g = vit_golden()
    name, over = CASES[tag]
    cfg = G.vit_config(name, **over)
    w = G.make_vit_weights(cfg, 0)
    px = G.make_pixels(1, cfg["image"], 1)[0]
    got = oracle.PortVit(cfg, w).forward(px)
    assert rel_inf(got["embedding"], g[f"{tag}.embedding"]) < 1e-6
    for k in ("ln_pre", "blk0", "blk_last", "ln_post"):
        assert rel_inf(got[k][0], g[f"{tag}.{k}.cls"]) < 1e-6
        t64 = got[k].astype(np.float64)
        np.testing.assert_allclose([t64.sum(), (t64 * t64).sum()], g[f"{tag}.{k}.sum"], rtol=1e-6, atol=1e-3)


def test_matvec_composition_is_dequant_then_linear():
    rng = np.random.default_rng(3)
    raw = G.make_kquant(G.Q4_K, 5, 512, seed=11)
    x = rng.standard_normal(512).astype(np.float32)
    Wf = oracle.dequant(raw, 5 * 512, oracle.Q4_K).reshape(5, 512)
    want = oracle.linear(x[None, :], Wf, None, 1, 5, 512)[0]
    assert np.array_equal(bits(oracle.matvec_q(raw, x, 5, 512, oracle.Q4_K)), bits(want))

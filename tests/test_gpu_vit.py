"""The batched ViT forward against the reference.

Bar (stated in the hot-path spec): every tap and the embedding within
max|err| <= 1e-4 * max|ref| per image, plus the reference's end-to-end gate
of embedding cosine >= 0.9999 (tests/test_vit.c:197).

* the committed outputs of the reference's own tc_vit_encode (vit_golden.npz)
  through the reference-shaped entry point tc_vit_encode;
* the full-depth ViT-B/32 over a batch, per image, against the oracle;
* batch invariance, graph replay == eager, and the argument checks.
"""
import ctypes

import numpy as np
import pytest

import oracle
import tcg
import tcg_gguf as G
from fixtures_io import rel_inf, vit_golden

pytestmark = pytest.mark.gpu

TOL = 1e-4
TAPS = ("ln_pre", "blk0", "blk_last", "ln_post")


def cosine(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def model(cache_dir, name, seed=0, **over):
    path, cfg = G.cached_vit_gguf(cache_dir, name, seed, **over)
    return path, cfg


CASES = {"b32x2": ("vit-b32", dict(n_layer=2)), "l14x1": ("vit-l14", dict(n_layer=1))}


@pytest.mark.parametrize("tag", sorted(CASES))
def test_reference_golden_through_tc_vit_encode(gpu, cache_dir, tag):
    g = vit_golden()
    name, over = CASES[tag]
    path, cfg = model(cache_dir, name, **over)
    m = tcg.VitModel(path)
    try:
        px = G.make_pixels(1, cfg["image"], 1)[0]
        out, taps = m.encode_single(px, taps=True)
        assert set(taps) == set(TAPS) | {"embedding"}
        assert rel_inf(out, g[f"{tag}.embedding"]) <= TOL
        assert cosine(out, g[f"{tag}.embedding"]) >= 0.9999
        for k in TAPS:
            assert taps[k].shape == (cfg["n_token"], cfg["d_model"])
            assert rel_inf(taps[k][0], g[f"{tag}.{k}.cls"]) <= TOL, k
            t64 = taps[k].astype(np.float64)
            s, ss = g[f"{tag}.{k}.sum"]
            assert abs(t64.sum() - s) <= TOL * np.abs(t64).sum()
            assert abs((t64 * t64).sum() - ss) <= 10 * TOL * ss
    finally:
        m.close()


def test_b32_full_depth_batch_vs_oracle(gpu, cache_dir):
    path, cfg = model(cache_dir, "vit-b32")
    w = G.make_vit_weights(cfg, 0)
    px = G.make_pixels(3, cfg["image"], 1)
    port = oracle.PortVit(cfg, w)
    m = tcg.VitModel(path)
    try:
        m.upload(8)
        out, taps = m.encode(px, taps=True)
        for i in (0, 2):
            ref = port.forward(px[i])
            assert rel_inf(out[i], ref["embedding"]) <= TOL
            assert cosine(out[i], ref["embedding"]) >= 0.9999
            for k in TAPS:
                assert rel_inf(taps[k][i], ref[k]) <= TOL, (i, k, rel_inf(taps[k][i], ref[k]))
    finally:
        m.close()


def test_b32_one_wave_shapes_vs_oracle(gpu, cache_dir):
    """64 images, the shard of a 4-GPU run: the patch, out and down GEMMs
    make one wave of 128 x 128 tiles plus two, so they run the 128 x 256 and
    separate-accumulator shapes. First and last image against the oracle;
    the whole batch against the forward with every GEMM on the 128 x 128
    shape."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=2)
    w = G.make_vit_weights(cfg, 0)
    px = G.make_pixels(64, cfg["image"], 3)
    m = tcg.VitModel(path)
    try:
        old_f16 = L.tcg_vit_set_f16(0)          # the tf32-pair GEMMs' shape rule
        try:
            m.upload(64)
        finally:
            L.tcg_vit_set_f16(old_f16)
        out, taps = m.encode(px, taps=True)
        plan = (ctypes.c_int * 4)()
        L.tcg_gemm_last_plan(plan)              # the last plan made: the last layer's down projection
        assert plan[2] == 7, list(plan)
        again, _ = m.encode(px)                 # graph replay
        assert np.array_equal(out, again)
    finally:
        m.close()
    port = oracle.PortVit(cfg, w)
    for i in (0, 63):
        ref = port.forward(px[i])
        assert rel_inf(out[i], ref["embedding"]) <= TOL
        for k in TAPS:
            assert rel_inf(taps[k][i], ref[k]) <= TOL, (i, k)
    old = L.tcg_gemm_force_cfg(13)
    try:
        m = tcg.VitModel(path)
        try:
            m.upload(64)
            wide, _ = m.encode(px)
        finally:
            m.close()
    finally:
        L.tcg_gemm_force_cfg(old)
    for i in range(64):
        assert rel_inf(out[i], wide[i]) <= TOL, i
    assert L.tcg_device_error() == 0


def test_l14_two_layers_vs_oracle(gpu, cache_dir):
    path, cfg = model(cache_dir, "vit-l14", n_layer=2)
    w = G.make_vit_weights(cfg, 0)
    px = G.make_pixels(2, cfg["image"], 4)
    m = tcg.VitModel(path)
    try:
        m.upload(2)
        out, taps = m.encode(px, taps=True)
        ref = oracle.PortVit(cfg, w).forward(px[1])
        assert rel_inf(out[1], ref["embedding"]) <= TOL
        for k in TAPS:
            assert rel_inf(taps[k][1], ref[k]) <= TOL, k
    finally:
        m.close()


def test_l14_tensor_core_attention_vs_oracle(gpu, cache_dir):
    """ViT-L/14 (T = 257) with attention on the tensor cores, two images."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-l14", n_layer=2)
    w = G.make_vit_weights(cfg, 0)
    px = G.make_pixels(2, cfg["image"], 4)
    old = L.tcg_set_attention_variant(3)
    m = tcg.VitModel(path)
    try:
        m.upload(2)
        out, taps = m.encode(px, taps=True)
        for i in (0, 1):
            ref = oracle.PortVit(cfg, w).forward(px[i])
            assert rel_inf(out[i], ref["embedding"]) <= TOL
            for k in TAPS:
                assert rel_inf(taps[k][i], ref[k]) <= TOL, (i, k)
        assert L.tcg_device_error() == 0
    finally:
        m.close()
        L.tcg_set_attention_variant(old)


def test_batch_invariance_and_graph_replay(gpu, cache_dir):
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=3)
    px = G.make_pixels(9, cfg["image"], 7)
    old = L.tcg_gemm_set_streamk(0)             # whole tiles: each row's K order is the batch's
    m = tcg.VitModel(path)
    try:
        m.upload(9)
        full, _ = m.encode(px)                  # first call: eager, then recorded
        again, _ = m.encode(px)                 # graph replay
        assert np.array_equal(full, again)
        one, _ = m.encode(px[4:5])
        assert np.array_equal(one[0], full[4])  # same K order whatever the batch
        L.tcg_vit_use_graphs(m.dev, False)
        eager, _ = m.encode(px)
        assert np.array_equal(eager, full)
        assert L.tcg_device_error() == 0
    finally:
        m.close()
        L.tcg_gemm_set_streamk(old)


def test_streamk_forward(gpu, cache_dir):
    """With the stream-K split (the default) a batch's result depends on how
    its GEMMs' last waves are cut, so it is deterministic per batch size and
    within the tolerance of the whole-tile result."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=3)
    px = G.make_pixels(9, cfg["image"], 7)
    outs = {}
    for sk in (0, 1):
        old = L.tcg_gemm_set_streamk(sk)
        m = tcg.VitModel(path)
        try:
            m.upload(9)
            a, _ = m.encode(px)
            b, _ = m.encode(px)                 # graph replay
            assert np.array_equal(a, b)
            outs[sk] = a
        finally:
            m.close()
            L.tcg_gemm_set_streamk(old)
    for i in range(9):
        assert rel_inf(outs[1][i], outs[0][i]) <= TOL
    assert L.tcg_device_error() == 0


def test_bulk_store_epilogue_matches_plain_stores(gpu, cache_dir):
    """The GEMM epilogue that writes through bulk tensor stores (rows one to
    one, lane = row) does the same round-to-nearest operations, in the same
    order, as the plain-store one: the embeddings are identical, bit for bit.
    Batch 9 leaves the last row tile partly and wholly below the matrix."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=3)
    px = G.make_pixels(9, cfg["image"], 11)
    outs = {}
    for t in (0, 1):
        old = L.tcg_gemm_set_tma_store(t)
        m = tcg.VitModel(path)
        try:
            m.upload(9)
            outs[t], _ = m.encode(px)
        finally:
            m.close()
            L.tcg_gemm_set_tma_store(old)
    assert np.array_equal(outs[0], outs[1])
    assert L.tcg_device_error() == 0


def test_async_submit_matches_blocking(gpu, cache_dir):
    import ctypes
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=2)
    m = tcg.VitModel(path)
    bufs = []
    try:
        m.upload(4)
        batches = [G.make_pixels(n, cfg["image"], 20 + i) for i, n in enumerate((4, 3, 4, 2))]
        want = [m.encode(b)[0] for b in batches]
        ins = [tcg.HostBuffer(b.shape) for b in batches]
        outs = [tcg.HostBuffer((b.shape[0], cfg["d_out"])) for b in batches]
        bufs = ins + outs
        tickets = []
        for hb, ob, b in zip(ins, outs, batches):       # the third submission waits for the first
            hb.array[...] = b
            t = ctypes.c_int(-1)
            tcg.check(L.tcg_vit_submit(m.dev, hb.ptr, b.shape[0], ob.ptr, ctypes.byref(t)), "submit")
            tickets.append(t.value)
        assert tickets == sorted(tickets) and len(set(tickets)) == 4
        for t in reversed(tickets):
            tcg.check(L.tcg_vit_wait(m.dev, t), "wait")
        for ob, w in zip(outs, want):
            assert np.array_equal(ob.array, w)
        again, _ = m.encode(batches[0])                 # a blocking call after the async ones
        assert np.array_equal(again, want[0])
        assert not L.tcg_vit_submit(m.dev, ins[0].ptr, 5, outs[0].ptr, None)     # > max_batch
        assert not L.tcg_vit_wait(m.dev, 99)
    finally:
        for b in bufs:
            b.close()
        m.close()


def test_quick_gelu_model(gpu, tmp_path):
    cfg = G.vit_config("vit-b32", n_layer=1)
    w = G.make_vit_weights(cfg, 3)
    path = str(tmp_path / "q.gguf")
    G.write_vit_gguf(path, cfg, w, activation="gelu_quick")
    px = G.make_pixels(1, cfg["image"], 2)
    m = tcg.VitModel(path)
    try:
        m.upload(1)
        out, _ = m.encode(px)
        ref = oracle.PortVit(cfg, w, quick_gelu=True).forward(px[0], taps=False)
        assert rel_inf(out[0], ref["embedding"]) <= TOL
    finally:
        m.close()


def _kquant_like(qt, rows, cols, seed, d_std):
    """Random K-quant blocks of a [rows, cols] matrix whose weights have a
    trained model's scale: the fp16 super-scales d (and dmin) ~ |N(0, d_std)|,
    many of them fp16 subnormals."""
    nb = rows * cols // 256
    blk = (G.make_q4k_blocks if qt == G.Q4_K else G.make_q6k_blocks)(nb, seed)
    rng = np.random.default_rng(seed + 1)
    half = lambda: np.abs(rng.normal(0.0, d_std, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)  # noqa: E731
    if qt == G.Q4_K:
        blk[:, 0:2] = half()
        blk[:, 2:4] = half()
    else:
        blk[:, 208:210] = half()
    return blk.reshape(-1)


def test_kquant_weights_model(gpu, tmp_path):
    """A ViT-B/32 (two layers) whose linear weights are K-quant tensors: Q4_K
    qkv and up projections, Q6_K out, down and the output projection.
    tc_vit_load materialises them through the dequant seam (src/vit.c:17-37,
    tc_dequant_view with the Q4_K / Q6_K arms), so the forward must equal the
    fp32 model of the dequantised weights."""
    cfg = G.vit_config("vit-b32", n_layer=2)
    w = G.make_vit_weights(cfg, 5)
    quant = {"attn_qkv.weight": (G.Q4_K, 4e-5), "ffn_up.weight": (G.Q4_K, 4e-5),
             "attn_out.weight": (G.Q6_K, 3e-6), "ffn_down.weight": (G.Q6_K, 3e-6), "v.proj": (G.Q6_K, 3e-6)}
    tensors = []
    for k, (name, arr) in enumerate(list(w.items())):
        key = name if name == "v.proj" else ".".join(name.split(".")[-2:])
        if key in quant:
            qt, d_std = quant[key]
            rows, cols = arr.shape
            raw = _kquant_like(qt, rows, cols, 100 + k, d_std)
            w[name] = oracle.dequant(raw, rows * cols, qt).reshape(rows, cols)
            tensors.append((name, raw, qt, arr.shape))
        else:
            tensors.append((name, arr, G.F32, arr.shape))
    assert sum(t[2] != G.F32 for t in tensors) == 4 * cfg["n_layer"] + 1
    path = str(tmp_path / "kq.gguf")
    G.write_gguf(path, G.vit_metadata(cfg), tensors)
    px = G.make_pixels(2, cfg["image"], 6)
    port = oracle.PortVit(cfg, w)
    m = tcg.VitModel(path)
    try:
        m.upload(2)
        out, taps = m.encode(px, taps=True)
        for i in range(2):
            ref = port.forward(px[i])
            assert rel_inf(out[i], ref["embedding"]) <= TOL, i
            assert cosine(out[i], ref["embedding"]) >= 0.9999
            for k in TAPS:
                assert rel_inf(taps[k][i], ref[k]) <= TOL, (i, k)
    finally:
        m.close()


@pytest.mark.parametrize("n_img,jit_rows", [(3, 0), (64, 0), (3, 1), (64, 1)])
def test_packed_q4k_weights_model(gpu, tmp_path, n_img, jit_rows):
    """Every block linear weight of a ViT-B/32 (two layers) in Q4_K: the
    device keeps them packed (144 bytes per 256 weights) and each GEMM
    dequantises its tiles in shared memory. Against the oracle's fp32 model
    of the dequantised weights, per tap; and against the same model uploaded
    with the weights dequantised at load. jit_rows 1: every batch dequantises
    each packed weight into a tf32 pair just before its GEMM instead."""
    L = tcg.lib()
    old_jit = L.tcg_vit_set_jit_rows(jit_rows if jit_rows else 1 << 40)
    cfg = G.vit_config("vit-b32", n_layer=2)
    path = str(tmp_path / "q4k.gguf")
    made = G.write_kquant_vit_gguf(path, cfg, seed=9)
    w = dict(made["fp32"])
    for name, (blocks, qt, shape) in made["kquant"].items():
        w[name] = oracle.dequant(blocks, int(np.prod(shape)), qt).reshape(shape)
    px = G.make_pixels(n_img, cfg["image"], 6)
    outs, nbytes, f16 = {}, {}, {}
    for packed in (1, 0):
        old = L.tcg_vit_set_packed_weights(packed)
        m = tcg.VitModel(path)
        try:
            m.upload(n_img)
            outs[packed] = m.encode(px, taps=True)
            nbytes[packed] = L.tcg_vit_gemm_weight_bytes(m.dev)
            f16[packed] = L.tcg_vit_uses_f16(m.dev)
        finally:
            m.close()
            L.tcg_vit_set_packed_weights(old)
    L.tcg_vit_set_jit_rows(old_jit)
    D, F, L_, K0 = cfg["d_model"], cfg["d_ffn"], cfg["n_layer"], 3 * cfg["patch"] ** 2
    linear = L_ * (3 * D * D + D * D + 2 * F * D)
    # packed blocks (each tensor's slot padded to 256 bytes) plus the patch embedding's tf32 pair
    assert f16[1] == 0
    assert abs(nbytes[1] - (linear // 256 * 144 + 8 * D * K0)) <= 256 * 4 * L_
    # dequantised at load, every weight fp32 on the device: fp16 pieces (4 bytes
    # a weight, one exponent per row, slots padded to 256 bytes)
    assert f16[0] == 2
    rows = L_ * (3 * D + D + F + D) + D
    assert 4 * (linear + D * K0) + rows <= nbytes[0] <= 4 * (linear + D * K0) + rows + 3 * 256 * (4 * L_ + 1)
    out, taps = outs[1]
    port = oracle.PortVit(cfg, w)
    for i in sorted({0, n_img - 1}):
        ref = port.forward(px[i])
        assert rel_inf(out[i], ref["embedding"]) <= TOL, i
        assert cosine(out[i], ref["embedding"]) >= 0.9999
        for k in TAPS:
            assert rel_inf(taps[k][i], ref[k]) <= TOL, (i, k)
    for i in range(n_img):
        assert rel_inf(out[i], outs[0][0][i]) <= 1e-5, i
    assert L.tcg_device_error() == 0


@pytest.mark.parametrize("n_img", [3, 64])
def test_fp16_piece_and_tf32_pair_gemms(gpu, cache_dir, n_img):
    """The same fp32 ViT-B/32 (two layers) with its GEMMs on fp16 pieces
    (tcg_vit_set_f16(1), the default: LayerNorm writes the pieces, the
    attention and GELU outputs are split) and on tf32 pairs: both against the
    oracle per tap, and against each other."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=2)
    px = G.make_pixels(n_img, cfg["image"], 12)
    outs = {}
    for mode in (1, 0):
        old = L.tcg_vit_set_f16(mode)
        m = tcg.VitModel(path)
        try:
            m.upload(n_img)
            assert L.tcg_vit_uses_f16(m.dev) == (2 if mode else 0)
            outs[mode] = m.encode(px, taps=True)
        finally:
            m.close()
            L.tcg_vit_set_f16(old)
    port = oracle.PortVit(cfg, G.make_vit_weights(cfg, 0))
    for i in range(n_img):
        assert rel_inf(outs[1][0][i], outs[0][0][i]) <= 1e-5, i
    for mode in (1, 0):
        out, taps = outs[mode]
        for i in sorted({0, n_img - 1}):
            ref = port.forward(px[i])
            assert rel_inf(out[i], ref["embedding"]) <= TOL, (mode, i)
            for k in TAPS:
                assert rel_inf(taps[k][i], ref[k]) <= TOL, (mode, i, k)
    assert L.tcg_device_error() == 0


def test_fp16_piece_gemm_configurations(gpu, cache_dir):
    """The fp16-piece ViT forward with each fp16 GEMM configuration (128 x 128
    tiles with three stages of 64 K-elements or six of 32; CTA pairs on 256 x
    256 or 256 x 128 tiles; the three products folded): against the default
    and the oracle."""
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=2)
    n_img = 64
    px = G.make_pixels(n_img, cfg["image"], 13)
    outs = {}
    for c in (16, 17, 18, 19, 20):
        old = L.tcg_gemm_set_f16_cfg(c)
        m = tcg.VitModel(path)
        try:
            m.upload(n_img)
            assert L.tcg_vit_uses_f16(m.dev) == 2
            outs[c] = m.encode(px)[0]
        finally:
            m.close()
            L.tcg_gemm_set_f16_cfg(old)
    port = oracle.PortVit(cfg, G.make_vit_weights(cfg, 0))
    refs = {i: port.forward(px[i])["embedding"] for i in (0, n_img - 1)}
    for c in (17, 18, 19, 20):
        for i in range(n_img):
            assert rel_inf(outs[c][i], outs[16][i]) <= 1e-5, (c, i)
        for i in refs:
            assert rel_inf(outs[c][i], refs[i]) <= TOL, (c, i)
    assert L.tcg_device_error() == 0


def test_device_entry_and_limits(gpu, cache_dir):
    L = tcg.lib()
    path, cfg = model(cache_dir, "vit-b32", n_layer=1)
    px = G.make_pixels(4, cfg["image"], 3)
    m = tcg.VitModel(path)
    try:
        m.upload(4)
        host_out, _ = m.encode(px)
        with tcg.DeviceBuffer.from_array(px) as dpx, tcg.DeviceBuffer(4 * cfg["d_out"] * 4) as dout:
            tcg.check(L.tcg_vit_encode_device(m.dev, dpx.ptr, 4, dout.ptr))
            tcg.sync()
            assert np.array_equal(dout.download((4, cfg["d_out"])), host_out)
            assert not L.tcg_vit_encode_device(m.dev, dpx.ptr, 5, dout.ptr)
            assert b"max_batch" in L.tcg_last_error()
            assert L.tcg_vit_encode_device(m.dev, dpx.ptr, 0, dout.ptr)
        assert L.tcg_vit_max_batch(m.dev) == 4
        assert L.tcg_vit_device_bytes(m.dev) > 0
    finally:
        m.close()

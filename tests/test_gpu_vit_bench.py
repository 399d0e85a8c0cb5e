"""The ViT forward at the shapes the benchmark times, against the
reference's own outputs.

bench.py times ViT-B/32 with a batch of 256 images per GPU, rank r's pixels
drawn with seed 1 + r (ViT-L/14: 128 per GPU); with --strong one batch of
256 is split into 128 / 64 / 32 images per GPU on 2 / 4 / 8 GPUs (ViT-L/14:
16 per GPU on 8). Both forms are covered: every rank's own batch, and the
shards of the seed-1 batch.
Every one of those batch sizes plans its GEMMs differently (tile shapes,
the one-wave rule, the stream-K split of the last wave) and ViT-L/14 runs
the tensor-core attention with its one-row tail. Here each of those
per-GPU batches runs at full depth, through the entry points the benchmark
uses (tcg_vit_encode_device for `value`, tcg_vit_submit/wait for `e2e`), on
the benchmark's own model (weights seed 0) and pixels (seed 1); the first
and last image of every shard and one middle image are compared with the
embeddings of roofline.c's tc_vit_encode (src/vit.c:219-305) frozen in
tests/golden/vit_bench_golden.npz.

Bar: max|err| <= 1e-4 * max|ref| per image and cosine >= 0.9999
(the reference's end-to-end gate, tests/test_vit.c:197).
"""
import ctypes

import numpy as np
import pytest

import tcg
import tcg_gguf as G
from fixtures_io import rel_inf, vit_bench_golden

pytestmark = pytest.mark.gpu

TOL = 1e-4


def cosine(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def _run_shards(cache_dir, name, per):
    g = vit_bench_golden()
    idx, ref, batch = g[f"{name}.index"], g[f"{name}.embedding"], int(g[f"{name}.batch"])
    path, cfg = G.cached_vit_gguf(cache_dir, name, 0)
    px = G.make_pixels(batch, cfg["image"], 1)
    L = tcg.lib()
    m = tcg.VitModel(path)
    worst = 0.0
    try:
        m.upload(per)
        d_out = cfg["d_out"]
        with tcg.DeviceBuffer(per * px[0].nbytes) as dpx, tcg.DeviceBuffer(per * d_out * 4) as dout:
            for s0 in range(0, batch, per):
                shard = np.ascontiguousarray(px[s0:s0 + per])
                dpx.upload(shard)
                tcg.check(L.tcg_vit_encode_device(m.dev, dpx.ptr, per, dout.ptr), "tcg_vit_encode_device")
                tcg.sync()
                out = dout.download((per, d_out))
                for j, i in enumerate(idx):
                    if s0 <= i < s0 + per:
                        e = rel_inf(out[i - s0], ref[j])
                        worst = max(worst, e)
                        assert e <= TOL, (name, per, int(i), e)
                        assert cosine(out[i - s0], ref[j]) >= 0.9999, (name, per, int(i))
                if s0 == 0:
                    # the serving entry point of the e2e measurement: same graph, same bits
                    hpx, hout = tcg.HostBuffer(shard.shape), tcg.HostBuffer((per, d_out))
                    try:
                        hpx.array[...] = shard
                        tk = ctypes.c_int(0)
                        tcg.check(L.tcg_vit_submit(m.dev, hpx.ptr, per, hout.ptr, ctypes.byref(tk)), "submit")
                        tcg.check(L.tcg_vit_wait(m.dev, tk.value), "wait")
                        assert np.array_equal(hout.array, out)
                    finally:
                        hpx.close()
                        hout.close()
        assert L.tcg_device_error() == 0
    finally:
        m.close()
    return worst


@pytest.mark.parametrize("per", [256, 128, 64, 32])
def test_b32_bench_shards_full_depth_vs_reference(gpu, cache_dir, per):
    _run_shards(cache_dir, "vit-b32", per)


@pytest.mark.slow
@pytest.mark.parametrize("per", [128, 16])
def test_l14_bench_shards_full_depth_vs_reference(gpu, cache_dir, per):
    _run_shards(cache_dir, "vit-l14", per)


def _run_rank_batches(cache_dir, name):
    """Every rank's own batch of bench.py's default form (pixel seed 1 + r,
    r < 8), one upload: first, middle and last image against the reference."""
    g = vit_bench_golden()
    seeds, widx, wref = g[f"{name}.weak_seeds"], g[f"{name}.weak_index"], g[f"{name}.weak_embedding"]
    batch = int(g[f"{name}.batch"])
    path, cfg = G.cached_vit_gguf(cache_dir, name, 0)
    L = tcg.lib()
    m = tcg.VitModel(path)
    try:
        m.upload(batch)
        d_out = cfg["d_out"]
        with tcg.DeviceBuffer(batch * 3 * cfg["image"] ** 2 * 4) as dpx, tcg.DeviceBuffer(batch * d_out * 4) as dout:
            for r, sd in enumerate(seeds):
                dpx.upload(G.make_pixels(batch, cfg["image"], int(sd)))
                tcg.check(L.tcg_vit_encode_device(m.dev, dpx.ptr, batch, dout.ptr), "tcg_vit_encode_device")
                tcg.sync()
                out = dout.download((batch, d_out))
                for j, i in enumerate(widx):
                    e = rel_inf(out[i], wref[r, j])
                    assert e <= TOL, (name, int(sd), int(i), e)
                    assert cosine(out[i], wref[r, j]) >= 0.9999, (name, int(sd), int(i))
        assert L.tcg_device_error() == 0
    finally:
        m.close()


def test_b32_rank_batches_full_depth_vs_reference(gpu, cache_dir):
    _run_rank_batches(cache_dir, "vit-b32")


@pytest.mark.slow
def test_l14_rank_batches_full_depth_vs_reference(gpu, cache_dir):
    _run_rank_batches(cache_dir, "vit-l14")

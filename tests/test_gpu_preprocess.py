"""CLIP preprocessing on the device (tcg_preprocess_rgb8, tcg_vit_preprocess)
against the fixture made by torchvision + Pillow and against the CPU
restatement (itself pinned to Pillow and torchvision in
tests/test_preprocess.py): the same float32 bits, since the 8-bit resized
pixels are exact and the rest is the same IEEE operations."""
import ctypes

import numpy as np
import pytest

import tcg
import tcg_gguf as G
from fixtures_io import GOLDEN
from oracle import preprocess as P

pytestmark = pytest.mark.gpu

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


def _dev_pre(rgb, image, mean, std, interp):
    L = tcg.lib()
    n, h, w, _ = rgb.shape
    m = (ctypes.c_float * 3)(*mean)
    s = (ctypes.c_float * 3)(*std)
    with tcg.DeviceBuffer.from_array(np.ascontiguousarray(rgb)) as d_in, \
            tcg.DeviceBuffer(n * 3 * image * image * 4) as d_out:
        tcg.check(L.tcg_preprocess_rgb8(d_out.ptr, d_in.ptr, n, h, w, image, m, s, interp), "tcg_preprocess_rgb8")
        return d_out.download((n, 3, image, image))


def test_device_preprocess_matches_fixture(gpu):
    g = dict(np.load(f"{GOLDEN}/preprocess_golden.npz"))
    i = 0
    while f"case{i}.rgb" in g:
        h, w, image, interp = (int(v) for v in g[f"case{i}.meta"])
        got = _dev_pre(g[f"case{i}.rgb"], image, g["mean"], g["std"], interp)
        assert np.array_equal(got, g[f"case{i}.pixels"]), i
        i += 1


@pytest.mark.parametrize("h,w,interp", [(480, 640, 0), (640, 480, 0), (300, 257, 1), (224, 224, 0),
                                        (1080, 1920, 0), (120, 90, 0)])
def test_device_preprocess_matches_restatement(gpu, h, w, interp):
    rng = np.random.default_rng(h + 7 * w)
    rgb = rng.integers(0, 256, (3, h, w, 3), dtype=np.uint8)
    got = _dev_pre(rgb, 224, CLIP_MEAN, CLIP_STD, interp)
    want = P.preprocess(rgb, 224, CLIP_MEAN, CLIP_STD, "bicubic" if interp == 0 else "bilinear")
    assert np.array_equal(got, want)
    assert tcg.lib().tcg_device_error() == 0


def test_vit_preprocess_reads_the_model(gpu, cache_dir):
    """tcg_vit_preprocess takes image size, mean, std and filter from the
    GGUF, and refuses a filter it does not implement."""
    L = tcg.lib()
    path, cfg = G.cached_vit_gguf(cache_dir, "vit-b32", 0, n_layer=1)
    m = tcg.VitModel(path)
    try:
        rng = np.random.default_rng(3)
        rgb = rng.integers(0, 256, (2, 300, 400, 3), dtype=np.uint8)
        with tcg.DeviceBuffer.from_array(rgb) as d_in, tcg.DeviceBuffer(2 * 3 * 224 * 224 * 4) as d_out:
            tcg.check(L.tcg_vit_preprocess(ctypes.byref(m.m), d_out.ptr, d_in.ptr, 2, 300, 400), "tcg_vit_preprocess")
            got = d_out.download((2, 3, 224, 224))
        want = P.preprocess(rgb, 224, list(m.m.mean), list(m.m.std), "bicubic")
        assert np.array_equal(got, want)
    finally:
        m.close()
    assert not L.tcg_preprocess_rgb8(None, None, 1, 10, 10, 8, (ctypes.c_float * 3)(1, 1, 1),
                                     (ctypes.c_float * 3)(1, 1, 1), 5)
    assert b"interpolation" in L.tcg_last_error()

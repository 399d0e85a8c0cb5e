"""CLIP image preprocessing: the CPU restatement (oracle/preprocess.py)
pinned against Pillow's resize and torchvision's transforms, and against
the committed fixture those made (tests/golden/preprocess_golden.npz).

The pipeline is open_clip's eval transform, which roofline.c leaves to the
caller (src/vit.h:75-78) and whose parameters its exporter records
(clip-vit.preprocess.*, tools/export_vit_gguf.py:291-294).
"""
import numpy as np
import pytest

from fixtures_io import GOLDEN
from oracle import preprocess as P

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


@pytest.mark.parametrize("h,w,image", [(37, 53, 24), (61, 40, 24), (100, 100, 24), (24, 24, 24),
                                       (300, 257, 224), (480, 640, 224), (23, 90, 16), (200, 199, 224)])
@pytest.mark.parametrize("interp", ["bicubic", "bilinear"])
def test_resize_matches_pillow(h, w, image, interp):
    Image = pytest.importorskip("PIL.Image")
    rng = np.random.default_rng(h * 1000 + w)
    a = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    rh, rw = P.resized_size(h, w, image)
    mode = Image.BICUBIC if interp == "bicubic" else Image.BILINEAR
    want = np.asarray(Image.fromarray(a).resize((rw, rh), mode))
    assert np.array_equal(P.resize_uint8(a, rh, rw, interp), want)


@pytest.mark.parametrize("h,w,image", [(37, 53, 24), (90, 23, 16), (300, 257, 224)])
def test_pipeline_matches_torchvision(h, w, image):
    pytest.importorskip("torchvision")
    import os
    import sys
    sys.path.insert(0, GOLDEN)
    import make_golden as M
    rng = np.random.default_rng(h + w)
    rgb = rng.integers(0, 256, (2, h, w, 3), dtype=np.uint8)
    want = M.torchvision_preprocess(rgb, image, "bicubic")
    assert np.array_equal(P.preprocess(rgb, image, CLIP_MEAN, CLIP_STD), want)


def test_pipeline_matches_fixture():
    g = dict(np.load(f"{GOLDEN}/preprocess_golden.npz"))
    i = 0
    while f"case{i}.rgb" in g:
        h, w, image, interp = (int(v) for v in g[f"case{i}.meta"])
        got = P.preprocess(g[f"case{i}.rgb"], image, g["mean"], g["std"], "bicubic" if interp == 0 else "bilinear")
        assert np.array_equal(got, g[f"case{i}.pixels"]), i
        i += 1
    assert i >= 6

#!/usr/bin/env python3
"""Regenerate the committed golden fixtures in tests/golden/.

Runs only where the reference tree and the third-party `gguf` package are
available (the build container); the fixtures it writes travel with the
repository, so the GPU tests never need either.

  ops.gguf           byte copy of roofline.c's op golden vectors
                     (tests/fixtures/ops.gguf, written by its
                     tools/gen_op_fixtures.py, numpy fp64 references), checked
                     against the sha256 recorded below.
  kquant_golden.npz  seeded Q4_K / Q6_K superblocks, including edge cases
                     (zero, subnormal, negative and largest fp16 scales; all-0
                     and all-1 bit patterns), with the fp32 values produced by
                     gguf 0.19.0's gguf.quants.dequantize -- an implementation
                     independent of this repository's oracle.
  vit_golden.npz     outputs of the reference's own tc_vit_encode
                     (oracle/_ref/libtcref.so, built from the reference
                     sources) on seeded synthetic models: embedding, CLS row
                     and per-tap float64 sums for two shapes.
  preprocess_golden.npz  uint8 RGB images and their CLIP preprocessing by
                     torchvision 0.26 + Pillow 12.2 (Resize of the shorter
                     side, CenterCrop, ToTensor, Normalize), small sizes.
  vit_bench_golden.npz  the same tc_vit_encode at full depth on the
                     benchmark's own models and batches (ViT-B/32 batch 256,
                     ViT-L/14 batch 128): embeddings of the first and last
                     image of every 1/2/4/8-GPU shard and one middle image.

    python tests/golden/make_golden.py
"""
import hashlib
import os
import shutil
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "roofline.c_b200")]
import oracle  # noqa: E402
import tcg_gguf as G  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TC_REFERENCE", "")
OPS_SHA256 = "56160063ceb733fe6ad2f8022bb8c2f75b64181511109fb657cc3b040537279a"


def ops_fixture():
    src = os.path.join(REF, "tests", "fixtures", "ops.gguf")
    digest = hashlib.sha256(open(src, "rb").read()).hexdigest()
    assert digest == OPS_SHA256, f"reference fixture changed: {digest}"
    shutil.copyfile(src, os.path.join(OUT, "ops.gguf"))


def _edge_q4k():
    rows = []
    for d, dmin, fill in ((0x0000, 0x0000, 0x5A), (0x0001, 0x03FF, 0xFF), (0x8400, 0x3C00, 0x00),
                          (0x7BFF, 0x7BFF, 0xFF), (0xBC00, 0x0001, 0x0F), (0x3555, 0x8001, 0xF0)):
        b = np.full(144, fill, np.uint8)
        b[0:2] = np.array([d], np.uint16).view(np.uint8)
        b[2:4] = np.array([dmin], np.uint16).view(np.uint8)
        rows.append(b)
    b = G.make_q4k_blocks(1, 99)[0].copy()
    b[4:16] = 0xFF          # every 6-bit scale and min = 63, top bits set
    rows.append(b)
    return np.stack(rows)


def _edge_q6k():
    rows = []
    for d, fill, sc in ((0x0000, 0x33, 5), (0x0001, 0xFF, -128), (0x8400, 0x00, 127),
                        (0x7BFF, 0xFF, 127), (0xBC00, 0x0F, -1), (0x03FF, 0xF0, -128)):
        b = np.full(210, fill, np.uint8)
        b[192:208] = np.array([sc] * 16, np.int8).view(np.uint8)
        b[208:210] = np.array([d], np.uint16).view(np.uint8)
        rows.append(b)
    return np.stack(rows)


def kquant_fixture():
    import gguf
    from gguf import quants
    out = {}
    for tag, qt, rand, edge in (("q4k", G.Q4_K, G.make_q4k_blocks(57, 2), _edge_q4k()),
                                ("q6k", G.Q6_K, G.make_q6k_blocks(57, 2), _edge_q6k())):
        blocks = np.concatenate([rand, edge])
        vals = quants.dequantize(blocks.reshape(-1), gguf.GGMLQuantizationType(qt)).reshape(-1)
        vals = np.ascontiguousarray(vals, np.float32)
        mine = oracle.dequant(blocks.reshape(-1), vals.size, qt)
        assert np.array_equal(mine.view(np.uint32), vals.view(np.uint32)), tag
        out[f"{tag}_blocks"] = blocks
        out[f"{tag}_values"] = vals
    out["gguf_version"] = np.array(gguf.__name__ + " 0.19.0")
    np.savez_compressed(os.path.join(OUT, "kquant_golden.npz"), **out)


# (name, config overrides, weight seed, pixel seed)
VIT_CASES = (
    ("b32x2", dict(name="vit-b32", n_layer=2), 0, 1),
    ("l14x1", dict(name="vit-l14", n_layer=1), 0, 1),
)


def vit_fixture():
    import tempfile
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for tag, over, wseed, pseed in VIT_CASES:
            over = dict(over)
            name = over.pop("name")
            cfg = G.vit_config(name, **over)
            w = G.make_vit_weights(cfg, wseed)
            path = os.path.join(tmp, tag + ".gguf")
            G.write_vit_gguf(path, cfg, w)
            px = G.make_pixels(1, cfg["image"], pseed)[0]
            rv = oracle.RefVit(path)
            taps = rv.encode(px, cfg["d_out"], taps=True)
            rv.close()
            out[f"{tag}.embedding"] = taps["embedding"]
            for k in ("ln_pre", "blk0", "blk_last", "ln_post"):
                t = taps[k].astype(np.float64)
                out[f"{tag}.{k}.cls"] = taps[k][0]
                out[f"{tag}.{k}.sum"] = np.array([t.sum(), (t * t).sum()])
    np.savez_compressed(os.path.join(OUT, "vit_golden.npz"), **out)


# Images of the benchmark's batches whose full-depth embeddings are frozen:
# the first and last image of every shard of a 1/2/4/8-GPU run (the shard
# edges), plus one from the middle of the batch.
BENCH_CASES = (
    # (model, batch, pixel seed)
    ("vit-b32", 256, 1),
    ("vit-l14", 128, 1),
)


def bench_indices(batch: int) -> list:
    idx = {batch // 2 + 5}
    for world in (1, 2, 4, 8):
        per = batch // world
        for r in range(world):
            idx.update((r * per, r * per + per - 1))
    return sorted(idx)


# bench.py's default multi-GPU form: rank r encodes a whole batch of its own,
# pixel seed 1 + r, and checks its first, middle and last image
WEAK_RANKS = 8


def weak_indices(batch: int) -> list:
    return [0, batch // 2, batch - 1]


def vit_bench_fixture(threads: int = 0):
    """Full-depth embeddings of the benchmark's own models (weights seed 0)
    and batches, from the reference's tc_vit_encode, one image per host
    thread at a time: the shard boundaries of the pixel-seed-1 batch split
    over 1/2/4/8 GPUs, and the first, middle and last image of every rank's
    own batch (pixel seeds 1..8)."""
    import tempfile
    import threading
    threads = threads or os.cpu_count() or 1
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, batch, pseed in BENCH_CASES:
            path, cfg = G.cached_vit_gguf(tmp, name, 0)
            idx, widx = bench_indices(batch), weak_indices(batch)
            seeds = list(range(pseed, pseed + WEAK_RANKS))
            jobs = []                                   # (slot, seed, image)
            for j, i in enumerate(idx):
                jobs.append((("strong", j), pseed, i))
            for r, sd in enumerate(seeds):
                for j, i in enumerate(widx):
                    jobs.append((("weak", r, j), sd, i))
            px = {sd: G.make_pixels(batch, cfg["image"], sd) for sd in seeds}
            emb = np.zeros((len(idx), cfg["d_out"]), np.float32)
            wemb = np.zeros((len(seeds), len(widx), cfg["d_out"]), np.float32)
            models = [oracle.RefVit(path) for _ in range(min(threads, len(jobs)))]
            todo = list(jobs)
            lock = threading.Lock()

            def work(m):
                while True:
                    with lock:
                        if not todo:
                            return
                        slot, sd, i = todo.pop()
                    e = m.encode(px[sd][i], cfg["d_out"])["embedding"]
                    if slot[0] == "strong":
                        emb[slot[1]] = e
                    else:
                        wemb[slot[1], slot[2]] = e

            ts = [threading.Thread(target=work, args=(m,)) for m in models]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            for m in models:
                m.close()
            out[f"{name}.index"] = np.array(idx, np.int32)
            out[f"{name}.embedding"] = emb
            out[f"{name}.batch"] = np.array(batch, np.int32)
            out[f"{name}.weak_seeds"] = np.array(seeds, np.int32)
            out[f"{name}.weak_index"] = np.array(widx, np.int32)
            out[f"{name}.weak_embedding"] = wemb
            print(f"{name}: {len(idx)} + {wemb.shape[0] * wemb.shape[1]} images of batches of {batch}", flush=True)
    np.savez_compressed(os.path.join(OUT, "vit_bench_golden.npz"), **out)


# CLIP preprocessing: (height, width, image size, filter); the outputs of
# open_clip's eval transform as torchvision + Pillow compute it.
PRE_CASES = ((37, 53, 24, "bicubic"), (61, 40, 24, "bicubic"), (23, 90, 16, "bicubic"),
             (64, 48, 32, "bilinear"), (24, 24, 24, "bicubic"), (50, 77, 28, "bicubic"))
CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


def torchvision_preprocess(rgb, image, interp):
    """open_clip's eval transform: Resize(image) (shorter side, Pillow),
    CenterCrop(image), ToTensor(), Normalize(mean, std)."""
    from PIL import Image
    from torchvision import transforms as T
    mode = T.InterpolationMode.BICUBIC if interp == "bicubic" else T.InterpolationMode.BILINEAR
    tf = T.Compose([T.Resize(image, interpolation=mode), T.CenterCrop(image), T.ToTensor(),
                    T.Normalize(CLIP_MEAN, CLIP_STD)])
    return np.stack([tf(Image.fromarray(a)).numpy() for a in rgb]).astype(np.float32)


def preprocess_fixture():
    out = {}
    rng = np.random.default_rng(17)
    for i, (h, w, image, interp) in enumerate(PRE_CASES):
        rgb = rng.integers(0, 256, (2, h, w, 3), dtype=np.uint8)
        out[f"case{i}.rgb"] = rgb
        out[f"case{i}.meta"] = np.array([h, w, image, 0 if interp == "bicubic" else 1], np.int32)
        out[f"case{i}.pixels"] = torchvision_preprocess(rgb, image, interp)
    out["mean"] = np.array(CLIP_MEAN, np.float32)
    out["std"] = np.array(CLIP_STD, np.float32)
    np.savez_compressed(os.path.join(OUT, "preprocess_golden.npz"), **out)


if __name__ == "__main__":
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        sys.exit("set TC_REFERENCE to the roofline.c source tree (the directory holding src/ and tests/)")
    oracle.build(with_ref=True, ref_dir=REF)
    only = set(sys.argv[1:])            # e.g. "bench": regenerate that fixture alone
    steps = {"ops": ops_fixture, "kquant": kquant_fixture, "vit": vit_fixture, "bench": vit_bench_fixture,
             "preprocess": preprocess_fixture}
    for key, fn in steps.items():
        if not only or key in only:
            fn()
    print("golden fixtures written to", OUT)

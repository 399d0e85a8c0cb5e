"""CPU restatement of CLIP image preprocessing -- TEST INFRASTRUCTURE ONLY.

The pipeline open_clip applies before roofline.c's tc_vit_encode (which takes
already-normalised pixels, src/vit.h:75-78, and records the normalisation in
clip-vit.preprocess.mean / std, src/vit.c:130-139; the exporter also records
the filter and the resize rule, tools/export_vit_gguf.py:291-294):

  resize the shorter side to `image` with PIL's resampling (the longer side
  to int(image * longer / shorter)), centre crop (offsets rounded half to
  even), uint8 / 255 in float32, minus mean, divided by std.

PIL's resampling, restated from its published algorithm (a third-party
library, Pillow, absent from the reference tree; the checker pins this
restatement against Pillow itself where it is importable): per output index
a window of inputs weighted by filter((x - centre + 0.5) / max(scale, 1))
with support = filter support * max(scale, 1), weights normalised to sum 1
and rounded half away from zero to 22-bit fixed point; a horizontal pass then
a vertical pass, each rounding to 8 bits ((sum + 2^21) >> 22, clamped).
"""
from __future__ import annotations

import math

import numpy as np

PRECISION_BITS = 22


def _bicubic(x):
    a = -0.5
    x = abs(x)
    if x < 1.0:
        return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0
    if x < 2.0:
        return (((x - 5.0) * x + 8.0) * x - 4.0) * a
    return 0.0


def _bilinear(x):
    x = abs(x)
    return 1.0 - x if x < 1.0 else 0.0


def axis_coeffs(in_size: int, out_size: int, interp: str = "bicubic"):
    """(first, count, int coefficients [out_size, ksize]) of one axis."""
    filt, support0 = (_bicubic, 2.0) if interp == "bicubic" else (_bilinear, 1.0)
    scale = in_size / out_size
    fscale = max(scale, 1.0)
    support = support0 * fscale
    ksize = int(math.ceil(support)) * 2 + 1
    first = np.zeros(out_size, np.int64)
    count = np.zeros(out_size, np.int64)
    coef = np.zeros((out_size, ksize), np.int64)
    for o in range(out_size):
        centre = (o + 0.5) * scale
        xmin = max(int(centre - support + 0.5), 0)
        xmax = min(int(centre + support + 0.5), in_size) - xmin
        k = [filt((x + xmin - centre + 0.5) / fscale) for x in range(xmax)]
        ww = sum(k)
        for x in range(xmax):
            w = k[x] / ww if ww != 0.0 else k[x]
            coef[o, x] = int(w * (1 << PRECISION_BITS) + (-0.5 if w < 0 else 0.5))
        first[o], count[o] = xmin, xmax
    return first, count, coef


def _pass(img: np.ndarray, first, count, coef, axis: int) -> np.ndarray:
    """Resample uint8 `img` along `axis` (0 rows, 1 columns) to len(first)."""
    src = np.moveaxis(img.astype(np.int64), axis, 0)
    out = np.empty((len(first),) + src.shape[1:], np.int64)
    for o in range(len(first)):
        acc = np.full(src.shape[1:], 1 << (PRECISION_BITS - 1), np.int64)
        for x in range(int(count[o])):
            acc += src[first[o] + x] * coef[o, x]
        out[o] = np.clip(acc >> PRECISION_BITS, 0, 255)
    return np.moveaxis(out, 0, axis).astype(np.uint8)


def resize_uint8(img: np.ndarray, out_h: int, out_w: int, interp: str = "bicubic") -> np.ndarray:
    """PIL's Image.resize((out_w, out_h)) of an HxWx3 uint8 image."""
    h, w = img.shape[:2]
    t = _pass(img, *axis_coeffs(w, out_w, interp), axis=1)
    return _pass(t, *axis_coeffs(h, out_h, interp), axis=0)


def resized_size(h: int, w: int, image: int):
    shorter, longer = min(h, w), max(h, w)
    new_long = int(image * longer / shorter)
    return (new_long, image) if w <= h else (image, new_long)


def crop_offsets(rh: int, rw: int, image: int):
    return int(round((rh - image) / 2.0)), int(round((rw - image) / 2.0))


def preprocess(rgb: np.ndarray, image: int, mean, std, interp: str = "bicubic") -> np.ndarray:
    """[n, h, w, 3] uint8 -> [n, 3, image, image] float32, open_clip's eval
    transform (Resize(image), CenterCrop(image), ToTensor, Normalize)."""
    n, h, w, _ = rgb.shape
    rh, rw = resized_size(h, w, image)
    top, left = crop_offsets(rh, rw, image)
    mean = np.asarray(mean, np.float32).reshape(3, 1, 1)
    std = np.asarray(std, np.float32).reshape(3, 1, 1)
    out = np.empty((n, 3, image, image), np.float32)
    for i in range(n):
        r = resize_uint8(rgb[i], rh, rw, interp)[top:top + image, left:left + image]
        x = r.transpose(2, 0, 1).astype(np.float32) / np.float32(255.0)
        out[i] = (x - mean) / std
    return out

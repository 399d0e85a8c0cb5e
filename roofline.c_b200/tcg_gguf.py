"""GGUF v3 writer and seeded synthetic inputs for the CLIP ViT and K-quant paths.

The file format is the one roofline.c reads (src/gguf.h:83-95): little-endian
header, metadata key/values, tensor infos with dims fastest-varying first, then
tensor data aligned to `general.alignment` (32). Tensors are passed with their
numpy (C-order) shape and written with the dims reversed, the convention of the
reference's own writer (tools/gguf_writer.py:8-9, :84).

Synthetic models follow the metadata key set of the reference's exporter
(tools/export_vit_gguf.py:279-295) and the tensor names its loader resolves
(src/vit.c:232-257). No network, no checkpoint: every value comes from a seeded
numpy Generator.
"""
from __future__ import annotations

import os
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
ALIGN = 32

# metadata value types (src/gguf.h:110-125)
KV_UINT32, KV_FLOAT32, KV_BOOL, KV_STRING, KV_ARRAY = 4, 6, 7, 8, 9
# ggml tensor types (src/gguf.h:130-152)
F32, F16, Q4_K, Q6_K = 0, 1, 12, 14
QK_K = 256
TYPE_BLOCK = {F32: (1, 4), F16: (1, 2), Q4_K: (256, 144), Q6_K: (256, 210)}


def _s(text: str) -> bytes:
    raw = text.encode()
    return struct.pack("<Q", len(raw)) + raw


def _kv(key, value) -> bytes:
    if isinstance(value, bool):
        return _s(key) + struct.pack("<IB", KV_BOOL, int(value))
    if isinstance(value, int):
        return _s(key) + struct.pack("<II", KV_UINT32, value)
    if isinstance(value, float):
        return _s(key) + struct.pack("<If", KV_FLOAT32, value)
    if isinstance(value, str):
        return _s(key) + struct.pack("<I", KV_STRING) + _s(value)
    if isinstance(value, (list, tuple)) and all(isinstance(v, float) for v in value):
        body = struct.pack("<IIQ", KV_ARRAY, KV_FLOAT32, len(value))
        return _s(key) + body + struct.pack(f"<{len(value)}f", *value)
    raise TypeError(f"unsupported metadata value for {key!r}: {value!r}")


def write_gguf(path: str, kvs: dict, tensors: list) -> int:
    """Write a GGUF v3 file. `tensors` holds (name, array, ggml_type, shape):
    for F32/F16 `array` is the values; for Q4_K/Q6_K it is the raw block bytes
    (uint8) and `shape` the logical [rows, cols]. Returns the file size."""
    infos, blobs, off = [], [], 0
    for name, arr, ty, shape in tensors:
        if ty == F32:
            payload = np.ascontiguousarray(arr, dtype="<f4").tobytes()
        elif ty == F16:
            payload = np.ascontiguousarray(arr, dtype="<f2").tobytes()
        elif ty in (Q4_K, Q6_K):
            payload = np.ascontiguousarray(arr, dtype=np.uint8).tobytes()
        else:
            raise ValueError(f"type {ty} not writable")
        dims = list(shape)[::-1]
        infos.append(_s(name) + struct.pack("<I", len(dims))
                     + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", ty, off))
        blobs.append(payload)
        off += len(payload)
        off += (-off) % ALIGN
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kvs))
    head += b"".join(_kv(k, v) for k, v in kvs.items()) + b"".join(infos)
    head += b"\0" * ((-len(head)) % ALIGN)
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(head)
        for blob in blobs:
            fh.write(blob)
            fh.write(b"\0" * ((-len(blob)) % ALIGN))
    os.replace(tmp, path)
    return len(head) + off


# ----------------------------------------------------------------- ViT models

VIT_CONFIGS = {
    # ViT-B/32: 224/32 -> 49 patches + CLS = 50 tokens
    "vit-b32": dict(n_layer=12, d_model=768, n_head=12, d_ffn=3072, patch=32, image=224, d_out=512),
    # ViT-L/14: 224/14 -> 256 patches + CLS = 257 tokens
    "vit-l14": dict(n_layer=24, d_model=1024, n_head=16, d_ffn=4096, patch=14, image=224, d_out=768),
}


def vit_config(name: str, **override) -> dict:
    cfg = dict(VIT_CONFIGS[name])
    cfg.update(override)
    cfg["n_token"] = (cfg["image"] // cfg["patch"]) ** 2 + 1
    return cfg


def make_vit_weights(cfg: dict, seed: int = 0, std: float = 0.02) -> dict:
    """Random weights in PyTorch layouts: every matrix, bias, embedding and LN
    beta ~ N(0, std); LN gamma = 1 + N(0, std), so activations keep unit scale
    through the stack as in a trained model."""
    rng = np.random.default_rng(seed)
    D, F, P, T = cfg["d_model"], cfg["d_ffn"], cfg["patch"], cfg["n_token"]

    def nrm(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    def gamma(n):
        return np.float32(1.0) + nrm(n)

    w = {
        "v.patch_embd.weight": nrm(D, 3, P, P),
        "v.cls_token": nrm(D),
        "v.pos_embd": nrm(T, D),
        "v.ln_pre.weight": gamma(D), "v.ln_pre.bias": nrm(D),
    }
    for i in range(cfg["n_layer"]):
        p = f"v.blk.{i}."
        w[p + "ln1.weight"] = gamma(D); w[p + "ln1.bias"] = nrm(D)
        w[p + "attn_qkv.weight"] = nrm(3 * D, D); w[p + "attn_qkv.bias"] = nrm(3 * D)
        w[p + "attn_out.weight"] = nrm(D, D); w[p + "attn_out.bias"] = nrm(D)
        w[p + "ln2.weight"] = gamma(D); w[p + "ln2.bias"] = nrm(D)
        w[p + "ffn_up.weight"] = nrm(F, D); w[p + "ffn_up.bias"] = nrm(F)
        w[p + "ffn_down.weight"] = nrm(D, F); w[p + "ffn_down.bias"] = nrm(D)
    w["v.ln_post.weight"] = gamma(D); w["v.ln_post.bias"] = nrm(D)
    w["v.proj"] = nrm(D, cfg["d_out"])
    return w


def vit_metadata(cfg: dict, activation: str = "gelu") -> dict:
    a = "clip-vit"
    return {
        "general.architecture": a,
        "general.name": "synthetic clip-vit",
        f"{a}.block_count": cfg["n_layer"],
        f"{a}.embedding_length": cfg["d_model"],
        f"{a}.attention.head_count": cfg["n_head"],
        f"{a}.feed_forward_length": cfg["d_ffn"],
        f"{a}.patch_size": cfg["patch"],
        f"{a}.image_size": cfg["image"],
        f"{a}.context_length": cfg["n_token"],
        f"{a}.projection_dim": cfg["d_out"],
        f"{a}.layer_norm_epsilon": 1e-5,
        f"{a}.activation": activation,
        f"{a}.pooling": "cls",
        f"{a}.preprocess.mean": [0.48145466, 0.4578275, 0.40821073],
        f"{a}.preprocess.std": [0.26862954, 0.26130258, 0.27577711],
        f"{a}.preprocess.interpolation": "bicubic",
        f"{a}.preprocess.resize_mode": "shortest",
    }


def write_vit_gguf(path: str, cfg: dict, weights: dict, activation: str = "gelu",
                   dtype: int = F32) -> int:
    tensors = [(n, a, dtype, a.shape) for n, a in weights.items()]
    return write_gguf(path, vit_metadata(cfg, activation), tensors)


def make_pixels(n_images: int, image: int, seed: int = 1) -> np.ndarray:
    """[n, 3, image, image] fp32, U[-1, 1): already-normalised inputs."""
    rng = np.random.default_rng(seed)
    return rng.uniform(-1.0, 1.0, size=(n_images, 3, image, image)).astype(np.float32)


def cached_vit_gguf(cache_dir: str, name: str, seed: int = 0, **override) -> tuple:
    """Write (once) the synthetic model for a named config; returns (path, cfg)."""
    cfg = vit_config(name, **override)
    tag = "-".join(f"{k}{v}" for k, v in sorted(override.items()))
    path = os.path.join(cache_dir, f"{name}{('-' + tag) if tag else ''}-s{seed}.gguf")
    if not os.path.exists(path):
        os.makedirs(cache_dir, exist_ok=True)
        write_vit_gguf(path, cfg, make_vit_weights(cfg, seed))
    return path, cfg


# ----------------------------------------------------------- K-quant blocks

def _half_abs_normal(rng, n, std=1e-3):
    return np.abs(rng.normal(0.0, std, size=n)).astype(np.float16)


def make_q4k_blocks(n_blocks: int, seed: int) -> np.ndarray:
    """[n_blocks, 144] uint8: d, dmin = fp16(|N(0, 1e-3)|) (small values land
    in fp16's subnormal range), 12 random scale/min bytes, 128 random nibble
    bytes."""
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(n_blocks, 144), dtype=np.uint8)
    blk[:, 0:2] = _half_abs_normal(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
    blk[:, 2:4] = _half_abs_normal(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
    return blk


def make_q6k_blocks(n_blocks: int, seed: int) -> np.ndarray:
    """[n_blocks, 210] uint8: random ql/qh bytes, random int8 scales,
    d = fp16(|N(0, 1e-3)|)."""
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(n_blocks, 210), dtype=np.uint8)
    blk[:, 208:210] = _half_abs_normal(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
    return blk


def make_kquant(qtype: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Raw blocks of a [rows, cols] matrix, row-major, as one uint8 vector."""
    if cols % QK_K:
        raise ValueError("K-quant rows must be whole superblocks")
    nb = rows * cols // QK_K
    blk = make_q4k_blocks(nb, seed) if qtype == Q4_K else make_q6k_blocks(nb, seed)
    return blk.reshape(-1)


def make_kquant_like(qt: int, rows: int, cols: int, seed: int, d_std: float) -> np.ndarray:
    """Random K-quant blocks of a [rows, cols] matrix whose weights have a
    trained model's scale: the fp16 super-scales d (and dmin) ~ |N(0, d_std)|,
    many of them fp16 subnormals. Flat uint8."""
    nb = rows * cols // 256
    blk = (make_q4k_blocks if qt == Q4_K else make_q6k_blocks)(nb, seed)
    rng = np.random.default_rng(seed + 1)

    def half():
        return np.abs(rng.normal(0.0, d_std, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if qt == Q4_K:
        blk[:, 0:2] = half()
        blk[:, 2:4] = half()
    else:
        blk[:, 208:210] = half()
    return blk.reshape(-1)


def write_kquant_vit_gguf(path: str, cfg: dict, seed: int = 0, qtype: int = Q4_K, d_std: float = 4e-5) -> dict:
    """A ViT GGUF whose block linear weights (qkv, out, up, down) are random
    K-quant blocks at a trained model's scale; every other tensor N(0, 0.02)
    fp32 like make_vit_weights (the 4-D patch embedding too: its innermost
    dimension of `patch` elements is no whole number of 256-weight blocks, so
    a ggml file keeps it unquantised). Returns the fp32 tensors and the
    K-quant ones raw as (blocks, type, shape); dequantising them for a
    reference model is the caller's business (this module computes nothing)."""
    w = make_vit_weights(cfg, seed)
    tensors, raw = [], {}
    for k, (name, arr) in enumerate(w.items()):
        if name.endswith(("attn_qkv.weight", "attn_out.weight", "ffn_up.weight", "ffn_down.weight")):
            rows = arr.shape[0]
            cols = arr.size // rows
            blocks = make_kquant_like(qtype, rows, cols, 1000 + k, d_std)
            tensors.append((name, blocks, qtype, arr.shape))
            raw[name] = (blocks, qtype, arr.shape)
        else:
            tensors.append((name, arr, F32, arr.shape))
    write_gguf(path, vit_metadata(cfg), tensors)
    return {"fp32": w, "kquant": raw}

#!/usr/bin/env python3
"""Per-kernel timing of libtcg's hot kernels (CUDA events on the library
stream), one case per invocation -- the command the ncu summaries in
profiles/ are taken with.

    python roofline.c_b200/kernel_bench.py gemm --M 12800 --N 3072 --K 768 [--cfg C]
    python roofline.c_b200/kernel_bench.py matvec --type q4k --N 4096 --K 14336
    python roofline.c_b200/kernel_bench.py dequant --type q6k --rows 14336 --cols 4096
    python roofline.c_b200/kernel_bench.py vit --model vit-b32 --batch 256 --steps 3

Each case runs `--warmup` untimed launches, then `--reps` timed ones with a
256 MB memset between them (L2 flush), and prints one JSON line.
"""
import argparse
import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402

import tcg  # noqa: E402
import tcg_gguf as G  # noqa: E402

QTYPES = {"q4k": (G.Q4_K, 144), "q6k": (G.Q6_K, 210)}


def timed(fn, warmup, reps, flush=None):
    L = tcg.lib()
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(reps):
        if flush is not None:
            tcg.check(L.tcg_memset(flush.ptr, 0, flush.nbytes))
        ts.append(tcg.time_ms(fn, 2, 3))
    tcg.sync()
    return statistics.median(ts), ts


def case_gemm(a):
    L = tcg.lib()
    rng = np.random.default_rng(0)
    x = rng.standard_normal((a.M, a.K), dtype=np.float32)
    W = (rng.standard_normal((a.N, a.K), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(a.N, dtype=np.float32)
    with tcg.DeviceBuffer.from_array(x) as dx, tcg.DeviceBuffer.from_array(W) as dw, \
            tcg.DeviceBuffer.from_array(b) as db, tcg.DeviceBuffer(a.M * a.N * 4) as dy, \
            tcg.DeviceBuffer(256 << 20) as flush:
        # the op entry point first splits both operands into tf32 hi/lo (two
        # small bandwidth-bound kernels), then runs the GEMM kernel
        run = lambda: tcg.check(L.tcg_linear_cfg(dy.ptr, dx.ptr, dw.ptr, db.ptr, a.M, a.N, a.K, a.cfg))  # noqa
        total, _ = timed(run, a.warmup, a.reps, flush)
    flops = 2.0 * a.M * a.N * a.K
    return {"case": "gemm", "M": a.M, "N": a.N, "K": a.K, "cfg": a.cfg, "ms_split_plus_gemm": round(total, 4),
            "tflops_incl_split": round(flops / total / 1e9, 1)}


def case_matvec(a):
    L = tcg.lib()
    qt, bb = QTYPES[a.type]
    raw = G.make_kquant(qt, a.N, a.K, seed=3)
    x = np.random.default_rng(4).standard_normal(a.K).astype(np.float32)
    with tcg.DeviceBuffer.from_array(raw) as w, tcg.DeviceBuffer.from_array(x) as xb, \
            tcg.DeviceBuffer(a.N * 4) as y, tcg.DeviceBuffer(256 << 20) as flush:
        ms, _ = timed(lambda: tcg.check(L.tcg_matvec_q(y.ptr, w.ptr, xb.ptr, a.N, a.K, qt)), a.warmup, a.reps, flush)
    nbytes = a.N * a.K // 256 * bb + 4 * (a.N + a.K)
    return {"case": "matvec", "type": a.type, "N": a.N, "K": a.K, "ms": round(ms, 5), "bytes": nbytes,
            "GB/s": round(nbytes / ms / 1e6, 1)}


def case_dequant(a):
    L = tcg.lib()
    qt, bb = QTYPES[a.type]
    raw = G.make_kquant(qt, a.rows, a.cols, seed=2)
    n = a.rows * a.cols
    with tcg.DeviceBuffer.from_array(raw) as src, tcg.DeviceBuffer(n * 4) as dst, \
            tcg.DeviceBuffer(256 << 20) as flush:
        ms, _ = timed(lambda: tcg.check(L.tcg_dequant(dst.ptr, src.ptr, n, qt)), a.warmup, a.reps, flush)
    nbytes = n // 256 * bb + 4 * n
    return {"case": "dequant", "type": a.type, "rows": a.rows, "cols": a.cols, "ms": round(ms, 5),
            "bytes": nbytes, "GB/s": round(nbytes / ms / 1e6, 1)}


def case_vit(a):
    L = tcg.lib()
    cache = os.environ.get("TCG_BENCH_CACHE", "/tmp/roofline_b200_bench")
    over = {"n_layer": a.layers} if a.layers else {}
    path, cfg = G.cached_vit_gguf(cache, a.model, 0, **over)
    m = tcg.VitModel(path)
    m.upload(a.batch)
    px = G.make_pixels(a.batch, cfg["image"], 1)
    with tcg.DeviceBuffer.from_array(px) as dpx, tcg.DeviceBuffer(a.batch * cfg["d_out"] * 4) as dout:
        step = lambda: tcg.check(L.tcg_vit_encode_device(m.dev, dpx.ptr, a.batch, dout.ptr))  # noqa: E731
        ms, _ = timed(step, a.warmup, a.steps)
    m.close()
    return {"case": "vit", "model": a.model, "layers": cfg["n_layer"], "batch": a.batch, "ms": round(ms, 4),
            "images/s": round(a.batch / ms * 1e3, 1)}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--M", type=int, default=12800)
    g.add_argument("--N", type=int, default=3072)
    g.add_argument("--K", type=int, default=768)
    g.add_argument("--cfg", type=int, default=-1)
    mv = sub.add_parser("matvec")
    mv.add_argument("--type", choices=sorted(QTYPES), default="q4k")
    mv.add_argument("--N", type=int, default=4096)
    mv.add_argument("--K", type=int, default=14336)
    dq = sub.add_parser("dequant")
    dq.add_argument("--type", choices=sorted(QTYPES), default="q4k")
    dq.add_argument("--rows", type=int, default=14336)
    dq.add_argument("--cols", type=int, default=4096)
    v = sub.add_parser("vit")
    v.add_argument("--model", default="vit-b32", choices=sorted(G.VIT_CONFIGS))
    v.add_argument("--batch", type=int, default=256)
    v.add_argument("--layers", type=int, default=0)
    v.add_argument("--steps", type=int, default=3)
    for p in (g, mv, dq, v):
        p.add_argument("--warmup", type=int, default=3)
        p.add_argument("--reps", type=int, default=5)
        p.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    tcg.init(a.device)
    res = {"gemm": case_gemm, "matvec": case_matvec, "dequant": case_dequant, "vit": case_vit}[a.case](a)
    res["device_error"] = tcg.lib().tcg_device_error()
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

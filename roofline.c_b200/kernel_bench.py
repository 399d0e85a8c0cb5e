#!/usr/bin/env python3
"""Per-kernel timing of libtcg's hot kernels (CUDA events on the library
stream), one case per invocation -- the command the ncu summaries in
profiles/ are taken with.

    python roofline.c_b200/kernel_bench.py gemm --M 12800 --N 3072 --K 768 [--cfg C]
    python roofline.c_b200/kernel_bench.py matvec --type q4k --N 4096 --K 14336
    python roofline.c_b200/kernel_bench.py dequant --type q6k --rows 14336 --cols 4096
    python roofline.c_b200/kernel_bench.py vit --model vit-b32 --batch 256 --steps 3
    python roofline.c_b200/kernel_bench.py attention --T 50 --heads 12 --images 256

Each case runs `--warmup` untimed launches, then `--reps` timed ones with a
256 MB memset between them (L2 flush), and prints one JSON line.
"""
import argparse
import ctypes
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


class SplitOperands:
    """x [M,K] and W [N,K] uploaded once and split into tf32 hi/lo on the
    device, so that a timed launch is the GEMM kernel alone."""

    def __init__(self, M, N, K, seed=0):
        L = tcg.lib()
        rng = np.random.default_rng(seed)
        self.x = rng.standard_normal((M, K), dtype=np.float32)
        self.W = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
        self.b = rng.standard_normal(N, dtype=np.float32)
        self.bufs = [tcg.DeviceBuffer.from_array(a) for a in (self.x, self.W, self.b)]
        self.xh, self.xl = tcg.DeviceBuffer(M * K * 4), tcg.DeviceBuffer(M * K * 4)
        self.wh, self.wl = tcg.DeviceBuffer(N * K * 4), tcg.DeviceBuffer(N * K * 4)
        self.y = tcg.DeviceBuffer(M * N * 4)
        self.bufs += [self.xh, self.xl, self.wh, self.wl, self.y]
        tcg.check(L.tcg_split_tf32(self.xh.ptr, self.xl.ptr, self.bufs[0].ptr, M * K))
        tcg.check(L.tcg_split_tf32(self.wh.ptr, self.wl.ptr, self.bufs[1].ptr, N * K))
        self.M, self.N, self.K = M, N, K

    def run(self, cfg):
        tcg.check(tcg.lib().tcg_linear_split_cfg(self.y.ptr, self.xh.ptr, self.xl.ptr, self.wh.ptr, self.wl.ptr,
                                                 self.bufs[2].ptr, self.M, self.N, self.K, cfg), f"cfg {cfg}")

    def rel_err(self):
        got = self.y.download((self.M, self.N)).astype(np.float64)
        want = self.x.astype(np.float64) @ self.W.astype(np.float64).T + self.b.astype(np.float64)
        return float(np.abs(got - want).max() / np.abs(want).max())

    def close(self):
        for b in self.bufs:
            b.close()


class F16Operands(SplitOperands):
    """x and W also as fp16 pieces with per-(row, 128-element K-block)
    exponents (tcg_split_f16), for the kind::f16 GEMM."""

    def __init__(self, M, N, K, seed=0, blk=128):
        super().__init__(M, N, K, seed)
        L = tcg.lib()
        self.blk = blk
        self.f = [tcg.DeviceBuffer(n) for n in (M * K * 2, M * K * 2, M * K // 128, N * K * 2, N * K * 2, N * K // 128)]
        self.bufs += self.f
        tcg.check(L.tcg_split_f16(self.f[0].ptr, self.f[1].ptr, self.f[2].ptr, self.bufs[0].ptr, M, K,
                                  0 if blk == 128 else 2))
        tcg.check(L.tcg_split_f16(self.f[3].ptr, self.f[4].ptr, self.f[5].ptr, self.bufs[1].ptr, N, K, 1))

    def run(self, cfg):
        f = self.f
        tcg.check(tcg.lib().tcg_linear_f16_split(self.y.ptr, f[0].ptr, f[1].ptr, f[2].ptr, f[3].ptr, f[4].ptr,
                                                 f[5].ptr, self.bufs[2].ptr, self.M, self.N, self.K, self.blk),
                  "f16 GEMM")


def case_gemm(a):
    old_sk = tcg.lib().tcg_gemm_set_streamk(a.streamk)
    old_tma = tcg.lib().tcg_gemm_set_tma_store(a.tma_store)
    old_f16 = tcg.lib().tcg_gemm_set_f16_cfg(a.f16_cfg)
    ops = F16Operands(a.M, a.N, a.K, blk=a.f16) if a.f16 else SplitOperands(a.M, a.N, a.K)
    with tcg.DeviceBuffer(256 << 20) as flush:
        ms, _ = timed(lambda: ops.run(a.cfg), a.warmup, a.reps, flush)
    err = ops.rel_err()
    plan = (ctypes.c_int * 4)()
    tcg.lib().tcg_gemm_last_plan(plan)
    ops.close()
    tcg.lib().tcg_gemm_set_streamk(old_sk)
    tcg.lib().tcg_gemm_set_tma_store(old_tma)
    tcg.lib().tcg_gemm_set_f16_cfg(old_f16)
    flops = 2.0 * a.M * a.N * a.K
    return {"case": "gemm", "M": a.M, "N": a.N, "K": a.K, "cfg": a.cfg, "f16": a.f16, "f16_cfg": a.f16_cfg,
            "rel_err": err,
            "streamk": a.streamk, "ms": round(ms, 4),
            "tflops": round(flops / ms / 1e9, 1), "grid": plan[0], "split": plan[1], "tma_store": plan[3]}


def case_gemmsweep(a):
    """Every tile configuration x TMEM chunk length on the four ViT-B/32
    GEMM shapes at batch 256; accuracy against a float64 product at M=256."""
    L = tcg.lib()
    shapes = {"qkv": (12800, 2304, 768), "out": (12800, 768, 768), "up": (12800, 3072, 768),
              "down": (12800, 768, 3072)}
    chunks = [int(c) for c in a.chunks.split(",")]
    cfgs = range(L.tcg_gemm_num_cfgs()) if a.cfgs == "all" else [int(c) for c in a.cfgs.split(",")]
    res = {"perf_ms": {}, "rel_err": {}}
    default_chunk = L.tcg_gemm_set_chunk_k(0)         # an invalid length only reads the current one
    flush = tcg.DeviceBuffer(256 << 20)
    for name, (M, N, K) in shapes.items():
        ops = SplitOperands(M, N, K)
        for ck in chunks:
            L.tcg_gemm_set_chunk_k(ck)
            for cfg in list(cfgs) + [-1]:
                ms, _ = timed(lambda: ops.run(cfg), a.warmup, a.reps, flush)
                res["perf_ms"][f"{name}/chunk{ck}/cfg{cfg}"] = round(ms, 4)
        ops.close()
    for K in (768, 3072):
        ops = SplitOperands(256, 768, K, seed=1)
        for ck in chunks:
            L.tcg_gemm_set_chunk_k(ck)
            for cfg in list(cfgs) + [-1]:
                ops.run(cfg)
                res["rel_err"][f"K{K}/chunk{ck}/cfg{cfg}"] = ops.rel_err()
        ops.close()
    L.tcg_gemm_set_chunk_k(default_chunk)
    flush.close()
    return {"case": "gemmsweep", **res}


def case_matvec(a):
    L = tcg.lib()
    qt, bb = QTYPES[a.type]
    raw = G.make_kquant(qt, a.N, a.K, seed=3)
    x = np.random.default_rng(4).standard_normal(a.K).astype(np.float32)
    old_tc, old_mma = L.tcg_matvec_set_tc(a.tc), L.tcg_matvec_set_mma(a.mma)
    old_segs = L.tcg_matvec_mma_segments(a.segs)
    old_static = L.tcg_matvec_set_static_weights(a.static_weights)
    old_split = L.tcg_matvec_mma_split(a.split)
    old_tiles = L.tcg_matvec_mma_tiles(a.tiles)
    old_direct = L.tcg_matvec_mma_direct(a.direct)
    old_slots = L.tcg_matvec_mma_slots(a.slots)
    # back to back: the matrix rotates over enough copies that each launch
    # reads from HBM, not L2 (as in a decode pass over successive layers)
    copies = max(1, min(10, -(-(300 << 20) // raw.nbytes)))
    ws = [tcg.DeviceBuffer.from_array(raw) for _ in range(copies)]
    with tcg.DeviceBuffer.from_array(x) as xb, tcg.DeviceBuffer(a.N * 4) as y, \
            tcg.DeviceBuffer(256 << 20) as flush:
        mv = [lambda w=w: tcg.check(L.tcg_matvec_q(y.ptr, w.ptr, xb.ptr, a.N, a.K, qt)) for w in ws]
        ms, _ = timed(mv[0], a.warmup, a.reps, flush)
        launches = max(10, copies)
        seq = lambda: [mv[i % copies]() for i in range(launches)]
        for _ in range(a.warmup):
            seq()
        ts = []
        for _ in range(a.reps):
            if a.delay:
                tcg.check(L.tcg_device_delay_us(a.delay))
            ts.append(tcg.time_ms(seq, 2, 3))
        b2b = statistics.median(ts) / launches
        rd = lambda: [tcg.check(L.tcg_read_ceiling(ws[i % copies].ptr, raw.nbytes)) for i in range(launches)]
        ts = []
        for _ in range(a.reps):
            if a.delay:
                tcg.check(L.tcg_device_delay_us(a.delay))
            ts.append(tcg.time_ms(rd, 2, 3))
        read_b2b = statistics.median(ts) / launches
    for w in ws:
        w.close()
    kern = L.tcg_matvec_last_kernel()
    L.tcg_matvec_set_tc(old_tc)
    L.tcg_matvec_set_mma(old_mma)
    L.tcg_matvec_mma_segments(old_segs)
    L.tcg_matvec_set_static_weights(old_static)
    L.tcg_matvec_mma_split(old_split)
    L.tcg_matvec_mma_tiles(old_tiles)
    L.tcg_matvec_mma_direct(old_direct)
    L.tcg_matvec_mma_slots(old_slots)
    nbytes = a.N * a.K // 256 * bb + 4 * (a.N + a.K)
    return {"case": "matvec", "type": a.type, "N": a.N, "K": a.K, "kernel": kern, "ms": round(ms, 5),
            "bytes": nbytes, "GB/s": round(nbytes / ms / 1e6, 1), "b2b_ms": round(b2b, 5),
            "b2b_GB/s": round(nbytes / b2b / 1e6, 1), "read_b2b_ms": round(read_b2b, 5), "copies": copies,
            "static_weights": a.static_weights, "delay_us": a.delay}


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
    if a.q4k:       # block linears as Q4_K blocks, kept packed on the device
        path = os.path.join(cache, f"{a.model}-L{cfg['n_layer']}-q4k-s0.gguf")
        if not os.path.exists(path):
            G.write_kquant_vit_gguf(path + ".tmp", cfg, seed=0)
            os.replace(path + ".tmp", path)
    old_jit = L.tcg_vit_set_jit_rows(a.jit_rows) if a.jit_rows else None
    old_f16 = L.tcg_gemm_set_f16_cfg(a.f16_cfg)
    # the GEMM plans of a batch size are made at its first forward
    old_cfg, old_sk = L.tcg_gemm_force_cfg(a.cfg), L.tcg_gemm_set_streamk(a.streamk)
    old_pdl = L.tcg_set_pdl(a.pdl)
    old_tma = L.tcg_gemm_set_tma_store(a.tma_store)
    old_chunk = L.tcg_gemm_set_chunk_k(a.chunk) if a.chunk else None
    m = tcg.VitModel(path)
    m.upload(a.batch)
    px = G.make_pixels(a.batch, cfg["image"], 1)
    with tcg.DeviceBuffer.from_array(px) as dpx, tcg.DeviceBuffer(a.batch * cfg["d_out"] * 4) as dout:
        step = lambda: tcg.check(L.tcg_vit_encode_device(m.dev, dpx.ptr, a.batch, dout.ptr))  # noqa: E731
        ms, _ = timed(step, a.warmup, a.steps)
    m.close()
    L.tcg_gemm_force_cfg(old_cfg)
    L.tcg_gemm_set_streamk(old_sk)
    L.tcg_set_pdl(old_pdl)
    L.tcg_gemm_set_tma_store(old_tma)
    if old_chunk is not None:
        L.tcg_gemm_set_chunk_k(old_chunk)
    if old_jit is not None:
        L.tcg_vit_set_jit_rows(old_jit)
    L.tcg_gemm_set_f16_cfg(old_f16)
    return {"case": "vit", "f16_cfg": a.f16_cfg, "chunk": a.chunk, "q4k": a.q4k, "jit_rows": a.jit_rows, "model": a.model, "layers": cfg["n_layer"], "batch": a.batch, "cfg": a.cfg,
            "streamk": a.streamk, "pdl": a.pdl, "tma_store": a.tma_store, "ms": round(ms, 4),
            "images/s": round(a.batch / ms * 1e3, 1)}


def case_attention(a):
    """Attention over --images images of --T tokens: q, k, v in one fused
    row of width 3D (the ViT encoder's layout), output as the tf32 hi/lo pair
    the next GEMM reads (--plain 1: fp32)."""
    L = tcg.lib()
    D = a.heads * 64
    rng = np.random.default_rng(0)
    qkv = rng.standard_normal((a.images * a.T, 3 * D), dtype=np.float32)
    old = L.tcg_set_attention_short_kernel(a.kernel)
    rows = a.images * a.T
    with tcg.DeviceBuffer.from_array(qkv) as dq, tcg.DeviceBuffer(rows * D * 4) as o1, \
            tcg.DeviceBuffer(rows * D * 4) as o2, tcg.DeviceBuffer(256 << 20) as flush:
        if a.plain:
            fn = lambda: tcg.check(L.tcg_mha_images(o1.ptr, None, None, dq.ptr, a.T, a.heads, 64, a.images))  # noqa: E731
        else:
            fn = lambda: tcg.check(L.tcg_mha_images(None, o1.ptr, o2.ptr, dq.ptr, a.T, a.heads, 64, a.images))  # noqa: E731
        ms, _ = timed(fn, a.warmup, a.reps, flush)
    L.tcg_set_attention_short_kernel(old)
    nbytes = rows * D * 4 * (3 + (1 if a.plain else 2))
    return {"case": "attention", "T": a.T, "heads": a.heads, "images": a.images, "kernel": a.kernel,
            "plain": a.plain, "ms": round(ms, 5), "GB/s": round(nbytes / ms / 1e6, 1)}


def case_upload(a):
    """Weight upload from the GGUF mapping in every mode (0 per tensor from
    the mapping, 1 staged through page-locked chunks, 2 mapping registered):
    tc_vit_load time, host-to-device time and GB/s of the weight bytes."""
    import time
    L = tcg.lib()
    cache = os.environ.get("TCG_BENCH_CACHE", "/tmp/roofline_b200_bench")
    path, cfg = G.cached_vit_gguf(cache, a.model, 0)
    res = {"case": "upload", "model": a.model, "bytes": None, "modes": {}}
    old = L.tcg_vit_set_upload_mode(1)
    for rep in range(a.reps):
        for mode in (0, 1, 2):
            L.tcg_vit_set_upload_mode(mode)
            t0 = time.perf_counter()
            m = tcg.VitModel(path)
            t1 = time.perf_counter()
            m.upload(1)
            t2 = time.perf_counter()
            up = L.tcg_vit_last_upload_ms()
            fb = (L.tcg_vit_upload_fallback() or b"").decode()
            m.close()
            wb = os.path.getsize(path)
            res["bytes"] = wb
            r = res["modes"].setdefault(str(mode), [])
            r.append({"load_ms": round((t1 - t0) * 1e3, 2), "h2d_ms": round(up, 2),
                      "upload_total_ms": round((t2 - t1) * 1e3, 2), "h2d_GB/s": round(wb / up / 1e6, 2),
                      **({"fell_back": fb} if fb else {})})
    L.tcg_vit_set_upload_mode(old)
    return res


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--M", type=int, default=12800)
    g.add_argument("--N", type=int, default=3072)
    g.add_argument("--K", type=int, default=768)
    g.add_argument("--cfg", type=int, default=-1)
    g.add_argument("--streamk", type=int, default=1)
    g.add_argument("--tma-store", type=int, default=1)
    g.add_argument("--f16-cfg", type=int, default=16, help="fp16-piece GEMM configuration: 16 or 17")
    g.add_argument("--f16", type=int, default=0,
                   help="128 or 256: fp16-piece operands on kind::f16 MMAs, A scaled per K-block of that size")
    gs = sub.add_parser("gemmsweep")
    gs.add_argument("--chunks", default="32,64,128,256,4096")
    gs.add_argument("--cfgs", default="all")
    mv = sub.add_parser("matvec")
    mv.add_argument("--type", choices=sorted(QTYPES), default="q4k")
    mv.add_argument("--N", type=int, default=4096)
    mv.add_argument("--K", type=int, default=14336)
    mv.add_argument("--tc", type=int, default=0, help="1: Q4_K on the tensor cores (opt-in kernel)")
    mv.add_argument("--mma", type=int, default=1, help="0: Q4_K on the CUDA-core kernels")
    mv.add_argument("--segs", type=int, default=0, help="K segments per tile of the mma kernel (0: automatic)")
    mv.add_argument("--split", type=int, default=1, help="warps per unit of the mma kernel: 1 by shape, 0 one, 2, 4")
    mv.add_argument("--tiles", type=int, default=-1,
                    help="mma kernel: 1 whole tiles per CTA, 0 segment-major unit ranges, -1 by shape")
    mv.add_argument("--slots", type=int, default=0, help="most unit slots per CTA of the mma kernel (0: all that fit)")
    mv.add_argument("--direct", type=int, default=1, help="0: refill slots instead of direct units (Q4_K mma)")
    mv.add_argument("--delay", type=int, default=500,
                    help="us of device delay queued before each back-to-back sequence (0: none)")
    mv.add_argument("--static-weights", type=int, default=0,
                    help="1: promise that no earlier kernel writes W (weights fetched before the previous ends)")
    dq = sub.add_parser("dequant")
    dq.add_argument("--type", choices=sorted(QTYPES), default="q4k")
    dq.add_argument("--rows", type=int, default=14336)
    dq.add_argument("--cols", type=int, default=4096)
    v = sub.add_parser("vit")
    v.add_argument("--model", default="vit-b32", choices=sorted(G.VIT_CONFIGS))
    v.add_argument("--batch", type=int, default=256)
    v.add_argument("--layers", type=int, default=0)
    v.add_argument("--steps", type=int, default=3)
    v.add_argument("--cfg", type=int, default=-1, help="GEMM configuration for every linear (-1: automatic)")
    v.add_argument("--streamk", type=int, default=1, help="0: every GEMM tile computed whole")
    v.add_argument("--pdl", type=int, default=1, help="0: no programmatic dependent launch")
    v.add_argument("--tma-store", type=int, default=1, help="0: GEMM epilogues on plain stores")
    v.add_argument("--chunk", type=int, default=0, help="K-elements per TMEM accumulator chunk (0: default)")
    v.add_argument("--f16-cfg", type=int, default=16, help="fp16-piece GEMM configuration: 16 or 17")
    v.add_argument("--q4k", type=int, default=0, help="1: the model with Q4_K block linears (kept packed)")
    v.add_argument("--jit-rows", type=int, default=0,
                   help="token rows from which packed weights are dequantised before their GEMMs (0: default)")
    at = sub.add_parser("attention")
    at.add_argument("--T", type=int, default=50)
    at.add_argument("--heads", type=int, default=12)
    at.add_argument("--images", type=int, default=256)
    at.add_argument("--kernel", type=int, default=1, help="T <= 64: 1 fp16-split tensor cores, 0 fp32 FMA")
    at.add_argument("--plain", type=int, default=0, help="1: fp32 output instead of the tf32 pair")
    up = sub.add_parser("upload")
    up.add_argument("--model", default="vit-b32", choices=sorted(G.VIT_CONFIGS))
    for p in (g, gs, mv, dq, v, at, up):
        p.add_argument("--warmup", type=int, default=3)
        p.add_argument("--reps", type=int, default=5)
        p.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    tcg.init(a.device)
    res = {"gemm": case_gemm, "gemmsweep": case_gemmsweep, "matvec": case_matvec, "dequant": case_dequant,
           "vit": case_vit, "attention": case_attention, "upload": case_upload}[a.case](a)
    res["device_error"] = tcg.lib().tcg_device_error()
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

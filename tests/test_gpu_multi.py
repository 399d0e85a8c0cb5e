"""Two GPUs, one process each: the one-time NCCL weight broadcast
(tcg_vit_upload_bcast) and the image-sharded forward.

* every rank runs its shard through a model whose weights came from rank 0
  over NCCL; the embeddings equal, bit for bit, those of a copy uploaded from
  the file on the same GPU (same kernels, same K order);
* a rank that leaves before the broadcast (between steps, none of its kernels
  or collectives in flight) makes rank 0's tcg_vit_upload_bcast return an
  error within the TCG_NCCL_TIMEOUT bound instead of hanging in NCCL's init.

NVLS is off (NCCL_NVLS_ENABLE=0). Skipped when fewer than two devices are
visible."""
import os
import socket
import sys
import time

import pytest
import torch.multiprocessing as mp

import tcg
import tcg_gguf as G

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NCCL_TIMEOUT = 20


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, path, image, q, leave_rank):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "roofline.c_b200")]
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), TCG_PG_TIMEOUT="90",
                      TCG_NCCL_TIMEOUT=str(NCCL_TIMEOUT), NCCL_NVLS_ENABLE="0")
    try:
        import ctypes

        import numpy as np

        import bench
        import tcg
        import tcg_gguf as G
        d = bench.Dist(world)
        tcg.init(rank)
        L = tcg.lib()
        uid = None
        if rank == 0:
            buf = ctypes.create_string_buffer(128)
            tcg.check(L.tcg_nccl_unique_id(buf), "tcg_nccl_unique_id")
            uid = buf.raw
        uid = d.bcast_bytes(uid)
        if rank == leave_rank:
            q.put((rank, "left", None))
            return
        m = tcg.VitModel(path)
        t0 = time.time()
        try:
            m.upload_bcast(4, rank, world, uid)
        except tcg.TcgError as e:
            q.put((rank, "bcast_error", (str(e), time.time() - t0)))
            return
        px = G.make_pixels(8, image, 5)
        lo, hi = bench.shard_range(8, world, rank)
        got, _ = m.encode(px[lo:hi])
        local = tcg.VitModel(path)
        local.upload(4)
        want, _ = local.encode(px[lo:hi])
        same = bool(np.array_equal(got, want))
        dev_err = int(L.tcg_device_error())
        m.close()
        local.close()
        d.barrier()
        d.close()
        q.put((rank, "ok", (same, got.shape, dev_err)))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))


def _run(path, image, leave_rank=-1, timeout=240):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, path, image, q, leave_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, status, info = q.get(timeout=timeout)
            out[r] = (status, info)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
                p.join()
    return out


@pytest.fixture()
def two_gpus(gpu):
    if tcg.lib().tcg_device_count() < 2:
        pytest.skip("needs two visible devices")


def test_broadcast_weights_and_sharded_forward(two_gpus, cache_dir):
    path, cfg = G.cached_vit_gguf(cache_dir, "vit-b32", 0, n_layer=2)
    out = _run(path, cfg["image"])
    for r in range(2):
        status, info = out[r]
        assert status == "ok", (r, status, info)
        same, shape, dev_err = info
        assert same, f"rank {r}: broadcast weights give different embeddings"
        assert shape == (4, cfg["d_out"]) and dev_err == 0


def test_rank_that_never_joins_ends_in_an_error(two_gpus, cache_dir):
    path, cfg = G.cached_vit_gguf(cache_dir, "vit-b32", 0, n_layer=1)
    out = _run(path, cfg["image"], leave_rank=1)
    assert out[1][0] == "left"
    status, info = out[0]
    assert status == "bcast_error", (status, info)
    msg, secs = info
    assert "did not answer" in msg
    assert secs < NCCL_TIMEOUT + 30

"""The N>1 host logic of the benchmark on CPU: two gloo ranks exercise the
coordination the GPU run relies on (barrier, max over ranks, handing rank
0's NCCL id to the others) and the image sharding (contiguous, disjoint,
covering the batch, identical shapes on every rank). A rank that fails
before the collective is reported, not hung on: the process group has a
short timeout and the parent joins with a bound."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q, fail_rank):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "roofline.c_b200")]
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), TCG_PG_TIMEOUT="15")
    try:
        import bench
        if rank == fail_rank:
            raise RuntimeError("injected failure before joining")
        d = bench.Dist(world)
        d.barrier()
        got_max = d.max(float(rank * 10 + 1))
        uid = d.bcast_bytes(bytes(range(128)) if rank == 0 else None)
        lo, hi = bench.shard_range(256, world, rank)
        d.close()
        q.put((rank, "ok", got_max, uid == bytes(range(128)), lo, hi))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e), None, None, None))


def _run(world, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world):
        try:
            out.append(q.get(timeout=timeout))
        except Exception:
            break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_two_gloo_ranks_coordinate_and_shard():
    res = _run(2)
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] == 11.0 for r in res)           # max over ranks
    assert all(r[3] for r in res)                   # rank 0's id reached rank 1
    assert [(r[4], r[5]) for r in res] == [(0, 128), (128, 256)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_the_batch(world):
    sys.path[:0] = [ROOT]
    import bench
    ranges = [bench.shard_range(256, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == 256
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    assert len({hi - lo for lo, hi in ranges}) == 1
    with pytest.raises(ValueError):
        bench.shard_range(256, 3, 0)


def test_failed_rank_is_reported_not_hung():
    res = _run(2, fail_rank=1, timeout=30)
    by_rank = {r[0]: r for r in res}
    assert by_rank[1][1] == "error" and "injected" in by_rank[1][2]
    # rank 0 either times out of the rendezvous with an error or is killed by
    # the bounded join; it never reports a successful collective
    assert 0 not in by_rank or by_rank[0][1] == "error"

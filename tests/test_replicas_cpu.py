"""CPU: the multi-GPU host logic of config 5 (partition of the job's
sequences over ranks, waves per rank, max-over-ranks timing) on world-size-2
``gloo`` process groups — no GPU involved."""

from __future__ import annotations

import os

import pytest
import torch.multiprocessing as mp

from transformer_b200.replicas import all_ranks, max_over_ranks, shard


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_the_job(world):
    seen = []
    for r in range(world):
        s = shard(2048, world, r, 256)
        assert s.n == 2048 // world and s.n_waves * s.wave == s.n and s.wave <= 256
        for i in range(s.n_waves):
            b0, b1 = s.wave_slice(i)
            assert s.begin <= b0 < b1 <= s.end
            seen.extend(range(b0, b1))
    assert sorted(seen) == list(range(2048))  # every sequence exactly once


def test_shard_rejects_uneven_splits():
    with pytest.raises(ValueError):
        shard(2048, 3, 0)
    with pytest.raises(ValueError):
        shard(2048, 2, 2)
    with pytest.raises(ValueError):
        shard(257, 1, 0, 256)  # 257 does not split into 2 equal waves


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = shard(2048, world, rank, 256)
        # per-rank "elapsed" values; every rank must see the slowest
        got = max_over_ranks(10.0 + rank * 5.0)
        tokens = max_over_ranks(float(s.n))  # equal shares: the max equals any rank's share
        every = all_ranks(10.0 + rank * 5.0)  # per-rank step times, reported in rank order
        out.put((rank, got, tokens, s.begin, s.end, every))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [r[1] for r in res] == [15.0, 15.0]
    assert [r[2] for r in res] == [1024.0, 1024.0]
    assert res[0][3:5] == (0, 1024) and res[1][3:5] == (1024, 2048)
    assert [r[5] for r in res] == [[10.0, 15.0], [10.0, 15.0]]


def test_max_over_ranks_without_group():
    assert max_over_ranks(3.5) == 3.5
    assert all_ranks(3.5) == [3.5]


def _dying_worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # a worker that dies between steps (host fault), without joining the collective
    try:
        max_over_ranks(1.0)
        out.put((rank, "completed"))
    except Exception as e:  # the survivor learns of it through the collective's error
        out.put((rank, type(e).__name__))


def test_dead_rank_is_reported_not_hung():
    """A rank that exits between steps: the surviving rank's next timing
    reduction fails with an error within the process-group timeout instead of
    waiting for ever."""
    import time
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 90
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[1].exitcode == 3
    rank, what = q.get(timeout=10)
    assert rank == 0 and what != "completed"
    assert time.time() - t0 < 120

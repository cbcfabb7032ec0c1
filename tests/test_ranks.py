"""The multi-GPU plumbing (one process per GPU, no data-path collective) on
CPU: two gloo ranks run the same rank logic bench.py runs over NCCL."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from rembed_b200 import ranks


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    info = ranks.RankInfo(rank, world, rank)
    dist = ranks.init(info, "gloo", timeout_s=60)
    try:
        ranks.barrier(dist)
        # each rank reports its own "device time"; the job's time is the max
        t = ranks.max_over_ranks(dist, 10.0 + rank)
        lo, hi = ranks.shard(7, rank, world)
        q.put((rank, t, ranks.batch_seed(rank), lo, hi))
    finally:
        ranks.finish(dist)


def test_two_gloo_ranks_max_and_shards():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(world))
    assert [g[1] for g in got] == [11.0, 11.0]       # max over ranks, seen by every rank
    assert got[0][2] != got[1][2]                      # distinct batches per rank (weak scaling)
    assert (got[0][3], got[0][4], got[1][3], got[1][4]) == (0, 4, 4, 7)


def test_single_process_needs_no_group():
    info = ranks.rank_info({})
    assert (info.rank, info.world, info.local_rank) == (0, 1, 0)
    assert ranks.init(info, "gloo") is None
    assert ranks.max_over_ranks(None, 3.5) == 3.5


def test_shard_covers_everything_once():
    for n in (0, 1, 5, 8, 13):
        for w in (1, 2, 3, 8):
            parts = [ranks.shard(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    with pytest.raises(ValueError):
        ranks.shard(4, 2, 2)

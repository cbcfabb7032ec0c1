"""Data-parallel rank plumbing for multi-GPU runs (one process per GPU).

Texts are independent (rembed.go:309-331), so ranks share nothing on the
data path: each rank embeds its own shard with its own model replica. The
only collectives are the timing ones: a barrier around the timed region and
the max over ranks of each rank's device time. The backend is "nccl" on
GPUs and "gloo" where the same logic runs on CPU processes (the tests).
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info(env=os.environ) -> RankInfo:
    """RANK / WORLD_SIZE / LOCAL_RANK as torchrun sets them (1 process: 0/1/0)."""
    return RankInfo(int(env.get("RANK", "0")), int(env.get("WORLD_SIZE", "1")), int(env.get("LOCAL_RANK", "0")))


def batch_seed(rank: int, base: int = 1000) -> int:
    """Seed of a rank's synthetic batch: distinct per rank (weak scaling:
    every rank embeds a different batch of the same shape)."""
    return base + rank


def shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous near-equal [lo, hi) share of n items for rank (for callers
    that split one global batch instead of generating one per rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    q, r = divmod(n, world)
    lo = rank * q + min(rank, r)
    return lo, lo + q + (1 if rank < r else 0)


def init(info: RankInfo, backend: str, timeout_s: float = 300.0, device=None):
    """Join the process group (a short timeout so that a rank that died ends
    the others' next collective with an error); None when world == 1."""
    if info.world <= 1:
        return None
    import torch.distributed as dist

    kw = {"device_id": device} if device is not None else {}
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), rank=info.rank,
                            world_size=info.world, **kw)
    return dist


def barrier(dist) -> None:
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, x: float, device="cpu") -> float:
    """The slowest rank's value (timings are reported as the max over ranks)."""
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finish(dist) -> None:
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()

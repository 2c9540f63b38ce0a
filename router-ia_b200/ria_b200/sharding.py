"""Sequence sharding across GPUs of one node (one process per GPU).

The attention path has no cross-sequence dependency: each rank owns a
subset of the requests (a contiguous slice, or a cost-balanced assignment
when request lengths differ), holds a replica of the weights and its own
DeltaNet / conv / KV state, and decodes with no collective on the data path.
The helpers here cover the host-side plumbing around that: which requests a
rank owns, and gathering small per-rank results after the work (over
``torch.distributed``: NCCL on GPUs, gloo in the CPU tests).  A rank that dies
or never arrives surfaces on the others as an error of the gather, bounded by
the process group's timeout.
"""

from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def shard_range(n: int, world: int, rank: int) -> Shard:
    """Contiguous, balanced slice of ``n`` requests for ``rank`` of ``world``:
    the first ``n % world`` ranks get one extra request."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n < 0:
        raise ValueError("n must be non-negative")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return Shard(rank, world, start, stop)


def balanced_assignment(costs: list[int], world: int, per_rank: int | None = None) -> list[list[int]]:
    """Request indices for each rank so that the ranks' summed costs (e.g. KV
    lengths, which set a decode step's time) are near equal while every rank
    gets the same number of requests (``per_rank``, default len/world).

    Longest-first greedy: requests in decreasing cost go to the least-loaded
    rank that still has room.  Deterministic (ties by rank, then index), so
    every rank computes the same assignment from the same list without
    communication.  Each rank's indices are returned in increasing order."""
    n = len(costs)
    if world < 1:
        raise ValueError(f"bad world {world}")
    if per_rank is None:
        if n % world:
            raise ValueError(f"{n} requests do not split evenly over {world} ranks")
        per_rank = n // world
    if per_rank * world < n:
        raise ValueError(f"{n} requests exceed {world} ranks x {per_rank}")
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(n), key=lambda k: (-costs[k], k)):
        r = min((r for r in range(world) if len(out[r]) < per_rank), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += costs[i]
    return [sorted(x) for x in out]


def env_rank_world() -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment (1 process if unset)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def gather_to_rank0(obj, world: int):
    """All ranks' ``obj`` (small, picklable) in rank order, on every rank.
    Raises if a peer fails or times out (process-group timeout)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj)
    return out

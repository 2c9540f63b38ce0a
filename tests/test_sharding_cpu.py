"""Host-side sequence sharding with world_size 2 on CPU (gloo): balanced
contiguous shards, per-rank results gathered after the work, and a rank that
fails surfacing on its peer as an error within the process-group timeout."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import pytest

from ria_b200.sharding import balanced_assignment, gather_to_rank0, shard_range


def test_shard_range_balanced_and_complete():
    for n in (0, 1, 7, 256, 513):
        for world in (1, 2, 3, 8):
            shards = [shard_range(n, world, r) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
            sizes = [s.size for s in shards]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        import torch
        import torch.distributed as dist

        from ria_b200.sharding import gather_to_rank0, shard_range

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        shard = shard_range(10, world, rank)
        # per-rank "decode": a deterministic function of the owned requests
        local = [i * i for i in range(shard.start, shard.stop)]
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the gather")
        results = gather_to_rank0({"rank": rank, "out": local}, world)
        q.put((rank, "ok", [r["out"] for r in results]))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-400:]}"))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, status, payload = q.get(timeout=120)
        res[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_two_ranks_gather_sharded_results():
    res = _run("ok")
    expect = [[i * i for i in range(0, 5)], [i * i for i in range(5, 10)]]
    assert res[0] == ("ok", expect) and res[1] == ("ok", expect)


def test_failed_rank_surfaces_as_error_on_peer():
    res = _run("fail")
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # the gather on rank 0 fails instead of hanging


def test_balanced_assignment_equal_counts_and_loads():
    import random

    rng = random.Random(0)
    for world in (1, 2, 4, 8):
        costs = [rng.randint(512, 32768) for _ in range(world * 256)]
        parts = balanced_assignment(costs, world)
        assert sorted(i for p in parts for i in p) == list(range(len(costs)))  # a partition
        assert all(len(p) == 256 for p in parts)
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= 32768  # within one request of each other
        assert parts == balanced_assignment(costs, world)  # deterministic


def test_balanced_assignment_rejects_uneven_split():
    with pytest.raises(ValueError):
        balanced_assignment([1, 2, 3], 2)


def test_benchmark_workload_splits():
    """bench.py's configuration-3 request lists: weak scaling gives every rank
    the same multiset of 256 KV lengths; strong scaling splits the one-GPU
    job of 256 sequences into disjoint, equal-count shards whose summed KV
    lengths are within one request's length of each other."""
    import argparse

    import bench
    from ria_b200 import synthetic

    args = argparse.Namespace(batch=256, len_lo=512, len_hi=32768)
    job = synthetic.stratified_lengths(256, 512, 32768, seed=0)
    for world in (1, 2, 4, 8):
        weak = [bench.weak_lengths(args, r, world) for r in range(world)]
        assert all(sorted(w) == sorted(job) for w in weak)
        strong = [bench.strong_lengths(args, r, world) for r in range(world)]
        assert all(len(s) == 256 // world for s in strong)
        assert sorted(x for s in strong for x in s) == sorted(job)
        sums = [sum(s) for s in strong]
        assert max(sums) - min(sums) <= max(job)

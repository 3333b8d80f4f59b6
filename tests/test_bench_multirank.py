"""Host logic of the multi-GPU path on CPU: two gloo ranks run the stream
sharding and the max-over-ranks timing that bench.py uses under torchrun
(one process per GPU, streams sharded, no data-path collective)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "voxtral.cpp_b200"))

from vxk_shard import assign_streams, gather_over_ranks, max_over_ranks  # noqa: E402


def test_assignment_is_a_balanced_partition():
    rng = np.random.default_rng(7)
    for world in (1, 2, 4, 8):
        ctx = rng.integers(400, 4097, size=64 * world)
        parts = assign_streams(ctx, world, 64)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64 * world))
        assert all(len(p) == 64 for p in parts)
        loads = [int(ctx[p].sum()) for p in parts]
        # LPT with equal counts: every rank within one longest context of the mean
        assert max(loads) - min(loads) <= int(ctx.max())


def test_assignment_rejects_overfull_ranks():
    with pytest.raises(ValueError):
        assign_streams([1, 2, 3], 1, 2)
    with pytest.raises(ValueError):
        assign_streams([1], 0)


def test_max_over_ranks_without_a_group():
    assert max_over_ranks(None, 3.5) == 3.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(20261201)  # every rank draws the job's contexts identically
        ctx = rng.integers(400, 4097, size=16 * world)
        mine = assign_streams(ctx, world, 16)[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        ms = 10.0 + 5.0 * rank  # a slower rank sets the job's time
        slowest = max_over_ranks(dist, ms)
        per_rank = gather_over_ranks(dist, ms)
        dist.barrier()
        queue.put((rank, gathered, slowest, per_rank))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_time():
    import multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    views = [g for _, g, _, _ in results]
    assert views[0] == views[1]  # both ranks agree on the assignment
    parts = views[0]
    assert sorted(parts[0] + parts[1]) == list(range(16 * world))
    assert not set(parts[0]) & set(parts[1])
    assert all(s == 15.0 for _, _, s, _ in results)
    assert all(p == [10.0, 15.0] for _, _, _, p in results)  # element r is rank r's time


def test_gather_over_ranks_without_a_group():
    assert gather_over_ranks(None, 2.5) == [2.5]

"""Stream-to-GPU sharding for the decoder KV path.

Each stream's pages, block table and steps are private to one GPU, so a node
with N GPUs runs N independent pools, one per process, and no collective is
on the data path.  This module holds the host logic of that split:

- `assign_streams`: greedy longest-processing-time assignment of streams to
  ranks by context length (the per-step HBM bytes of a stream grow with its
  context), with an equal stream count per rank;
- `max_over_ranks`: the timing reduction every multi-GPU number uses (the
  slowest rank sets the job's time);
- `gather_over_ranks`: every rank's value (per-rank times, so that a report
  can name the slowest rank).

Used by bench.py under torchrun and tested with gloo ranks on CPU.
"""
from __future__ import annotations

import heapq
from typing import List, Sequence


def assign_streams(ctx_lengths: Sequence[int], world: int, per_rank: int | None = None) -> List[List[int]]:
    """Splits stream indices over `world` ranks.

    Streams are taken longest context first and each goes to the rank with the
    smallest total context that still has room (`per_rank` streams; by default
    ceil(n / world)).  Ties go to the lower rank and, within a context length,
    the lower stream index comes first, so every rank computes the same
    assignment from the same inputs.  Returns one sorted index list per rank.
    """
    n = len(ctx_lengths)
    if world < 1:
        raise ValueError("world must be >= 1")
    cap = per_rank if per_rank is not None else -(-n // world)
    if cap * world < n:
        raise ValueError(f"{n} streams do not fit {world} ranks of {cap}")
    order = sorted(range(n), key=lambda i: (-int(ctx_lengths[i]), i))
    heap = [(0, r) for r in range(world)]  # (total ctx, rank)
    counts = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        parked = []
        while True:
            load, r = heapq.heappop(heap)
            if counts[r] < cap:
                break
            parked.append((load, r))
        out[r].append(i)
        counts[r] += 1
        heapq.heappush(heap, (load + int(ctx_lengths[i]), r))
        for item in parked:
            heapq.heappush(heap, item)
    return [sorted(x) for x in out]


def max_over_ranks(dist, value: float, device=None) -> float:
    """All-reduce MAX of a per-rank float (a timed region in ms).  `device`
    is where the reduction tensor lives: a CUDA device for NCCL, None (CPU)
    for gloo.  Returns `value` unchanged when dist is None."""
    if dist is None:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(dist, value: float, device=None) -> List[float]:
    """All-gather of a per-rank float; element r is rank r's value.  Returns
    [value] when dist is None."""
    if dist is None:
        return [float(value)]
    import torch

    world = dist.get_world_size()
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]

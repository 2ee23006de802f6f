"""Sequence sharding and timing reduction for one-process-per-GPU runs.

Relative-position attention never mixes sequences, so a packed batch shards by sequence
with no collective on the data path; the only cross-rank traffic is the barrier and the
reduction of the per-rank timings (max time, summed work).
"""
from __future__ import annotations

import heapq
from typing import Sequence

import torch


def lpt_shard(costs: Sequence[float], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of items (sequences) to `world` ranks.

    Returns, per rank, the item indices it owns (each item exactly once).  Items are
    taken in decreasing cost and each goes to the currently least-loaded rank, which
    bounds the makespan by 4/3 of optimal.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    heap = [(0.0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(s) for s in shards]


def attention_cost(length: int, heads: int = 16, head_dim: int = 64, positions: int = 0) -> float:
    """Attention FLOPs of one sequence: 4*H*D*L^2 (+ 4*H*D*L*P for DeBERTa positions)."""
    return 4.0 * heads * head_dim * length * (length + positions)


def reduce_timing(ms: float, flops: float, tokens: float, device=None):
    """(max ms over ranks, total FLOPs, total tokens).  Collective only when initialised."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return ms, flops, tokens
    dev = device if device is not None else torch.device("cpu")
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    w = torch.tensor([flops, tokens], dtype=torch.float64, device=dev)
    dist.all_reduce(w, op=dist.ReduceOp.SUM)
    return t.item(), w[0].item(), w[1].item()

"""Sharding of rollout sequences across GPUs (one process per GPU).

Decode of one sequence never reads another sequence's pages, so the
multi-GPU form of the paged-KV path is a partition: each rank owns whole
sequences (or whole GRPO groups, so shared prompt pages stay on one GPU),
its own page pool and its own block tables, and no collective runs on the
hot path. The reference runs on one GPU only; this module decides who owns
what.

Balance matters because decode time is proportional to the KV bytes a rank
reads, i.e. to the sum of its context lengths: items are assigned
longest-processing-time first (LPT), which keeps the max rank load within
4/3 of optimal and, for many similar items, within a fraction of a percent.
"""

from __future__ import annotations

import heapq
from typing import Sequence


def lpt_assign(costs: Sequence[float], world_size: int) -> list[list[int]]:
    """Assign item indices to `world_size` ranks, heaviest item first to the lightest rank.

    Deterministic: ties between items break by index, ties between ranks by
    rank id, so every rank computes the same assignment from the same costs.
    Each rank's list is returned in ascending index order.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    heap = [(0.0, r) for r in range(world_size)]
    out: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(x) for x in out]


def shard_groups(group_costs: Sequence[float], world_size: int, rank: int) -> list[int]:
    """Group indices owned by `rank` (a GRPO group never straddles two GPUs)."""
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside [0, {world_size})")
    return lpt_assign(group_costs, world_size)[rank]


def shard_loads(costs: Sequence[float], assignment: list[list[int]]) -> list[float]:
    return [sum(float(costs[i]) for i in part) for part in assignment]


def imbalance(costs: Sequence[float], assignment: list[list[int]]) -> float:
    """max rank load / mean rank load (1.0 = perfect)."""
    loads = shard_loads(costs, assignment)
    mean = sum(loads) / len(loads) if loads else 0.0
    return max(loads) / mean if mean > 0 else 1.0

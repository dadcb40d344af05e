"""Data-parallel decisions over the GPUs of one node: every rank holds a full model replica and
runs its own share of independent tree decisions; nothing crosses GPUs on the data path.

The only exchanges are on the host: the shard plan (computed identically on every rank from the
same decision list, so it needs no communication) and a gather of the per-decision results (a
few floats each) to rank 0 over the process group, which may be gloo (tests, CPU) or NCCL.

A decision's cost is estimated from its shape: the linear layers scale with its token count and
attention with its visible (query, key) pairs (trunk^2/2 + branch x trunk). Shards are balanced
longest-first (LPT): each decision, in decreasing cost, goes to the least-loaded rank.
"""
from __future__ import annotations

import heapq
from typing import Any, List, Optional, Sequence, Tuple

# Linear FLOPs per token and attention FLOPs per visible pair of Ministral-3 3B (26 layers).
LINEAR_FLOPS_PER_TOKEN = 2 * 3_026_190_336
ATTN_FLOPS_PER_PAIR = 425_984


def decision_pairs(trunk_len: int, branch_lens: Sequence[int]) -> int:
    """Visible (query, key) pairs of a tree pass: causal trunk, each branch sees trunk + itself."""
    pairs = trunk_len * (trunk_len + 1) // 2
    for b in branch_lens:
        pairs += b * trunk_len + b * (b + 1) // 2
    return pairs


def decision_cost(trunk_len: int, branch_lens: Sequence[int]) -> float:
    """Estimated FLOPs of one ForwardTreeAsync decision."""
    tokens = trunk_len + sum(branch_lens)
    return float(tokens) * LINEAR_FLOPS_PER_TOKEN + float(decision_pairs(trunk_len, branch_lens)) * ATTN_FLOPS_PER_PAIR


def shard_decisions(costs: Sequence[float], world: int) -> List[List[int]]:
    """Indices of the decisions each rank runs: longest-first onto the least-loaded rank.

    Deterministic (ties broken by decision index, then rank), so every rank derives the same
    plan from the same list. Each rank's list is in increasing index order.
    """
    if world < 1:
        raise ValueError("world must be at least 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap: List[Tuple[float, int]] = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    for s in shards:
        s.sort()
    return shards


def shard_loads(costs: Sequence[float], shards: Sequence[Sequence[int]]) -> List[float]:
    return [sum(costs[i] for i in s) for s in shards]


def gather_results(dist: Any, rank: int, world: int, mine: Sequence[Tuple[int, Any]]) -> Optional[List[Any]]:
    """Collect (decision index, result) pairs from every rank on rank 0, in decision order.

    `dist` is torch.distributed with an initialised process group; with world == 1 it may be
    None. Returns the ordered results on rank 0 and None elsewhere.
    """
    if world == 1 or dist is None:
        return [r for _, r in sorted(mine, key=lambda p: p[0])]
    box: List[Any] = [None] * world if rank == 0 else None  # type: ignore[assignment]
    dist.gather_object(list(mine), box, dst=0)
    if rank != 0:
        return None
    merged = [p for part in box for p in part]
    merged.sort(key=lambda p: p[0])
    return [r for _, r in merged]

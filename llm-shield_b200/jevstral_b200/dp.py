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


# ------------------------------------------------------------------ failure handling
#
# A rank that dies (raises, exits, or never starts) must not lose its decisions. run_requeued
# keeps the same longest-first shard plan, but every decision is claimed in a shared key-value
# store before it runs and its result is published there; ranks beat a heartbeat after every
# decision (and from a background thread). A rank that finishes its own shard takes over any
# decision whose owner is marked failed or whose heartbeat is older than `timeout_s`, stealing
# the claim of a dead rank atomically (compare-and-set), so each decision's published result
# comes from one completed run. Rank 0 hosts the store and collects the results in decision
# order; its own failure ends the job. Nothing here touches a GPU: the store is
# torch.distributed's TCPStore (or any object with set/get/check/compare_set).

import pickle
import threading
import time


def _key(kind: str, i: int) -> str:
    return f"jvdp/{kind}/{i}"


class RankFailed(RuntimeError):
    """Raised by run_requeued on the rank whose own run_one raised, after it has marked itself
    failed in the store (so the survivors take its decisions at once)."""


def _alive(store, rank: int, now: float, timeout_s: float, started: float, startup_s: float) -> bool:
    if store.check([_key("failed", rank)]):
        return False
    if store.check([_key("hb", rank)]):
        return now - float(store.get(_key("hb", rank)).decode()) <= timeout_s
    return now - started <= startup_s  # never started: dead once the start-up grace has passed


def run_requeued(store, rank: int, world: int, costs: Sequence[float], run_one, timeout_s: float = 10.0,
                 poll_s: float = 0.05, startup_s: float = 60.0) -> Optional[List[Any]]:
    """Run decision i (run_one(i) -> picklable result) for every i, sharded longest-first over
    `world` ranks, surviving the failure of any rank but 0. Returns the results in decision order
    on rank 0 and None elsewhere. A rank is dead once it has marked itself failed, once its
    heartbeat is older than `timeout_s`, or, if it never beat, once `startup_s` have passed since
    rank 0 opened the job (the time rank 0 publishes in the store, which every rank reads)."""
    if rank == 0:
        store.set("jvdp/start", repr(time.time()))
    started = float(store.get("jvdp/start").decode())
    n = len(costs)
    plan = shard_decisions(costs, world)
    owner = {i: r for r, s in enumerate(plan) for i in s}
    me = str(rank).encode()
    stop = threading.Event()

    def beat():
        while not stop.is_set():
            store.set(_key("hb", rank), repr(time.time()))
            stop.wait(timeout_s / 4)

    hb = threading.Thread(target=beat, daemon=True)
    store.set(_key("hb", rank), repr(time.time()))
    hb.start()

    def run(i: int) -> None:
        try:
            res = run_one(i)
        except BaseException as e:
            store.set(_key("failed", rank), repr(e))
            stop.set()
            raise RankFailed(f"rank {rank} failed on decision {i}") from e
        store.set(_key("res", i), pickle.dumps(res))
        store.set(_key("hb", rank), repr(time.time()))

    def claim(i: int, holder: bytes) -> bool:
        got = store.compare_set(_key("claim", i), holder, me)
        return got == me

    try:
        for i in plan[rank]:
            if not store.check([_key("res", i)]) and claim(i, b""):
                run(i)
        while True:
            missing = [i for i in range(n) if not store.check([_key("res", i)])]
            if not missing:
                break
            took = False
            now = time.time()
            for i in missing:
                if store.check([_key("res", i)]):
                    continue
                held = store.get(_key("claim", i)) if store.check([_key("claim", i)]) else b""
                holder = int(held.decode()) if held else owner[i]
                if holder == rank or _alive(store, holder, now, timeout_s, started, startup_s):
                    continue
                if claim(i, held):
                    run(i)
                    took = True
            if not took:
                time.sleep(poll_s)
    finally:
        stop.set()
    store.set(_key("done", rank), b"1")
    if rank != 0:
        return None
    results = [pickle.loads(store.get(_key("res", i))) for i in range(n)]
    # rank 0 hosts the store: stay until every rank still alive has left the loop above
    while True:
        now = time.time()
        waiting = [r for r in range(1, world)
                   if not store.check([_key("done", r)]) and _alive(store, r, now, timeout_s, started, startup_s)]
        if not waiting:
            return results
        time.sleep(poll_s)

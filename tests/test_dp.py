"""The data-parallel plumbing (jevstral_b200.dp): the shard plan and the host gather, including a
two-rank gloo process group on the CPU (the GPU runs use the same calls over NCCL)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from jevstral_b200 import dp


def c5_shapes(n, seed=7):
    """Decision shapes with C5's distributions: trunk U[128, 4096], 2-9 branches of U[16, 64]."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        trunk = int(rng.integers(128, 4097))
        branches = [int(rng.integers(16, 65)) for _ in range(int(rng.integers(2, 10)))]
        out.append((trunk, branches))
    return out


def test_pairs_follow_the_tree_mask():
    # causal trunk of 3: 1 + 2 + 3 keys; a branch of 2 sees the trunk and itself: 2*3 + 1 + 2
    assert dp.decision_pairs(3, []) == 6
    assert dp.decision_pairs(3, [2]) == 6 + 2 * 3 + 3


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_cover_every_decision_once_and_balance(world):
    shapes = c5_shapes(257)
    costs = [dp.decision_cost(t, b) for t, b in shapes]
    shards = dp.shard_decisions(costs, world)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(costs)))
    assert all(s == sorted(s) for s in shards)
    loads = dp.shard_loads(costs, shards)
    # longest-processing-time bound: no rank exceeds the mean load by more than one decision
    assert max(loads) <= sum(costs) / world + max(costs) + 1e-6
    assert dp.shard_decisions(costs, world) == shards  # every rank derives the same plan


def test_shard_plan_rejects_an_empty_world():
    with pytest.raises(ValueError):
        dp.shard_decisions([1.0], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = c5_shapes(40, seed=3)
        costs = [dp.decision_cost(t, b) for t, b in shapes]
        mine = dp.shard_decisions(costs, world)[rank]
        # stand-in for a decision: its z_i would come from the GPU; here a function of the shape
        results = [(i, [float(shapes[i][0]), float(len(shapes[i][1]))]) for i in mine]
        gathered = dp.gather_results(dist, rank, world, results)
        import torch

        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the bench's max-over-ranks of the device time
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), np.asarray(gathered))
            np.save(os.path.join(out_dir, "tmax.npy"), t.numpy())
        else:
            assert gathered is None
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    shapes = c5_shapes(40, seed=3)
    want = np.asarray([[float(t), float(len(b))] for t, b in shapes])
    got = np.load(tmp_path / "gathered.npy")
    assert np.array_equal(got, want)
    assert float(np.load(tmp_path / "tmax.npy")[0]) == float(world)


def test_single_rank_gather_needs_no_process_group():
    assert dp.gather_results(None, 0, 1, [(2, "c"), (0, "a"), (1, "b")]) == ["a", "b", "c"]


# ------------------------------------------------------------ failure handling (host side)


def _requeue_main(rank, world, port, out_dir, scenario):
    import datetime
    import time

    from torch.distributed import TCPStore

    ready = os.path.join(out_dir, "store_ready")
    if rank != 0:  # connect once the store is listening (a client that starts first backs off for long)
        t0 = time.time()
        while not os.path.exists(ready) and time.time() - t0 < 60:
            time.sleep(0.02)
    store = TCPStore("127.0.0.1", port, None, rank == 0, datetime.timedelta(seconds=60), wait_for_workers=False)
    if rank == 0:
        open(ready, "w").close()
    shapes = c5_shapes(30, seed=5)
    costs = [dp.decision_cost(t, b) for t, b in shapes]
    count = [0]

    def run_one(i):
        count[0] += 1
        if scenario == "raise" and rank == 2 and count[0] == 2:
            raise RuntimeError("injected failure")
        if scenario == "exit" and rank == 1 and count[0] == 2:
            os._exit(3)  # dies mid-decision, with its claim held and without marking itself failed
        time.sleep(0.01)
        return (i, float(shapes[i][0]) * len(shapes[i][1]), rank)

    res = dp.run_requeued(store, rank, world, costs, run_one, timeout_s=1.0, poll_s=0.02, startup_s=6.0)
    if rank == 0:
        np.save(os.path.join(out_dir, "results.npy"), np.asarray(res, dtype=np.float64))


@pytest.mark.parametrize("scenario", ["raise", "exit", "absent"])
def test_a_failed_rank_s_decisions_are_requeued_onto_the_survivors(tmp_path, scenario):
    """Three ranks share a 30-decision list over a TCPStore. One of them fails: rank 2 raises on its
    second decision (and marks itself failed), or rank 1 exits mid-decision holding its claim (found
    by its stale heartbeat), or rank 2 never starts (found once the start-up grace passes). The survivors
    run every orphaned decision and rank 0 returns all 30 results, correct and in order."""
    import multiprocessing as mpx

    world, port = 3, _free_port()
    ctx = mpx.get_context("spawn")
    ranks = [0, 1] if scenario == "absent" else [0, 1, 2]
    procs = [ctx.Process(target=_requeue_main, args=(r, world, port, str(tmp_path), scenario)) for r in ranks]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = {r: p.exitcode for r, p in zip(ranks, procs)}
    failed = {"raise": 2, "exit": 1, "absent": None}[scenario]
    for r, c in codes.items():
        assert (c != 0) if r == failed else (c == 0), codes
    got = np.load(tmp_path / "results.npy")
    shapes = c5_shapes(30, seed=5)
    assert got[:, 0].tolist() == list(range(30))
    assert got[:, 1].tolist() == [float(t) * len(b) for t, b in shapes]
    costs = [dp.decision_cost(t, b) for t, b in shapes]
    lost = dp.shard_decisions(costs, world)[failed if failed is not None else 2]
    assert len(lost) > 0
    # the decisions the failed rank never finished were run by a survivor
    ran_by = {int(i): int(r) for i, _, r in got}
    assert all(ran_by[i] != (failed if failed is not None else 2) for i in lost[1:])

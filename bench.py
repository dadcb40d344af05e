#!/usr/bin/env python3
"""Benchmark of the B200 Jevstral hot path ("tree-decision prefill tokens/s/GPU and
decisions/s at 1/2/4/8 B200; % roofline").

Default workload (configs[1], "C2"): one ForwardTreeAsync decision per step on a random-init
Ministral-3 3B with Q8_0 weights — a 512-token causal trunk and 5 option branches of 32
tokens, verdict rows only (2 rows per branch), then z_i and softmax(z/T=1) on the host.
A step is one such decision (672 tokens) on every GPU; GPUs are independent replicas
(data parallel, no collective on the data path; weak scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c1|c2|c3|c4|c5]

Prints one JSON line (rank 0). `value` is device time (CUDA events on the context's
stream bracketing the K steps, max over ranks); `e2e` is host wall-clock around the same
public-API calls with host buffers (token upload and result download inside).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
for p in (REPO / "llm-shield_b200", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

MODEL_DIR = Path(os.environ.get("JV_BENCH_DIR", "/tmp/jv_bench"))
VOCAB = 131072
ROWS = [13059, 2649]
LINEAR_FLOPS_PER_TOKEN = 2 * 3_026_190_336  # 26 layers x (Q+K+V+O+gate+up+down)
LAYER_WEIGHTS = 116_391_936                  # Q+K+V+O+gate+up+down of one layer


def peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- workloads


def c2_decision(rng):
    trunk = [1] + rng.integers(1000, VOCAB, 511).tolist()
    branches = [rng.integers(1000, VOCAB, 32).tolist() for _ in range(5)]
    return trunk, branches


def c5_decision(rng):
    trunk = [1] + rng.integers(1000, VOCAB, int(rng.integers(128, 4097)) - 1).tolist()
    nb = int(rng.integers(2, 10))
    branches = [rng.integers(1000, VOCAB, int(rng.integers(16, 65))).tolist() for _ in range(nb)]
    return trunk, branches


def attention_pairs(trunk_len, branch_lens):
    """Visible (query, key) pairs of a tree pass: causal trunk, each branch sees trunk + itself."""
    pairs = trunk_len * (trunk_len + 1) // 2
    for b in branch_lens:
        pairs += b * trunk_len + b * (b + 1) // 2
    return pairs


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *e):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# -------------------------------------------------------------- cpu oracle


def cpu_baseline_c2(steps: int = 1, min_seconds: float = 10.0):
    """The oracle (CPU restatement, all host threads) on a bounded sample of the C2 workload: the
    same 512+5x32 tree decision through a 2-layer model of the full width, best of repeated runs
    until `min_seconds` of CPU work, scaled to 26 layers (per-layer cost is identical)."""
    from jevstral_b200.synth import SynthConfig, write_random_gguf
    from oracle import binding as ob

    MODEL_DIR.mkdir(parents=True, exist_ok=True)
    path = MODEL_DIR / "wide2_q8_0.gguf"
    if not path.exists():
        write_random_gguf(path, SynthConfig(layers=2), "Q8_0", seed=0, backend="fast")
    rng = np.random.default_rng(99)
    trunk, branches = c2_decision(rng)
    tokens = len(trunk) + sum(len(b) for b in branches)
    best, spent, runs = float("inf"), 0.0, 0
    with ob.OracleModel(path) as o:
        while runs < max(steps, 1) or spent < min_seconds:
            o.kv_reset()
            t0 = time.perf_counter()
            o.forward_tree(trunk, branches, ROWS)
            dt = time.perf_counter() - t0
            best, spent, runs = min(best, dt), spent + dt, runs + 1
            if runs >= 50:
                break
    per_layer = best / 2
    full = per_layer * 26
    return {"value": tokens / full, "unit": "tokens/s", "cores": int(ob.lib.orc_threads()), "kind": "port",
            "sample": f"C2 tree decision ({tokens} tokens) through 2 of 26 layers at full width, best of {runs} runs "
                      f"({spent:.1f} s CPU), scaled x13 to 26 layers",
            "seconds_per_decision": full}


# ------------------------------------------------------------------- b200 arm


def ensure_model(qtype: str, rank: int, dist, layers: int = 26) -> Path:
    from jevstral_b200.synth import SynthConfig, write_random_gguf

    MODEL_DIR.mkdir(parents=True, exist_ok=True)
    path = MODEL_DIR / f"ministral3b_{layers}l_{qtype.lower()}_seed0.gguf"
    if rank == 0 and not path.exists():
        write_random_gguf(path, SynthConfig(layers=layers), qtype, seed=0, backend="fast")
    if dist is not None:
        dist.barrier()
    return path


def run_b200(args, rank, world, local_rank, dist):
    import torch

    import jevstral_b200 as jv

    torch.cuda.set_device(local_rank)
    qtype = {"c3": "Q5_1", "c4": "Q4_0"}.get(args.config, "Q8_0")
    path = ensure_model(qtype, rank, dist, args.layers)
    model = jv.Model(path, device=local_rank, kv_pool_mb=args.kv_pool_mb)
    ctx = jv.MinistralModel(model, 512)
    stream = torch.cuda.ExternalStream(ctx.stream, device=local_rank)
    rng = np.random.default_rng(1000 + rank)

    if args.config == "c4":
        return run_decode(args, rank, world, dist, model, ctx, stream, rng)

    gen = c5_decision if args.config == "c5" else c2_decision
    if args.config == "c1":
        gen = lambda r: ([1] + r.integers(1000, VOCAB, 255).tolist(), None)  # noqa: E731
    if args.config == "c3":
        # decision 1: 4096-token trunk + 9 x 48; decision 2 shares the trunk's pages and, per
        # the decider's never-empty-trunk rule, re-runs its last token before 9 fresh branches
        gen = lambda r: ([1] + r.integers(1000, VOCAB, 4095).tolist(),  # noqa: E731
                         [r.integers(1000, VOCAB, 48).tolist() for _ in range(9)],
                         [r.integers(1000, VOCAB, 48).tolist() for _ in range(9)])
    work = [gen(rng) for _ in range(args.warmup + args.steps)]

    def step(trunk, branches, second=None):
        ctx.kv_cache.reset()
        if branches is None:  # C1: causal prefill, verdict rows of the last position
            v = ctx.forward_selected(trunk, ROWS)[None, :]
        else:
            v = ctx.forward_tree(trunk, branches, ROWS)
        z = jv.margins_from_verdicts(v, 1)
        p = jv.decision_probs(z)
        if second is not None:
            ctx.kv_cache.truncate(len(trunk) - 1)
            v2 = ctx.forward_tree([trunk[-1]], second, ROWS)
            p = jv.decision_probs(jv.margins_from_verdicts(v2, 1))
        return p

    for w in work[: args.warmup]:
        step(*w)
    torch.cuda.synchronize()

    timed = work[args.warmup:]
    shard = None
    if args.config == "c5":
        # C5: one seeded list of world x steps random trees, the same on every rank, sharded
        # longest-first by estimated cost (jevstral_b200.dp); the z_i come back to rank 0.
        grng = np.random.default_rng(4242)
        glob = [c5_decision(grng) for _ in range(world * args.steps)]
        costs = [jv.dp.decision_cost(len(t), [len(b) for b in br]) for t, br in glob]
        shard = jv.dp.shard_decisions(costs, world)[rank]
        timed = [glob[i] for i in shard]
    # C5 runs its shard through jv_decide_batch: consecutive decisions are grouped into one pass of
    # at most --c5-batch-tokens tokens (each decision bit-identical to running it alone).
    batches = None
    if args.config == "c5" and args.c5_batch_tokens > 0:
        batches, cur, n = [], [], 0
        for w in timed:
            k = len(w[0]) + sum(len(b) for b in w[1])
            if cur and n + k > args.c5_batch_tokens:
                batches.append(cur)
                cur, n = [], 0
            cur.append(w)
            n += k
        if cur:
            batches.append(cur)

    def run_all():
        out = []
        if batches is None:
            for w in timed:
                out.append(step(*w))
            return out
        for bt in batches:
            ctx.kv_cache.reset()
            for v in ctx.decide_batch(bt, ROWS):
                out.append(jv.decision_probs(jv.margins_from_verdicts(v, 1)))
        return out

    if args.config == "c5":
        # size every buffer before the clock starts: the shard's largest tree (or batch) once
        if batches is None:
            step(*max(timed, key=lambda w: len(w[0]) + sum(len(b) for b in w[1])))
        else:
            big = max(batches, key=lambda bt: sum(len(w[0]) + sum(len(b) for b in w[1]) for w in bt))
            ctx.kv_cache.reset()
            ctx.decide_batch(big, ROWS)
        torch.cuda.synchronize()
    results = []

    def toks_of(w):
        n = len(w[0]) + (sum(len(b) for b in w[1]) if w[1] else 0)
        if len(w) > 2:
            n += 1 + sum(len(b) for b in w[2])
        return n

    def pairs_of(w):
        p = attention_pairs(len(w[0]), [len(b) for b in w[1]] if w[1] else [])
        if len(w) > 2:  # the re-run trunk token sees the trunk; each branch the trunk, that token and itself
            L = len(w[0])
            p += L + sum(b * L + b * (b + 1) // 2 for b in (len(x) for x in w[2]))
        return p

    tokens = sum(toks_of(w) for w in timed)
    pairs = sum(pairs_of(w) for w in timed)
    h2d = sum(4 * 3 * toks_of(w) for w in timed) // len(timed)
    d2h = 4 * len(ROWS) * (len(timed[0][1]) if timed[0][1] else 1) * (2 if len(timed[0]) > 2 else 1)

    launches0 = jv.kernel_launches()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        ev0.record(stream)
        results = run_all()
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    if dist is not None:
        dist.barrier()
    launches = jv.kernel_launches() - launches0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    # Per-kernel-class device time (roofline.achieved): the same decisions once more with CUDA
    # events around every GEMM / attention launch, outside the timed region (the events would
    # serialise launches that otherwise overlap).
    ctx.profile(True)
    ctx.profile_reset()
    run_all()
    torch.cuda.synchronize()
    prof = {k: ctx.profile_read(k) for k in ("gemm", "attention", "gemv")}
    ctx.profile(False)

    if dist is not None:
        t = torch.tensor([dev_s, wall], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, wall = t.tolist()
        # the whole job's tokens: ranks may hold different shares (C5 shards by cost)
        tt = torch.tensor([float(tokens), float(len(timed))], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        job_tokens, job_decisions = tt.tolist()
    else:
        job_tokens, job_decisions = float(tokens), float(len(timed))
    gathered = None
    if shard is not None:
        gathered = jv.dp.gather_results(dist, rank, world, list(zip(shard, [r.tolist() for r in results])))

    res = None
    if rank == 0:
        pk, src = peaks()
        g = prof["gemm"]
        gemm_tflops = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
        peak = pk["bf16_tflops_sustained"]
        n_dec = len(timed)
        res = {
            "metric": f"tree-decision prefill tokens/s ({args.config.upper()})",
            "value": job_tokens / dev_s,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dev_s / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 (Q8_0/Q5_1/Q4_0 weights decoded to fp16 in SMEM; fp32 accumulate)",
            "data": "synthetic (random-init Ministral-3 3B, N(0,0.02) weights, uniform token ids, seeded)",
            "config": {"workload": WORKLOADS[args.config], "weights": qtype, "tokens_per_step": tokens // n_dec,
                       "parallelism": f"dp{world} (independent replicas, no collective)",
                       "l2": "weights (3.2+ GB) exceed the 126 MB L2 and stream from HBM every step",
                       **({"batching": f"jv_decide_batch, {len(batches)} passes of up to {args.c5_batch_tokens} tokens"}
                          if batches is not None else {})},
            "decisions_per_s": job_decisions / dev_s,
            "linear_tflops": job_tokens * LINEAR_FLOPS_PER_TOKEN * args.layers / 26 / dev_s / 1e12,
            "attention_pairs_per_step": pairs // n_dec,
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc (all four projections)",
                         "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": gemm_tflops / peak if peak else None,
                         "peak_source": f"{src} bf16 dense sustained (fp16 runs at the same rate)",
                         "traffic": gemm_traffic_per_launch(),
                         "launches": g["launches"], "avg_launch_us": g["ms"] / max(1, g["launches"]) * 1e3,
                         "algorithmic_flops_per_launch": g["flops"] / max(1, g["launches"])},
            "kernels": {k: {"ms_per_step": v["ms"] / n_dec, "launches_per_step": v["launches"] / n_dec,
                            "tflops": (v["flops"] / (v["ms"] / 1e3) / 1e12) if v["ms"] else None,
                            "gbs": (v["bytes"] / (v["ms"] / 1e3) / 1e9) if v["ms"] else None}
                        for k, v in prof.items()},
            "e2e": {"value": job_tokens / wall, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "host wall-clock around the public C-ABI calls ("
                           + ("jv_decide_batch" if batches is not None else "jv_forward_tree") + ") with host buffers"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if gathered is not None:
            res["gathered_decisions"] = len(gathered)  # z_i of every rank's shard, collected on rank 0
    ctx.close()
    model.close()
    return res


def run_decode(args, rank, world, dist, model, ctx, stream, rng):
    """C4: 1024-token prompt, then greedy decode steps with the full LM head (HBM-bound GEMV)."""
    import torch

    import jevstral_b200 as jv

    prompt = [1] + rng.integers(1000, VOCAB, 1023).tolist()
    ctx.prefill(prompt)
    base = ctx.kv_cache.length
    # warm-up: the same call as the timed one (it captures the step graph), then rewind
    for _ in range(max(1, args.warmup // 3)):
        ctx.decode_greedy(1500, args.steps)
        ctx.kv_cache.truncate(base)
    torch.cuda.synchronize()
    l0 = jv.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(rank) as clocks:
        t0 = time.perf_counter()
        ev0.record(stream)
        toks = ctx.decode_greedy(1500, args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    pk, src = peaks()
    # Algorithmic bytes of one step: every layer matrix and the LM head once (Q4_0: 18 bytes
    # per 32 weights) plus the K/V rows of the visible context (fp16, 106,496 B per position).
    weight_bytes = (LAYER_WEIGHTS * args.layers + VOCAB * 3072) * 18 / 32
    mean_ctx = base + (args.steps + 1) / 2
    step_bytes = weight_bytes + mean_ctx * 106_496
    gbs = step_bytes * args.steps / dev_s / 1e9
    return {
        "metric": "greedy decode tokens/s (C4)", "value": world * args.steps / dev_s, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_s / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (Q4_0 weights)",
        "data": "synthetic", "config": {"workload": WORKLOADS["c4"], "parallelism": f"dp{world}"},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (k_dec_gemv x5 per layer + k_dec_attn + head)",
                     "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
                     "traffic": None, "peak_source": src, "algorithmic_bytes_per_step": step_bytes},
        "e2e": {"value": world * args.steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": jv.kernel_launches() - l0, "clocks": clocks.summary(), "last_tokens": toks[-4:].tolist(),
    }


def gemm_traffic_per_launch():
    """DRAM bytes per k_gemm_tc launch from the committed ncu summary, when one exists."""
    f = REPO / "profiles" / "gemm_tc_c2.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


WORKLOADS = {
    "c1": "C1: single 256-token causal prefill (BOS + 255), verdict rows at the last position, Q8_0",
    "c2": "C2: one tree decision, 512-token trunk + 5 branches x 32, 2 verdict rows per branch, Q8_0",
    "c3": "C3: long-trunk tree, 4096-token trunk + 9 branches x 48, then a second decision on the same trunk pages (last trunk token re-run + 9 fresh branches x 48), Q5_1",
    "c4": "C4: greedy decode after a 1024-token prompt, full LM head + argmax, Q4_0, batch 1",
    "c5": "C5: random trees (trunk U[128,4096], 2-9 branches of U[16,64]), Q8_0",
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=26, help="fewer layers of the same width (profiling only)")
    ap.add_argument("--kv-pool-mb", type=int, default=4096)
    ap.add_argument("--c5-batch-tokens", type=int, default=0,
                    help="C5: group decisions into jv_decide_batch passes of at most this many tokens "
                         "(0, the default: one jv_forward_tree per decision; measured no faster at C5's sizes)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return
        # The reference is managed C# (.NET 10) and cannot be built or run on this image; its
        # CPU path is timed through the oracle, the op-for-op C++ restatement.
        t0 = time.perf_counter()
        cb = cpu_baseline_c2(steps=args.steps + args.warmup, min_seconds=10.0)
        wall = time.perf_counter() - t0
        out = {"impl": "reference", "metric": f"tree-decision prefill tokens/s ({args.config.upper()})",
               "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": cb["seconds_per_decision"] * 1e3, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic",
               "config": {"workload": WORKLOADS["c2"], "weights": "Q8_0", "parallelism": "host cores"},
               "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
               "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
               "wall_s": wall}
        print(json.dumps(out), flush=True)
        return

    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    res = run_b200(args, rank, world, local_rank, dist)
    if rank == 0 and res is not None:
        if world == 1 and not args.no_cpu_baseline and args.config == "c2":
            cb = cpu_baseline_c2()
            res["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

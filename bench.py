#!/usr/bin/env python3
"""Benchmark of the B200 Jevstral hot path ("tree-decision prefill tokens/s/GPU and
decisions/s at 1/2/4/8 B200; % roofline").

Default workload ("C5"): independent ForwardTreeAsync decisions on a
random-init Ministral-3 3B with Q8_0 weights — trunks U[128, 4096] tokens, 2-9 branches of
U[16, 64] tokens, token ids U[1000, 131072), verdict rows only, then z_i and softmax(z/T=1) on
the host. One seeded decision list is sharded longest-first by cost over the ranks (one GPU
each, full replicas, no collective on the data path). A step is --c5-per-step decisions per GPU
(weak scaling: per-GPU work fixed as N grows).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c1|c2|c3|c4|c5]

Prints one JSON line (rank 0). `value` is whole-job tokens/s from device time (CUDA events on the
context's stream around the K steps, max over ranks); `e2e` is host wall-clock around the same
public C-ABI calls with host token buffers and host results (uploads and downloads inside).

`--impl reference` times the reference's CPU path — the oracle restatement of the reference's
managed code (oracle/), since the C# reference cannot run on this image — on the same
configuration, the same seeded inputs and the same 26-layer model file, with every host thread.
That process loads no library of this package: its model file is filled by the stand-alone
`jvsynth` program.
"""
from __future__ import annotations

import argparse
import importlib.util
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
PKG = REPO / "llm-shield_b200"
for p in (PKG, REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

MODEL_DIR = Path(os.environ.get("JV_BENCH_DIR", "/tmp/jv_bench"))
VOCAB = 131072
ROWS = [13059, 2649]
LINEAR_FLOPS_PER_TOKEN = 2 * 3_026_190_336  # 26 layers x (Q+K+V+O+gate+up+down)
LAYER_WEIGHTS = 116_391_936                  # Q+K+V+O+gate+up+down of one layer
QTYPE = {"c1": "Q8_0", "c2": "Q8_0", "c3": "Q5_1", "c4": "Q4_0", "c5": "Q8_0"}
C5_SEED, C5_SIZE = 4242, 4096

WORKLOADS = {
    "c1": "C1: single 256-token causal prefill (BOS + 255), verdict rows at the last position, Q8_0",
    "c2": "C2: one tree decision, 512-token trunk + 5 branches x 32, 2 verdict rows per branch, Q8_0",
    "c3": "C3: long-trunk tree, 4096-token trunk + 9 branches x 48, then a second decision on the same trunk pages "
          "(last trunk token re-run + 9 fresh branches x 48), Q5_1",
    "c4": "C4: greedy decode after a 1024-token prompt, full LM head + argmax, Q4_0, batch 1",
    "c5": "C5: independent tree decisions (trunk U[128,4096], 2-9 branches of U[16,64], ids U[1000,131072)) from "
          "seed 4242, sharded by cost over the GPUs, Q8_0",
}


def peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_synth():
    """jevstral_b200/synth.py on its own: the package __init__ loads libjv.so, which the reference
    arm must not do."""
    name = "jv_synth_standalone"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG / "jevstral_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def model_path(qtype: str, layers: int = 26) -> Path:
    return MODEL_DIR / f"ministral3b_{layers}l_{qtype.lower()}_seed0.gguf"


def ensure_model(qtype: str, layers: int = 26, backend: str = "fast") -> Path:
    """The random-init 3B model of BASELINE's configs (seed 0), written once per box. Both arms use
    the same file; the "exe" backend writes the same bytes without loading a package library."""
    synth = load_synth()
    MODEL_DIR.mkdir(parents=True, exist_ok=True)
    path = model_path(qtype, layers)
    if not path.exists():
        cfg = synth.SynthConfig(layers=layers)
        synth.write_random_gguf(path, cfg, qtype, seed=0, backend=backend)
    return path


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


def c5_list(n: int):
    """The first n decisions of C5's seeded stream (the 4096-decision job is its first 4096)."""
    rng = np.random.default_rng(C5_SEED)
    return [c5_decision(rng) for _ in range(n)]


def c1_item(rng):
    return [1] + rng.integers(1000, VOCAB, 255).tolist(), None


def c3_item(rng):
    # decision 1: 4096-token trunk + 9 x 48; decision 2 shares the trunk's pages and, per the
    # decider's never-empty-trunk rule, re-runs its last token before 9 fresh branches
    return ([1] + rng.integers(1000, VOCAB, 4095).tolist(), [rng.integers(1000, VOCAB, 48).tolist() for _ in range(9)],
            [rng.integers(1000, VOCAB, 48).tolist() for _ in range(9)])


GEN = {"c1": c1_item, "c2": c2_decision, "c3": c3_item}


def attention_pairs(trunk_len, branch_lens):
    """Visible (query, key) pairs of a tree pass: causal trunk, each branch sees trunk + itself."""
    pairs = trunk_len * (trunk_len + 1) // 2
    for b in branch_lens:
        pairs += b * trunk_len + b * (b + 1) // 2
    return pairs


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


def timed_items(config: str, steps: int, per_step: int, world: int, rank: int):
    """The work of the timed region: (this rank's items, every rank's item count, shard indices)."""
    if config == "c5":
        n = world * steps * per_step
        glob = c5_list(max(n, 1))[:n]
        from jevstral_b200 import dp

        costs = [dp.decision_cost(len(t), [len(b) for b in br]) for t, br in glob]
        shard = dp.shard_decisions(costs, world)[rank]
        return [glob[i] for i in shard], shard
    rng = np.random.default_rng(1000 + rank)
    return [GEN[config](rng) for _ in range(steps)], None


def config_block(config: str, per_step: int):
    """The `config` object both arms print (identical for the same --config)."""
    c = {"workload": WORKLOADS[config], "weights": QTYPE[config], "layers": 26,
         "model": "random-init Ministral-3 3B (26 layers, hidden 3072, 32/8 heads, FFN 9216, vocab 131072), seed 0",
         "verdict_rows": ROWS}
    if config == "c5":
        c["decisions_per_step_per_gpu"] = per_step
    c["l2"] = "inputs larger than L2: the weights (1.7-3.2 GB) stream from HBM on every pass"
    return c


def metric_name(config: str) -> str:
    if config == "c4":
        return "greedy decode tokens/s (C4)"
    return f"tree-decision prefill tokens/s ({config.upper()})"


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
            time.sleep(0.3)  # the first sample lands before the timed work starts
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


def time_oracle(config: str, path: Path, budget_s: float, max_steps: int):
    """The oracle (the CPU restatement of the reference's managed path, every host thread) on the
    configuration's own work items at full depth, one step at a time until `max_steps` steps or
    `budget_s` seconds of timed work (at least one step). Warm-up: one 16-token prefill, which
    touches every weight page of the memory-mapped model. Returns the measured totals."""
    from oracle import binding as ob

    cap = 5120 if config == "c3" else 1536
    steps, seconds, tokens, decisions = 0, 0.0, 0, 0
    per_step = []
    with ob.OracleModel(path, cap) as o:
        o.forward([1] + list(range(1000, 1015)), logits=False)
        if config == "c4":
            rng = np.random.default_rng(1000)
            o.kv_reset()
            o.forward([1] + rng.integers(1000, VOCAB, 1023).tolist(), logits=False)
            tok = 1500
            while steps < max_steps and (steps == 0 or seconds < budget_s):
                t0 = time.perf_counter()
                tok = int(np.argmax(o.forward([tok])))
                dt = time.perf_counter() - t0
                steps, seconds, tokens = steps + 1, seconds + dt, tokens + 1
                per_step.append(dt)
            sample = f"{steps} greedy decode steps (full LM head + argmax) after a 1024-token prompt, 26 layers"
        else:
            items = c5_list(max_steps) if config == "c5" else timed_items(config, max_steps, 1, 1, 0)[0]
            for w in items:
                if steps > 0 and seconds >= budget_s:
                    break
                o.kv_reset()
                t0 = time.perf_counter()
                if w[1] is None:
                    o.forward_selected(w[0], ROWS)
                else:
                    o.forward_tree(w[0], w[1], ROWS)
                    if len(w) > 2:
                        o.kv_truncate(len(w[0]) - 1)
                        o.forward_tree(w[0][-1:], w[2], ROWS)
                dt = time.perf_counter() - t0
                steps, seconds, tokens = steps + 1, seconds + dt, tokens + toks_of(w)
                decisions += 1 if w[1] is None else (2 if len(w) > 2 else 1)
                per_step.append(dt)
            what = {"c1": "256-token prefills", "c2": "C2 tree decisions", "c3": "C3 decision pairs",
                    "c5": "decisions of the C5 list (its first ones)"}[config]
            sample = f"{steps} {what} ({tokens} tokens), 26 layers"
        cores = int(ob.lib.orc_threads())
    return {"value": tokens / seconds, "unit": "tokens/s", "steps": steps, "seconds": seconds, "tokens": tokens,
            "decisions": decisions, "ms_per_step": seconds / steps * 1e3, "best_step_ms": min(per_step) * 1e3,
            "cores": cores, "kind": "port", "sample": sample + f", {seconds:.1f} s timed"}


def run_reference(args, world):
    """--impl reference: the reference's CPU path (oracle port) on this configuration, rank 0 only."""
    t0 = time.perf_counter()
    path = ensure_model(QTYPE[args.config], 26, backend="exe")
    r = time_oracle(args.config, path, args.ref_budget_s, args.steps)
    out = {"impl": "reference", "metric": metric_name(args.config), "value": r["value"], "unit": "tokens/s",
           "n_gpus": world, "steps": r["steps"], "warmup": 1, "ms_per_step": r["ms_per_step"],
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (random-init Ministral-3 3B, N(0,0.02) weights, uniform token ids, seeded)",
           "config": config_block(args.config, args.c5_per_step),
           "host": {"cores": r["cores"], "steps_requested": args.steps, "budget_s": args.ref_budget_s,
                    "warmup_sample": "one 16-token prefill (pages the weights in)"},
           "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
           "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "wall_s": time.perf_counter() - t0}
    if args.config != "c4":
        out["decisions_per_s"] = r["decisions"] / r["seconds"]
    return out


# ------------------------------------------------------------------- b200 arm


def run_b200(args, rank, world, local_rank, dist):
    import torch

    import jevstral_b200 as jv

    torch.cuda.set_device(local_rank)
    qtype = QTYPE[args.config]
    if rank == 0:
        ensure_model(qtype, args.layers)
    if dist is not None:
        dist.barrier()
    model = jv.Model(model_path(qtype, args.layers), device=local_rank, kv_pool_mb=args.kv_pool_mb)
    ctx = jv.MinistralModel(model, 512)
    stream = torch.cuda.ExternalStream(ctx.stream, device=local_rank)
    try:
        if args.config == "c4":
            return run_decode(args, rank, world, dist, ctx, stream)
        return run_prefill(args, rank, world, local_rank, dist, ctx, stream)
    finally:
        ctx.close()
        model.close()


def run_prefill(args, rank, world, local_rank, dist, ctx, stream):
    import torch

    import jevstral_b200 as jv

    def step(trunk, branches, second=None):
        ctx.kv_cache.reset()
        if branches is None:  # C1: causal prefill, verdict rows of the last position
            v = ctx.forward_selected(trunk, ROWS)[None, :]
        else:
            v = ctx.forward_tree(trunk, branches, ROWS)
        p = jv.decision_probs(jv.margins_from_verdicts(v, 1))
        if second is not None:
            ctx.kv_cache.truncate(len(trunk) - 1)
            v2 = ctx.forward_tree([trunk[-1]], second, ROWS)
            p = jv.decision_probs(jv.margins_from_verdicts(v2, 1))
        return p

    per_step = args.c5_per_step if args.config == "c5" else 1
    timed, shard = timed_items(args.config, args.steps, per_step, world, rank)
    wrng = np.random.default_rng(7000 + rank)
    warm = [c5_decision(wrng) if args.config == "c5" else GEN[args.config](wrng)
            for _ in range(args.warmup * per_step)]
    # size every buffer before the clock starts: the largest item first
    for w in [max(timed, key=toks_of)] + warm:
        step(*w)
    torch.cuda.synchronize()

    tokens = sum(toks_of(w) for w in timed)
    pairs = sum(pairs_of(w) for w in timed)
    n_items = len(timed)
    launches0 = jv.kernel_launches()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        ev0.record(stream)
        results = [step(*w) for w in timed]
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    launches = jv.kernel_launches() - launches0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    # Per-kernel-class device time (roofline.achieved): a sample of the same items once more with
    # CUDA events around every GEMM / attention launch, outside the timed region (the events would
    # serialise launches that otherwise overlap).
    sample = timed[: max(1, min(len(timed), 48 if args.config == "c5" else 20))]
    ctx.profile(True)
    ctx.profile_reset()
    for w in sample:
        step(*w)
    torch.cuda.synchronize()
    prof = {k: ctx.profile_read(k) for k in ("gemm", "attention", "gemv", "other")}
    ctx.profile(False)
    sample_tokens = sum(toks_of(w) for w in sample)

    if dist is not None:
        t = torch.tensor([dev_s, wall], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, wall = t.tolist()
        # the whole job's tokens: ranks may hold different shares (C5 shards by cost)
        tt = torch.tensor([float(tokens), float(n_items), float(launches)], dtype=torch.float64,
                          device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.SUM)
        job_tokens, job_items, job_launches = tt.tolist()
    else:
        job_tokens, job_items, job_launches = float(tokens), float(n_items), float(launches)
    if shard is not None:
        jv.dp.gather_results(dist, rank, world, list(zip(shard, [r.tolist() for r in results])))
    if rank != 0:
        return None

    pk, src = peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
    burst, sustained = pk["bf16_tflops"], pk["bf16_tflops_sustained"]
    decisions = job_items * (2 if args.config == "c3" else 1) if args.config != "c1" else 0
    h2d = sum(4 * (3 * toks_of(w) + 8 * (len(w[1]) if w[1] else 1)) for w in timed) // args.steps
    d2h = sum(4 * len(ROWS) * ((len(w[1]) if w[1] else 1) + (len(w[2]) if len(w) > 2 else 0)) for w in timed) \
        // args.steps
    res = {
        "metric": metric_name(args.config),
        "value": job_tokens / dev_s,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_s / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 (Q8_0/Q5_1/Q4_0 weights decoded to fp16 in shared memory; fp32 accumulate)",
        "data": "synthetic (random-init Ministral-3 3B, N(0,0.02) weights, uniform token ids, seeded)",
        "config": config_block(args.config, args.c5_per_step),
        "parallelism": f"dp{world} (independent replicas, no collective on the data path)",
        "decisions_per_s": (decisions / dev_s) if decisions else None,
        "decisions": int(decisions),
        "tokens_per_s_per_gpu": job_tokens / dev_s / world,
        "linear_tflops": job_tokens * LINEAR_FLOPS_PER_TOKEN * args.layers / 26 / dev_s / 1e12,
        "attention_pairs_per_item": pairs // max(1, n_items),
        "roofline": {"bound": "tensor", "kernel": f"{gemm_kernel_name()} (all four projections)",
                     "achieved": gemm_tflops, "peak": burst, "unit": "TFLOP/s",
                     "frac": gemm_tflops / burst if burst else None,
                     "peak_source": f"{src} bf16 dense burst (each launch is event-timed alone; fp16 runs at the "
                                    f"same rate)",
                     "frac_of_sustained": gemm_tflops / sustained if sustained else None,
                     "traffic": gemm_traffic_per_launch(args.config),
                     "launches": g["launches"], "avg_launch_us": g["ms"] / max(1, g["launches"]) * 1e3,
                     "algorithmic_flops_per_launch": g["flops"] / max(1, g["launches"]),
                     "sample": f"{len(sample)} items of rank 0's timed list ({sample_tokens} tokens)"},
        "kernels": {k: {"ms_per_item": v["ms"] / len(sample), "launches_per_item": v["launches"] / len(sample),
                        "tflops": (v["flops"] / (v["ms"] / 1e3) / 1e12) if v["ms"] and v["flops"] else None,
                        "gbs": (v["bytes"] / (v["ms"] / 1e3) / 1e9) if v["ms"] and v["bytes"] else None}
                    for k, v in prof.items()},
        "e2e": {"value": job_tokens / wall, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": "host wall-clock around the public C-ABI calls (jv_forward_tree / jv_forward_selected) with "
                       "host token buffers in and host verdict logits out"},
        "gpu_launches": int(job_launches),
        "clocks": clocks.summary(),
    }
    return res


def run_decode(args, rank, world, dist, ctx, stream):
    """C4: 1024-token prompt, then greedy decode steps with the full LM head (HBM-bound GEMV)."""
    import torch

    import jevstral_b200 as jv

    steps = args.decode_steps
    rng = np.random.default_rng(1000)
    prompt = [1] + rng.integers(1000, VOCAB, 1023).tolist()
    ctx.prefill(prompt)
    base = ctx.kv_cache.length
    # warm-up: the same call as the timed one (it captures the step graph), then rewind
    for _ in range(max(1, args.warmup)):
        ctx.decode_greedy(1500, steps)
        ctx.kv_cache.truncate(base)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = jv.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(rank) as clocks:
        t0 = time.perf_counter()
        ev0.record(stream)
        toks = ctx.decode_greedy(1500, steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    launches = jv.kernel_launches() - l0
    if dist is not None:
        t = torch.tensor([dev_s, wall], dtype=torch.float64, device=f"cuda:{rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, wall = t.tolist()
    if rank != 0:
        return None
    pk, src = peaks()
    # Algorithmic bytes of one step: every layer matrix and the LM head once (Q4_0: 18 bytes
    # per 32 weights) plus the K/V rows of the visible context (fp16, 106,496 B per position).
    weight_bytes = (LAYER_WEIGHTS * args.layers + VOCAB * 3072) * 18 / 32
    mean_ctx = base + (steps + 1) / 2
    step_bytes = weight_bytes + mean_ctx * 106_496
    gbs = step_bytes * steps / dev_s / 1e9
    return {
        "metric": metric_name("c4"), "value": world * steps / dev_s, "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": max(1, args.warmup), "ms_per_step": dev_s / steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 x int (Q4_0 integers and fp16-split activations in mma.sync, fp32 block scales and sums)",
        "data": "synthetic (random-init Ministral-3 3B, N(0,0.02) weights, uniform token ids, seeded)",
        "config": config_block("c4", 0), "parallelism": f"dp{world}",
        "roofline": {"bound": "hbm", "kernel": "whole decode step (k_dec_gemv x5 per layer + k_dec_attn + head)",
                     "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
                     "traffic": None, "peak_source": f"{src} HBM copy bandwidth",
                     "algorithmic_bytes_per_step": step_bytes},
        "e2e": {"value": world * steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 4 * 8 // max(1, steps) + 4,
                "d2h_bytes_per_step": 4,
                "how": "host wall-clock around jv_decode_greedy (first token in, the chosen tokens out)"},
        "gpu_launches": launches, "clocks": clocks.summary(), "last_tokens": toks[-4:].tolist(),
    }


def gemm_kernel_name() -> str:
    """The prefill GEMM kernel the library runs (JV_GEMM_KERNEL selects another; see gemm_tc.cu)."""
    return {"tmem": "k_gemm_tm"}.get(os.environ.get("JV_GEMM_KERNEL", ""), "k_gemm_tc")


def gemm_traffic_per_launch(config: str):
    """DRAM bytes per GEMM launch from the committed ncu summary of this configuration and kernel."""
    for name in (f"gemm_tc_{config}.md", "gemm_tc_c2.md"):
        f = REPO / "profiles" / name
        if not f.exists():
            continue
        for line in f.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1])
                except ValueError:
                    return None
    return None


def json_stdout():
    """The result line's own handle on the process's standard output. File descriptor 1 then points
    at standard error, so whatever a library writes there on its own (NCCL prints its version banner
    from C when a communicator starts) cannot land beside the one JSON line the driver reads."""
    out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    return out


def main():
    result_out = json_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="c5")
    ap.add_argument("--c5-per-step", type=int, default=24, help="C5: decisions per GPU per step")
    ap.add_argument("--decode-steps", type=int, default=128, help="C4: greedy steps in the timed call")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the C4 decode line added to a 1-GPU C5 run")
    ap.add_argument("--cpu-budget-s", type=float, default=25.0, help="timed CPU work of the cpu_baseline leg")
    ap.add_argument("--ref-budget-s", type=float, default=150.0, help="timed CPU work of --impl reference")
    ap.add_argument("--layers", type=int, default=26, help="fewer layers of the same width (profiling only)")
    ap.add_argument("--kv-pool-mb", type=int, default=4096)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, world)), file=result_out, flush=True)
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
    if rank == 0 and res is not None and world == 1 and args.layers == 26:
        if args.config == "c5" and not args.no_extra:
            # C4, the HBM-bound decode configuration, measured in the same run
            sub = argparse.Namespace(**{**vars(args), "config": "c4"})
            c4 = run_b200(sub, 0, 1, local_rank, None)
            res["extra"] = {"c4": {k: c4[k] for k in ("metric", "value", "unit", "steps", "ms_per_step", "roofline",
                                                      "e2e", "gpu_launches", "clocks", "dtype")}}
        if not args.no_cpu_baseline:
            cb = time_oracle(args.config, model_path(QTYPE[args.config]), args.cpu_budget_s,
                             10**6 if args.config == "c4" else max(1, args.steps))
            res["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0 and res is not None:
        print(json.dumps(res), file=result_out, flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

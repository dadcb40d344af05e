"""Full-depth parity: the 26-layer random-init Ministral-3 3B of BASELINE.json's configurations
(C1 256-token prefill, C2 512 + 5 x 32 tree, C3 4096 + 9 x 48 tree at Q5_1 with a second decision on
the reused trunk pages, C4 1024-token prompt + greedy decode at Q4_0) against the CPU oracle.

Gates: `blk.{l}.output` within 1e-2 relative L2 for every one of the 26
layers; per-option log-odds z_i within 2e-2 absolute with the same argmax; decode logits within
1e-2 relative L2 and every greedy token the oracle's argmax (or within 2e-2 of it: a near tie the
tolerance cannot order). The reference's own gates at depth are ActivationParityTests.cs:41-129
(every layer's tensors of a real checkpoint) and DeciderTests.cs:54-115 (decisions and reuse).

Hidden states come from the activation-capture path (every projection drained whole, each
activation copied out); verdicts and decode logits come from the product path the benchmark
times (split-K halves folded by the next RMSNorm, fused decode kernels in a CUDA graph).
"""
from __future__ import annotations

import numpy as np
import pytest

import jevstral_b200 as jv
from jevstral_b200 import TokenDecider, margins_from_verdicts
from jevstral_b200.synth import MINISTRAL_3B, write_random_gguf
from oracle import binding as ob

pytestmark = pytest.mark.gpu

HIDDEN_TOL = 1e-2   # relative L2 per layer (north star)
Z_TOL = 2e-2        # absolute, per-option log-odds (north star)
VOCAB = MINISTRAL_3B.vocab
LAYERS = MINISTRAL_3B.layers
ROWS = [13059, 2649]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ids(rng, n):
    return rng.integers(1000, VOCAB, n).tolist()


def keep_layer_outputs(d):
    """An activation sink that keeps every layer's output (and the attention/FFN outputs)."""
    def sink(name, arr):
        if name.endswith((".output", ".attn_out", ".ffn_out")) or name == "final_norm":
            d[name] = arr
    return sink


@pytest.fixture(scope="module")
def full_model(tmp_path_factory):
    """The 3B model of BASELINE's configurations, one file per weight type, written once."""
    root = tmp_path_factory.mktemp("full")
    made = {}

    def get(qtype):
        if qtype not in made:
            made[qtype] = write_random_gguf(root / f"ministral3b_{qtype}.gguf", MINISTRAL_3B, qtype, seed=0,
                                            backend="fast")
        return made[qtype]

    yield get
    for p in made.values():
        p.unlink(missing_ok=True)


def check_layers(gpu, cpu):
    errs = {f"blk.{l}.output": rel_l2(gpu[f"blk.{l}.output"], cpu[f"blk.{l}.output"]) for l in range(LAYERS)}
    bad = {k: e for k, e in errs.items() if not e < HIDDEN_TOL}
    assert not bad, (bad, max(errs.values()))
    return max(errs.values())


def check_margins(v_gpu, v_cpu):
    z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
    err = float(np.abs(z_gpu - z_cpu).max())
    assert err < Z_TOL, (err, z_gpu, z_cpu)
    assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu)), (z_gpu, z_cpu)
    return err


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
def test_c1_prefill_every_layer_matches_the_oracle(full_model, qtype):
    """C1: BOS + 255 random ids, causal, empty cache. Every layer's hidden state, the final norm,
    and the last position's verdict logits (the product path's selected head)."""
    path = full_model(qtype)
    rng = np.random.default_rng(1)
    prompt = [1] + ids(rng, 255)
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=1024) as m, jv.MinistralModel(m) as c:
        c.set_activation_sink(keep_layer_outputs(gpu))
        logits_gpu = c.forward(prompt)
        c.set_activation_sink(None)
        c.kv_cache.reset()
        v_gpu = c.forward_selected(prompt, ROWS)
    with ob.OracleModel(path) as o:
        logits = o.forward(prompt, sink=keep_layer_outputs(cpu))
    worst = check_layers(gpu, cpu)
    assert rel_l2(gpu["final_norm"][-1], cpu["final_norm"][-1]) < HIDDEN_TOL
    assert rel_l2(logits_gpu, logits) < HIDDEN_TOL
    v_cpu = logits[ROWS]
    assert np.abs(v_gpu - v_cpu).max() < Z_TOL, (v_gpu, v_cpu, worst)
    print(f"C1 {qtype}: worst layer rel-L2 {worst:.2e}, logits rel-L2 {rel_l2(logits_gpu, logits):.2e}, "
          f"verdict |d| {np.abs(v_gpu - v_cpu).max():.2e}")


def test_c2_tree_decision_matches_the_oracle(full_model):
    """C2: a 512-token trunk and 5 branches of 32 (Q8_0). Every layer's hidden state over all 672
    tokens, and z_i with the same argmax from the product path."""
    path = full_model("Q8_0")
    rng = np.random.default_rng(2)
    trunk = [1] + ids(rng, 511)
    branches = [ids(rng, 32) for _ in range(5)]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=1024) as m, jv.MinistralModel(m) as c:
        c.set_activation_sink(keep_layer_outputs(gpu))
        c.forward_tree(trunk, branches, ROWS)
        c.set_activation_sink(None)
        c.kv_cache.reset()
        v_gpu = c.forward_tree(trunk, branches, ROWS)
    with ob.OracleModel(path) as o:
        v_cpu = o.forward_tree(trunk, branches, ROWS, sink=keep_layer_outputs(cpu))
    worst = check_layers(gpu, cpu)
    err = check_margins(v_gpu, v_cpu)
    print(f"C2: worst layer rel-L2 {worst:.2e}, max |dz| {err:.2e}")


def test_c3_long_trunk_and_reused_trunk_match_the_oracle(full_model):
    """C3 (Q5_1): a 4096-token trunk and 9 branches of 48, then a second decision on the same
    trunk. The decider keeps the trunk's pages and re-runs only its last token (the never-empty
    trunk rule, JevstralDecider.cs:287-289) before 9 fresh branches. Both decisions' z_i against
    the oracle, which reuses its own cache the same way."""
    path = full_model("Q5_1")
    rng = np.random.default_rng(3)
    trunk = [1] + ids(rng, 4095)
    b1 = [ids(rng, 48) for _ in range(9)]
    b2 = [ids(rng, 48) for _ in range(9)]
    with jv.Model(path, kv_pool_mb=2048) as m, jv.MinistralModel(m, 4608) as c:
        d = TokenDecider(c, [ROWS[0]], [ROWS[1]])
        r1 = d.decide(trunk, b1)
        r2 = d.decide(trunk, b2)
        assert r1.cached_tokens == 0 and r2.cached_tokens == len(trunk) - 1
    with ob.OracleModel(path, 4608) as o:
        v1 = o.forward_tree(trunk, b1, ROWS)
        o.kv_truncate(len(trunk) - 1)
        v2 = o.forward_tree(trunk[-1:], b2, ROWS)
    for got, v_cpu in ((r1, v1), (r2, v2)):
        z_cpu = margins_from_verdicts(v_cpu, 1)
        err = float(np.abs(got.margins - z_cpu).max())
        assert err < Z_TOL, (err, got.margins, z_cpu)
        assert int(np.argmax(got.margins)) == int(np.argmax(z_cpu))
        print(f"C3 decision (cached {got.cached_tokens}): max |dz| {err:.2e}")


def test_c4_greedy_decode_matches_the_oracle(full_model):
    """C4 (Q4_0): a 1024-token prompt, then 16 greedy steps of the device-resident decode loop
    (jv_decode_greedy, full LM head + argmax on the device). The oracle replays the same tokens:
    each chosen token must be its argmax, or within 2e-2 of its maximum logit. Then the same steps
    one call at a time (jv_forward, single token): full logits within 1e-2 relative L2."""
    path = full_model("Q4_0")
    rng = np.random.default_rng(4)
    prompt = [1] + ids(rng, 1023)
    first, steps = 1500, 16
    with jv.Model(path, kv_pool_mb=1024) as m, jv.MinistralModel(m, 1280) as c:
        c.prefill(prompt)
        chosen = c.decode_greedy(first, steps).tolist()
        c.kv_cache.truncate(len(prompt))
        fed = [first] + chosen[:-1]
        logits_gpu = [c.forward([t]) for t in fed]
    worst = 0.0
    with ob.OracleModel(path, 1280) as o:
        o.forward(prompt, logits=False)
        for step, (t, want_tok, lg) in enumerate(zip(fed, chosen, logits_gpu)):
            lo = o.forward([t])
            worst = max(worst, rel_l2(lg, lo))
            assert rel_l2(lg, lo) < HIDDEN_TOL, step
            top = int(np.argmax(lo))
            assert top == want_tok or lo[top] - lo[want_tok] < Z_TOL, (step, top, want_tok, lo[top] - lo[want_tok])
            assert int(np.argmax(lg)) == want_tok, step  # the loop and the single-token call agree
    print(f"C4: {steps} greedy steps, worst logits rel-L2 {worst:.2e}, tokens {chosen}")

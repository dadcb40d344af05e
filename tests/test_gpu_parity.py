"""Parity of the B200 path with the CPU oracle, through the C ABI (libjv.so).

Gates: dequantization bit-exact; per-layer hidden states within
1e-2 relative L2; per-option log-odds z_i within 2e-2 absolute with the same argmax.
Self-consistency gates from the reference's own suites: a branch is bit-identical to the
same continuation run alone (DeciderTests.cs:54-91) and a cached prefix is bit-identical
to running the prompt whole (SystemPromptCacheTests.cs:41-68).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import jevstral_b200 as jv
from jevstral_b200 import margins_from_verdicts
from oracle import binding as ob
from small_model import SMALL_CFG, SMALL_PROMPT, VERDICT_ROWS, WIDE_CFG

pytestmark = pytest.mark.gpu

HIDDEN_TOL = 1e-2   # relative L2 per layer (north star)
Z_TOL = 2e-2        # absolute, per-option log-odds (north star)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def toks(n, seed, vocab=16384):
    return np.random.default_rng(seed).integers(1000, vocab, n).tolist()


def capture_into(d):
    return lambda name, arr: d.__setitem__(name, arr)


@pytest.fixture(scope="module")
def small(small_gguf):
    m = jv.Model(small_gguf, kv_pool_mb=256)
    yield m
    m.close()


def ctx(model, cap=512):
    return jv.MinistralModel(model, cap)


# ------------------------------------------------------------------ dequant


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0", "Q4_1", "Q5_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_embedding_gather_is_bit_exact(model_factory, qtype):
    """GatherRows decodes rows bit-exactly (d*q, d*(n-8), d*q5+m; no FMA), the K-quants and the
    other affine formats through the affine layout (a*q + c per 16 weights)."""
    path = model_factory(SMALL_CFG, qtype, seed=3)
    prompt = [1] + toks(30, 5)
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c:
        c.set_activation_sink(capture_into(gpu))
        c.forward(prompt)
    with ob.OracleModel(path) as o:
        o.forward(prompt, sink=capture_into(cpu))
    assert gpu["embeddings"].view(np.uint32).tobytes() == cpu["embeddings"].view(np.uint32).tobytes()


# ------------------------------------------------------------- forward parity


def test_causal_forward_matches_the_reference_numpy_golden(small, golden_small):
    """Per-layer outputs against the reference's own NumPy model (committed golden)."""
    caps = {}
    with ctx(small) as c:
        c.set_activation_sink(capture_into(caps))
        logits = c.forward(SMALL_PROMPT)
    for l in range(SMALL_CFG.layers):
        key = f"blk.{l}.output"
        assert rel_l2(caps[key], golden_small["cap/" + key]) < HIDDEN_TOL, key
    assert rel_l2(logits, golden_small["logits"]) < HIDDEN_TOL
    assert int(np.argmax(logits)) == int(np.argmax(golden_small["logits"]))


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
def test_tree_decision_matches_the_oracle(model_factory, qtype):
    """A ForwardTreeAsync decision: per-layer hidden states and z_i against the oracle."""
    path = model_factory(SMALL_CFG, qtype, seed=11)
    trunk = [1] + toks(70, 21)
    branches = [toks(n, 30 + i) for i, n in enumerate((12, 7, 20, 3, 16))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c:
        c.set_activation_sink(capture_into(gpu))
        v_gpu = c.forward_tree(trunk, branches, VERDICT_ROWS)
    with ob.OracleModel(path) as o:
        v_cpu = o.forward_tree(trunk, branches, VERDICT_ROWS, sink=capture_into(cpu))
    for l in range(SMALL_CFG.layers):
        assert rel_l2(gpu[f"blk.{l}.output"], cpu[f"blk.{l}.output"]) < HIDDEN_TOL
    z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
    assert np.abs(z_gpu - z_cpu).max() < Z_TOL
    assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu))


def test_repeated_short_prefills_are_bit_identical_from_the_first_call(model_factory):
    """The first forward on a freshly loaded model and forty more after it give the same logits.
    The first call allocates the context's buffers (a zeroing memset left pending on the legacy
    stream once wiped what the first call's kernels had written); 91 full-width tokens are one
    token tile of 96, so every GEMM launch is short, one work unit per CTA."""
    path = model_factory(WIDE_CFG, "Q8_0", seed=31)
    prompt = [1] + toks(90, 71)
    with jv.Model(path, kv_pool_mb=256) as m, ctx(m) as c:
        first = c.forward(prompt)
        for i in range(40):
            c.kv_cache.reset()
            again = c.forward(prompt)
            assert again.tobytes() == first.tobytes(), i
        assert np.isfinite(first).all()


@pytest.mark.parametrize("entry", ["forward_tree", "forward_selected", "decode_greedy"])
def test_the_first_call_on_a_fresh_model_matches_the_second(model_factory, entry):
    """Every public entry point's first call on a freshly loaded model (which allocates the
    context's buffers) gives the same bits as the same call repeated on the reset cache."""
    path = model_factory(WIDE_CFG, "Q8_0", seed=32)
    trunk = [1] + toks(150, 81)
    branches = [toks(n, 90 + i) for i, n in enumerate((20, 7, 33))]

    def call(c):
        if entry == "forward_tree":
            return np.asarray(c.forward_tree(trunk, branches, VERDICT_ROWS))
        if entry == "forward_selected":
            return np.asarray(c.forward_selected(trunk, VERDICT_ROWS))
        c.prefill(trunk)
        return np.asarray(c.decode_greedy(1500, 8))

    with jv.Model(path, kv_pool_mb=256) as m, ctx(m) as c:
        first = call(c)
        c.kv_cache.reset()
        second = call(c)
    assert first.tobytes() == second.tobytes(), (first, second)


def test_odd_row_tile_counts_match_the_oracle(model_factory):
    """A width of 384 leaves the O and down projections three 128-row tiles each (and one head per
    KV head group of four): per-layer hidden states (activation capture) and the product path's
    verdicts against the oracle."""
    from jevstral_b200.synth import SynthConfig

    cfg = SynthConfig(layers=2, hidden=384, heads=4, kv_heads=1, head_dim=128, ff=512, vocab=16384)
    path = model_factory(cfg, "Q8_0", seed=23)
    trunk = [1] + toks(90, 41)
    branches = [toks(n, 50 + i) for i, n in enumerate((14, 5, 23))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c:
        c.set_activation_sink(capture_into(gpu))
        c.forward_tree(trunk, branches, VERDICT_ROWS)
        c.set_activation_sink(None)
        c.kv_cache.reset()
        v_gpu = c.forward_tree(trunk, branches, VERDICT_ROWS)
    with ob.OracleModel(path) as o:
        v_cpu = o.forward_tree(trunk, branches, VERDICT_ROWS, sink=capture_into(cpu))
    for l in range(cfg.layers):
        assert rel_l2(gpu[f"blk.{l}.output"], cpu[f"blk.{l}.output"]) < HIDDEN_TOL, l
    z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
    assert np.abs(z_gpu - z_cpu).max() < Z_TOL
    assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu))


@pytest.mark.parametrize("qtype", ["Q4_K", "Q6_K", "Q2_K", "Q5_K"])
def test_k_quant_tree_decision_matches_the_oracle(model_factory, qtype):
    """The K-quant formats (Dequantizer.cs:323-471) on the tensor-core path: weights converted on
    load to the affine layout and decoded to fp16 in the GEMM; per-layer hidden states and z_i
    against the oracle."""
    path = model_factory(SMALL_CFG, qtype, seed=11)
    trunk = [1] + toks(70, 21)
    branches = [toks(n, 30 + i) for i, n in enumerate((12, 7, 20, 3, 16))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c:
        assert m.config.weight_type == {"Q4_K": 12, "Q6_K": 14, "Q2_K": 10, "Q5_K": 13}[qtype]
        c.set_activation_sink(capture_into(gpu))
        c.forward_tree(trunk, branches, VERDICT_ROWS)
        c.set_activation_sink(None)
        c.kv_cache.reset()
        v_gpu = c.forward_tree(trunk, branches, VERDICT_ROWS)
    with ob.OracleModel(path) as o:
        v_cpu = o.forward_tree(trunk, branches, VERDICT_ROWS, sink=capture_into(cpu))
    for l in range(SMALL_CFG.layers):
        assert rel_l2(gpu[f"blk.{l}.output"], cpu[f"blk.{l}.output"]) < HIDDEN_TOL
    z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
    assert np.abs(z_gpu - z_cpu).max() < Z_TOL
    assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu))


def test_mixed_k_quant_checkpoint_at_full_width_matches_the_oracle(model_factory):
    """A "Q4_K_M"-style file at every real matrix shape: Q4_K everywhere but attn_v and ffn_down in
    Q6_K, so the fused QKV matrix mixes two formats. Tree decision (hidden states, z_i), then
    single-token steps (the step-by-step decode path these files take) and the greedy loop."""
    from jevstral_b200.synth import SynthConfig

    mix = (("attn_v.weight", "Q6_K"), ("ffn_down.weight", "Q6_K"))
    cfg = SynthConfig(layers=2, vocab=16384, type_overrides=mix)
    path = model_factory(cfg, "Q4_K", seed=5)
    trunk = [1] + toks(190, 7)
    branches = [toks(n, 40 + i) for i, n in enumerate((32, 17, 48))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=512) as m, ctx(m) as c, ob.OracleModel(path) as o:
        c.set_activation_sink(capture_into(gpu))
        v_gpu = c.forward_tree(trunk, branches, VERDICT_ROWS)
        v_cpu = o.forward_tree(trunk, branches, VERDICT_ROWS, sink=capture_into(cpu))
        for key in [f"blk.{l}.{n}" for l in range(cfg.layers) for n in ("attn_out", "ffn_out", "output")]:
            assert rel_l2(gpu[key], cpu[key]) < HIDDEN_TOL, key
        z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
        assert np.abs(z_gpu - z_cpu).max() < Z_TOL
        assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu))
        c.set_activation_sink(None)
        c.kv_cache.reset()
        o.kv_reset()
        prompt = [1] + toks(60, 9)
        c.prefill(prompt)
        o.forward(prompt, logits=False)
        nxt = 2000
        for step in range(3):
            lg = c.forward([nxt])
            lo = o.forward([nxt])
            assert rel_l2(lg, lo) < HIDDEN_TOL, step
            nxt = int(np.argmax(lo))
        base = c.kv_cache.length
        got = c.decode_greedy(1500, 4)
        c.kv_cache.truncate(base)
        want, tok = [], 1500
        for _ in range(4):
            tok = int(np.argmax(c.forward([tok])))
            want.append(tok)
        assert got.tolist() == want


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
def test_full_width_tree_matches_the_oracle(model_factory, qtype):
    """Every real matrix shape of Ministral-3 3B (two layers): tree decision parity."""
    path = model_factory(WIDE_CFG, qtype, seed=5)
    trunk = [1] + toks(190, 7)
    branches = [toks(n, 40 + i) for i, n in enumerate((32, 17, 48))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=512) as m, ctx(m) as c:
        c.set_activation_sink(capture_into(gpu))
        v_gpu = c.forward_tree(trunk, branches, VERDICT_ROWS)
    with ob.OracleModel(path) as o:
        v_cpu = o.forward_tree(trunk, branches, VERDICT_ROWS, sink=capture_into(cpu))
    for key in [f"blk.{l}.{n}" for l in range(WIDE_CFG.layers) for n in ("attn_out", "ffn_out", "output")]:
        assert rel_l2(gpu[key], cpu[key]) < HIDDEN_TOL, key
    z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(v_cpu, 1)
    assert np.abs(z_gpu - z_cpu).max() < Z_TOL
    assert int(np.argmax(z_gpu)) == int(np.argmax(z_cpu))


@pytest.mark.parametrize("window", [16384, 64])
def test_yarn_rope_and_query_temperature_match_the_oracle(model_factory, window):
    """The real checkpoint's RoPE scaling (YaRN factor 16, beta 32/1, magnitude scale 1) and the
    llama-4 query temperature q *= 1 + 0.1 ln(1 + floor(pos / window)) (Rope.cs:33-106,
    MinistralModel.cs:676-682). With the 16384 window the prompt stays inside it (the YaRN table
    alone); with a 64-token window a 300-token prompt crosses four interval boundaries, and the tree
    branches and single-token steps after it run at positions 300-330. Every layer's rotated q and
    k and output, the logits, the branch verdicts and the decode logits against the oracle."""
    from jevstral_b200.synth import SynthConfig, yarn_metadata

    cfg = SynthConfig(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=16384,
                      extra=yarn_metadata(original_context=window))
    path = model_factory(cfg, "Q8_0", seed=14)
    prompt = [1] + toks(299, 61)
    branches = [toks(n, 62 + i) for i, n in enumerate((9, 4, 17))]
    gpu, cpu = {}, {}
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c, ob.OracleModel(path) as o:
        assert m.config.yarn_active and m.config.rope_mscale == 1.0
        assert abs(m.config.temperature_scale - 0.1) < 1e-7 and m.config.rope_orig_ctx == window
        c.set_activation_sink(capture_into(gpu))
        lg = c.forward(prompt)
        lo = o.forward(prompt, sink=capture_into(cpu))
        for l in range(cfg.layers):
            for n in ("q_rope", "k_rope", "output"):
                key = f"blk.{l}.{n}"
                assert rel_l2(gpu[key], cpu[key]) < HIDDEN_TOL, key
        assert rel_l2(lg, lo) < HIDDEN_TOL
        c.set_activation_sink(None)
        c.kv_cache.truncate(len(prompt) - 1)
        o.kv_truncate(len(prompt) - 1)
        v_gpu = c.forward_tree([prompt[-1]], branches, VERDICT_ROWS)
        o_v = o.forward_tree([prompt[-1]], branches, VERDICT_ROWS)
        z_gpu, z_cpu = margins_from_verdicts(v_gpu, 1), margins_from_verdicts(o_v, 1)
        assert np.abs(z_gpu - z_cpu).max() < Z_TOL
        c.kv_cache.truncate(len(prompt))
        o.kv_truncate(len(prompt))
        nxt = int(np.argmax(lo))
        for step in range(3):  # the fused single-token kernels apply the temperature on the device
            lg = c.forward([nxt])
            lo = o.forward([nxt])
            assert rel_l2(lg, lo) < HIDDEN_TOL, step
            nxt = int(np.argmax(lo))


def test_decode_steps_match_the_oracle(small):
    """Single-token forwards (the decode GEMV path) with the full LM head."""
    prompt = [1] + toks(40, 9)
    with ctx(small) as c, ob.OracleModel(small.path) as o:
        lg = c.forward(prompt)
        lo = o.forward(prompt)
        assert rel_l2(lg, lo) < HIDDEN_TOL
        nxt = int(np.argmax(lo))
        for step in range(4):
            lg = c.forward([nxt])
            lo = o.forward([nxt])
            assert rel_l2(lg, lo) < HIDDEN_TOL, step
            nxt = int(np.argmax(lo))


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
def test_full_width_decode_steps_match_the_oracle(model_factory, qtype):
    """The fused single-token kernels on every real matrix shape: logits of decode steps."""
    path = model_factory(WIDE_CFG, qtype, seed=8)
    prompt = [1] + toks(90, 4)
    with jv.Model(path, kv_pool_mb=512) as m, ctx(m) as c, ob.OracleModel(path) as o:
        c.prefill(prompt)
        o.forward(prompt, logits=False)
        nxt = 2000
        for step in range(3):
            lg = c.forward([nxt])
            lo = o.forward([nxt])
            assert rel_l2(lg, lo) < HIDDEN_TOL, step
            assert int(np.argmax(lg)) == int(np.argmax(lo)), step
            nxt = int(np.argmax(lo))


def test_decode_greedy_follows_its_own_argmax(small):
    prompt = [1] + toks(20, 19)
    with ctx(small) as a, ctx(small) as b:
        a.prefill(prompt)
        got = a.decode_greedy(1500, 5)
        b.prefill(prompt)
        want, tok = [], 1500
        for _ in range(5):
            tok = int(np.argmax(b.forward([tok])))
            want.append(tok)
        assert got.tolist() == want


# -------------------------------------------------------- bit-identity gates


def test_branches_match_running_each_continuation_alone(small):
    trunk = [1] + toks(80, 1)
    branches = [toks(n, 10 + i) for i, n in enumerate((5, 19, 33, 2))]
    with ctx(small) as c:
        tree = c.forward_tree(trunk, branches, VERDICT_ROWS)
        for b, br in enumerate(branches):
            c.kv_cache.reset()
            c.prefill(trunk)
            alone = c.forward_selected(br, VERDICT_ROWS)
            assert alone.tobytes() == tree[b].tobytes(), f"branch {b}"


def test_cached_and_uncached_produce_identical_logits(small):
    prompt = [1] + toks(100, 3)
    with ctx(small) as c:
        whole = c.forward(prompt)
        c.kv_cache.reset()
        c.prefill(prompt[:61])
        snap = c.kv_cache.snapshot(61)
        c.kv_cache.reset()
        c.kv_cache.restore(snap, 61)
        cached = c.forward(prompt[61:])
        assert whole.tobytes() == cached.tobytes()
        # zero-copy pages shared with a second context
        c.kv_cache.reset()
        c.prefill(prompt[:61])
        shared = c.kv_cache.share(61)
        with ctx(small) as d:
            d.kv_cache.adopt(shared)
            again = d.forward(prompt[61:])
        shared.release()
        assert whole.tobytes() == again.tobytes()


def test_reusing_the_trunk_for_a_second_decision_is_bit_identical(small):
    """C3's second decision: the trunk stays in the cache; the decider re-runs its last token."""
    from jevstral_b200 import TokenDecider

    prefix = [1] + toks(150, 2)
    b1 = [toks(n, 50 + i) for i, n in enumerate((6, 9, 4))]
    b2 = [toks(n, 60 + i) for i, n in enumerate((8, 3, 12))]
    with ctx(small) as c, ctx(small) as fresh:
        d = TokenDecider(c, [13059], [2649])
        d.decide(prefix, b1)
        r2 = d.decide(prefix, b2)
        assert r2.cached_tokens == len(prefix) - 1
        ref = TokenDecider(fresh, [13059], [2649]).decide(prefix, b2)
        assert r2.margins.tobytes() == ref.margins.tobytes()


def test_system_prompt_snapshot_file_and_the_verdict_scorer_flow(small, tmp_path):
    """SystemPromptCache and VerdictScorer on device pages (SystemPromptCache.cs:51-164,
    VerdictScorer.cs:231-254): capture the system prefix, Save it as an SHKV file straight from the
    pages (byte for byte the reference's format of KvCache.Snapshot), TryLoad it into a fresh
    context, and ForwardSelectedAsync the request: the same bits as an uncached forward of the whole
    prompt. A wrong fingerprint, a missing file and a truncated file are misses that leave the cache
    as it was; the loaded prefix shared zero-copy into another context gives the same bits again
    (the per-request restore without a copy)."""
    import shkv_format as shkv

    system = [1] + toks(70, 81)
    request = toks(25, 82)
    fp = "model.gguf|123|456|mistral3|2x2x128|71:" + "x" * 150  # > 127 bytes: two-byte length prefix
    path = tmp_path / "system.shkv"
    with ctx(small) as a:
        a.prefill(system)
        a.kv_cache.save_shkv(path, fp, system)
        snap = a.kv_cache.snapshot(len(system))
    data = path.read_bytes()
    assert data == shkv.write(fp, system, snap)
    with ctx(small) as whole:
        want = whole.forward_selected(system + request, VERDICT_ROWS)
    with ctx(small) as b:
        b.prefill([1, 2000, 3000])  # a cache the load replaces
        assert b.kv_cache.load_shkv(path, fp) == system
        assert b.kv_cache.length == len(system)
        got = b.forward_selected(request, VERDICT_ROWS)
        assert got.tobytes() == want.tobytes()
        b.kv_cache.truncate(len(system))
        assert b.kv_cache.load_shkv(path, fp + "?") is None
        assert b.kv_cache.load_shkv(tmp_path / "absent.shkv", fp) is None
        (tmp_path / "short.shkv").write_bytes(data[:-100])
        assert b.kv_cache.load_shkv(tmp_path / "short.shkv", fp) is None
        assert b.kv_cache.length == len(system)
        assert np.array_equal(b.kv_cache.snapshot(len(system)), snap)
        shared = b.kv_cache.share(len(system))
        with ctx(small) as c2:
            c2.kv_cache.adopt(shared)
            again = c2.forward_selected(request, VERDICT_ROWS)
        shared.release()
        assert again.tobytes() == want.tobytes()


def test_snapshot_round_trip_and_errors(small):
    with ctx(small) as c:
        c.prefill([1] + toks(70, 4))
        assert c.kv_cache.length == 71
        snap = c.kv_cache.snapshot(70)
        assert snap.size == 2 * SMALL_CFG.layers * SMALL_CFG.kv_heads * 70 * 128
        with pytest.raises(jv.ArgumentOutOfRangeError):
            c.kv_cache.snapshot(72)
        with pytest.raises(jv.ArgumentError):
            c.kv_cache.restore(snap, 71)
        c.kv_cache.reset()
        c.kv_cache.restore(snap, 70)
        assert np.array_equal(c.kv_cache.snapshot(70), snap)


def test_errors_map_to_the_reference_exceptions(small, tmp_path):
    with ctx(small) as c:
        with pytest.raises(jv.ArgumentOutOfRangeError):
            c.forward([1, 16384])
        with pytest.raises(jv.ArgumentError):
            c.forward_tree([1, 2000], [], VERDICT_ROWS)
        with pytest.raises(jv.ArgumentError):
            c.forward_tree([1, 2000], [[1500], []], VERDICT_ROWS)
        flag = np.ones(1, np.int32)
        c.set_cancellation(flag)
        with pytest.raises(jv.OperationCanceledError):
            c.forward([1, 2000, 3000])
        c.set_cancellation(None)
        assert len(c.forward([1, 2000])) == SMALL_CFG.vocab
    with open(small.path, "rb") as f:
        data = f.read()
    short = tmp_path / "short.gguf"
    short.write_bytes(data[: len(data) // 3])
    with pytest.raises(jv.GgufIOError):
        jv.Model(short)


def test_activations_beyond_the_fp16_range_raise_a_numeric_error(model_factory):
    """Norm gains of 1e5 put the RMSNorm output far outside fp16 (|x| >= 65520). The reference
    computes this in fp32; the device path packs its GEMM operands in fp16, so every fp16 writer
    checks its values and the call raises NumericError (ArithmeticException), naming where, instead
    of returning logits built from infinities. Prefill, tree and single-token paths; the context
    stays usable (a second call raises the same way)."""
    from jevstral_b200.synth import SynthConfig

    cfg = SynthConfig(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=16384,
                      norm_gain=1e5)
    path = model_factory(cfg, "Q8_0", seed=15)
    prompt = [1] + toks(40, 71)
    with jv.Model(path, kv_pool_mb=128) as m, ctx(m) as c:
        for _ in range(2):
            c.kv_cache.reset()
            with pytest.raises(jv.NumericError, match="RMSNorm"):
                c.forward(prompt)
        c.kv_cache.reset()
        with pytest.raises(jv.NumericError):
            c.forward_tree(prompt, [[2000, 3000], [4000]], VERDICT_ROWS)
        c.kv_cache.reset()
        with pytest.raises(jv.NumericError):
            c.forward([1])  # the fused single-token kernels
    # a model inside the range is unaffected
    ok = model_factory(SMALL_CFG, "Q8_0", seed=15)
    with jv.Model(ok, kv_pool_mb=128) as m, ctx(m) as c:
        assert np.isfinite(c.forward(prompt)).all()


def test_a_device_wait_that_runs_out_reports_and_leaves_the_context_usable(small):
    """The bounded-wait path of the tensor-core kernels: a wait that nothing completes gives
    up after its bound, the call raises the device-timeout error naming the wait, and the
    next forward on the same context is bit-identical to one before it."""
    prompt = [1] + toks(90, 8)
    with ctx(small) as c:
        before = c.forward(prompt)
        c.kv_cache.reset()
        with pytest.raises(jv.DeviceTimeoutError, match="wait check"):
            c.check_wait_timeout(20_000_000)  # ~10 ms of SM clock
        with pytest.raises(jv.ArgumentOutOfRangeError):
            c.check_wait_timeout(0)
        after = c.forward(prompt)
        assert before.tobytes() == after.tobytes()


def test_tensor_core_gemm_matches_the_reference_gemm(model_factory):
    """The tcgen05 GEMM against a CUDA-core product over the same fp16 operands, at every real
    matrix shape: only the accumulation order differs."""
    path = model_factory(WIDE_CFG, "Q8_0", seed=5)
    code = (
        "import sys, numpy as np; sys.path[:0] = sys.argv[2:];"
        "import jevstral_b200 as jv;"
        "m = jv.Model(sys.argv[1], kv_pool_mb=512); c = jv.MinistralModel(m); caps = {};"
        "c.set_activation_sink(lambda n, a: caps.__setitem__(n, a));"
        "c.forward([1] + list(range(1000, 1300)));"
        "np.savez(sys.stdout.buffer, **{k: v for k, v in caps.items() "
        "if k.endswith(('.v', 'k_rope', 'attn_out', 'ffn_out', 'output'))})"
    )
    import io

    from conftest import REPO

    paths = [str(REPO / "llm-shield_b200"), str(REPO)]
    outs = []
    for ref in (False, True):
        env = dict(os.environ)
        env.pop("JV_GEMM_REFERENCE", None)
        if ref:
            env["JV_GEMM_REFERENCE"] = "1"
        r = subprocess.run([sys.executable, "-c", code, str(path)] + paths, env=env, capture_output=True, timeout=900)
        assert r.returncode == 0, r.stderr.decode()[-2000:]
        outs.append(np.load(io.BytesIO(r.stdout)))
    tc, ref = outs
    # Layer 0's QKV product sees identical operands in both runs: only the accumulation order
    # differs. Later tensors also inherit fp16 re-rounding of slightly different activations
    # (one fp16 ulp is 4.9e-4 relative), hence the looser bound there.
    errs = {k: rel_l2(tc[k], ref[k]) for k in ref.files}
    for k in ("blk.0.v", "blk.0.k_rope"):
        assert errs[k] < 1e-5, (k, errs)
    for k, e in errs.items():
        assert e < 2e-3, (k, errs)


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
def test_gemm_kernels_are_bit_identical(model_factory, qtype):
    """The two prefill GEMM kernels on the same model: k_gemm_tc (the default: decoded weights
    staged in shared memory) and k_gemm_tm (decoded weights in TMEM, JV_GEMM_KERNEL=tmem). The same
    fp16 operands and the same K order, so every captured activation (the capture path's
    counter-combined K split) and the product path's verdict logits (split-K halves folded by
    the next RMSNorm) are the same bits, for a causal prefill of 300 tokens and a tree after it."""
    path = model_factory(WIDE_CFG, qtype, seed=12)
    code = (
        "import sys, numpy as np; sys.path[:0] = sys.argv[2:];"
        "import jevstral_b200 as jv;"
        "m = jv.Model(sys.argv[1], kv_pool_mb=512); c = jv.MinistralModel(m); caps = {};"
        "c.set_activation_sink(lambda n, a: caps.__setitem__(n, a));"
        "c.forward([1] + [(11 * i) % 16000 + 100 for i in range(299)]);"
        "c.set_activation_sink(None); c.kv_cache.reset();"
        "v = c.forward_tree([1] + list(range(2000, 2150)), [[5, 6, 7] * 10, [8] * 37, [9, 10]], [13059, 2649, 40]);"
        "caps['verdicts'] = np.asarray(v, dtype=np.float32);"
        "np.savez(sys.stdout.buffer, **caps)"
    )
    import io

    from conftest import REPO

    paths = [str(REPO / "llm-shield_b200"), str(REPO)]
    outs = {}
    for kernel in ("tc", "tmem"):
        env = dict(os.environ)
        env.pop("JV_GEMM_KERNEL", None)
        if kernel != "tc":
            env["JV_GEMM_KERNEL"] = kernel
        r = subprocess.run([sys.executable, "-c", code, str(path)] + paths, env=env, capture_output=True, timeout=900)
        assert r.returncode == 0, r.stderr.decode()[-2000:]
        outs[kernel] = np.load(io.BytesIO(r.stdout))
    ref = outs["tc"]
    assert len(ref.files) > 20
    for kernel in ("tmem",):
        other = outs[kernel]
        assert set(other.files) == set(ref.files)
        diff = [k for k in ref.files if other[k].tobytes() != ref[k].tobytes()]
        assert not diff, (kernel, {k: rel_l2(other[k], ref[k]) for k in diff})


def test_debug_sync_gives_the_same_bits(model_factory):
    """JV_DEBUG_SYNC=1 (a synchronisation after every programmatic-dependent launch, for naming a
    failing kernel) runs the same kernels without overlap: a full-width tree decision gives the same
    verdict logits, bit for bit, as the default path in this process."""
    path = model_factory(WIDE_CFG, "Q8_0", seed=33)
    trunk = [1] + list(range(3000, 3140))
    branches = [[5, 6, 7] * 9, [8] * 41, [9, 10, 11]]
    code = (
        "import sys, numpy as np; sys.path[:0] = sys.argv[2:];"
        "import jevstral_b200 as jv;"
        "m = jv.Model(sys.argv[1], kv_pool_mb=256); c = jv.MinistralModel(m);"
        f"v = c.forward_tree({trunk!r}, {branches!r}, {VERDICT_ROWS!r});"
        "np.save(sys.stdout.buffer, np.asarray(v, dtype=np.float32))"
    )
    import io

    from conftest import REPO

    env = dict(os.environ, JV_DEBUG_SYNC="1")
    r = subprocess.run([sys.executable, "-c", code, str(path), str(REPO / "llm-shield_b200"), str(REPO)], env=env,
                       capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    synced = np.load(io.BytesIO(r.stdout))
    with jv.Model(path, kv_pool_mb=256) as m, ctx(m) as c:
        want = np.asarray(c.forward_tree(trunk, branches, VERDICT_ROWS), dtype=np.float32)
    assert synced.tobytes() == want.tobytes()


def test_tensor_core_attention_matches_the_mma_sync_attention(model_factory):
    """The tcgen05 prefill attention against the mma.sync one on the same cache: a 1100-token
    causal trunk (nine 128-key blocks, ragged last block) and then a tree over it, per layer."""
    path = model_factory(WIDE_CFG, "Q8_0", seed=6)
    code = (
        "import sys, numpy as np; sys.path[:0] = sys.argv[2:];"
        "import jevstral_b200 as jv;"
        "m = jv.Model(sys.argv[1], kv_pool_mb=512); c = jv.MinistralModel(m); caps = {};"
        "c.set_activation_sink(lambda n, a: caps.__setitem__('t.' + n, a));"
        "trunk = [1] + [(7 * i) % 16000 + 100 for i in range(1099)];"
        "c.forward(trunk);"
        "c.set_activation_sink(lambda n, a: caps.__setitem__('b.' + n, a));"
        "z = c.forward_tree([5, 6, 7], [[11, 12, 13, 14], [21], [31, 32]], [40, 41, 42]);"
        "caps['z'] = np.asarray(z, dtype=np.float32);"
        "np.savez(sys.stdout.buffer, **{k: v for k, v in caps.items() if k == 'z' or k.endswith('attn_weighted')})"
    )
    import io

    from conftest import REPO

    paths = [str(REPO / "llm-shield_b200"), str(REPO)]
    outs = []
    for kernel in ("tc", "mma"):
        env = dict(os.environ)
        env["JV_ATTN_KERNEL"] = kernel
        r = subprocess.run([sys.executable, "-c", code, str(path)] + paths, env=env, capture_output=True, timeout=900)
        assert r.returncode == 0, r.stderr.decode()[-2000:]
        outs.append(np.load(io.BytesIO(r.stdout)))
    tc, mma = outs
    # Layer 0 sees identical Q/K/V in both runs (exp rounding and summation order differ);
    # later layers also inherit fp16 re-rounding of slightly different activations.
    errs = {k: rel_l2(tc[k], mma[k]) for k in mma.files if k != "z"}
    assert len(errs) == 2 * WIDE_CFG.layers
    for k in ("t.blk.0.attn_weighted", "b.blk.0.attn_weighted"):
        assert errs[k] < 2e-3, (k, errs)
    for k, e in errs.items():
        assert e < 1e-2, (k, errs)
    assert np.abs(tc["z"] - mma["z"]).max() < 2e-2


def test_batched_rows_match_the_oracle(small):
    """ForwardRowsAsync (MinistralModel.cs:282-294, TokenLayout.Rows :758-780): rows that each
    append to their own KV region after a shared prefix, stepped together as ReasoningDecider's
    batched decode does. Full-vocabulary logits of every row's last token against the oracle for
    a first multi-token step and a one-token-per-row step; a row gives bit-identical logits in a
    four-row and a two-row pass (the head stays a GEMM from two rows up)."""
    prefix = [1] + toks(40, 21)
    p = len(prefix)
    bases = [p + 64 * r for r in range(4)]
    first = [toks(n, 30 + r) for r, n in enumerate((3, 1, 6, 2))]
    lengths = [len(f) for f in first]
    with ctx(small) as c, ctx(small) as d, ob.OracleModel(small.path) as o:
        c.prefill(prefix)
        o.forward(prefix, logits=False)
        got = c.forward_rows(p, bases, [0] * 4, first)
        want = o.forward_rows(p, bases, [0] * 4, first)
        assert got.shape == want.shape == (4, SMALL_CFG.vocab)
        for r in range(4):
            assert rel_l2(got[r], want[r]) < HIDDEN_TOL, r
            assert int(np.argmax(got[r])) == int(np.argmax(want[r])), r
        nxt = [[int(np.argmax(want[r]))] for r in range(4)]
        got2 = c.forward_rows(p, bases, lengths, nxt)
        want2 = o.forward_rows(p, bases, lengths, nxt)
        for r in range(4):
            assert rel_l2(got2[r], want2[r]) < HIDDEN_TOL, r
            assert int(np.argmax(got2[r])) == int(np.argmax(want2[r])), r
        # rows 2 and 0 in a pass of their own: the same bits as in the four-row pass
        d.prefill(prefix)
        two = d.forward_rows(p, [bases[2], bases[0]], [0, 0], [first[2], first[0]])
        assert two[0].tobytes() == got[2].tobytes()
        assert two[1].tobytes() == got[0].tobytes()


def test_tree_logits_match_the_oracle(small):
    """ForwardTreeLogitsAsync (MinistralModel.cs:227-255): full-vocabulary logits at every branch
    token, each against the oracle's logits for the trunk followed by that branch prefix."""
    trunk = [1] + toks(30, 23)
    branches = [toks(n, 40 + i) for i, n in enumerate((3, 1, 4))]
    with ctx(small) as c, ob.OracleModel(small.path) as o:
        got = c.forward_tree_logits(trunk, branches)
        assert [len(g) for g in got] == [len(b) for b in branches]
        for b, br in enumerate(branches):
            for i in range(len(br)):
                o.kv_reset()
                want = o.forward_tree(trunk, [br[: i + 1]], None)[0]
                assert rel_l2(got[b][i], want) < HIDDEN_TOL, (b, i)
                assert int(np.argmax(got[b][i])) == int(np.argmax(want)), (b, i)


def test_long_tree_logits_are_bit_identical_to_each_branch_alone(small):
    """Full-vocabulary logits at 600 branch tokens: the head GEMM runs three token tiles over the
    128 row tiles of the 16384-row head, so many CTAs take three work units of four k steps each
    (the decoder warps then drain the last of several short units). Every branch's logits equal
    the same branch run alone after the trunk, bit for bit."""
    trunk = [1] + toks(39, 61)
    branches = [toks(n, 70 + i) for i, n in enumerate((200, 150, 250))]
    with ctx(small, cap=2048) as c:
        got = c.forward_tree_logits(trunk, branches)
        for b, br in enumerate(branches):
            c.kv_cache.reset()
            alone = c.forward_tree_logits(trunk, [br])[0]
            assert np.asarray(got[b]).tobytes() == np.asarray(alone).tobytes(), b
            assert np.isfinite(np.asarray(alone)).all()


def test_decision_batch_is_bit_identical_to_single_decisions(small):
    """jv_decide_batch: each decision of a batch (trunks of different lengths, branches of odd
    lengths so segments start off multiples of 8, one decision without a trunk) gives exactly the
    logits it gives alone on an empty cache, and the cache is left as it was."""
    rng = np.random.default_rng(77)
    decisions = []
    for trunk_len, blens in [(37, [5, 11]), (130, [3, 9, 17]), (0, [4]), (300, [33, 1, 7, 40]), (64, [32, 32])]:
        trunk = ([1] + toks(trunk_len - 1, int(rng.integers(1 << 30)))) if trunk_len else []
        decisions.append((trunk, [toks(n, int(rng.integers(1 << 30))) for n in blens]))
    with ctx(small, cap=2048) as c:
        c.forward([1] + toks(20, 5))  # something in the cache that the batch must neither see nor disturb
        before = c.cached_token_count
        got = c.decide_batch(decisions, VERDICT_ROWS)
        assert c.cached_token_count == before
    for (trunk, branches), g in zip(decisions, got):
        with ctx(small, cap=2048) as c:
            want = c.forward_tree(trunk, branches, VERDICT_ROWS)
        assert np.array_equal(g, want)


def test_long_context_prefill_matches_the_decode_path(small):
    """A prefill past ~28.6K visible keys, where the tensor-core attention reads the page table from
    global memory instead of its staged copy: the last position's logits against prefilling all but
    the last token and running that one through the single-token path (a separate attention kernel)."""
    n = 29_500
    tokens = [1] + toks(n - 1, 21)
    with ctx(small, cap=n + 8) as c1:
        full = c1.forward(tokens)
    with ctx(small, cap=n + 8) as c2:
        c2.prefill(tokens[:-1])
        last = c2.forward([tokens[-1]])
    assert rel_l2(full, last) < HIDDEN_TOL
    assert int(np.argmax(full)) == int(np.argmax(last))


def test_kernel_launches_are_counted(small):
    before = jv.kernel_launches()
    with ctx(small) as c:
        c.forward_tree([1, 1500, 2500], [[3000, 4000], [5000]], VERDICT_ROWS)
    assert jv.kernel_launches() - before >= 7 * SMALL_CFG.layers


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1", "Q4_0"])
@pytest.mark.parametrize("rows,cols", [(128, 256), (3072, 3072), (1024, 9216)])
def test_quant_matvec_matches_the_oracle(qtype, rows, cols):
    """jv_qmatvec (QuantMatMul.ForwardAsync, one token) against the oracle's RunRowsFloat."""
    import torch

    from jevstral_b200 import quant
    from jevstral_b200.synth import synth_normal, synth_quantize

    w = synth_normal(7, rows, rows * cols, 0.02)
    raw = synth_quantize(w, qtype)
    x = np.random.default_rng(rows + cols).uniform(-2, 2, cols).astype(np.float32)
    dev = torch.device("cuda:0")
    d_raw = torch.from_numpy(raw).to(dev)
    d_tiled = torch.empty(quant.qweight_bytes(qtype, rows, cols), dtype=torch.uint8, device=dev)
    d_x = torch.from_numpy(x).to(dev)
    d_y = torch.empty(rows, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    quant.qweight_pack(qtype, d_raw.data_ptr(), rows, cols, d_tiled.data_ptr())
    quant.qmatvec(qtype, d_tiled.data_ptr(), rows, cols, d_x.data_ptr(), d_y.data_ptr())
    torch.cuda.synchronize()
    want = ob.matmul(quant.TYPE_IDS[qtype], raw, rows, cols, x, 1)[0]
    got = d_y.cpu().numpy()
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert err.max() < 1e-5, err.max()

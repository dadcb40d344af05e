"""The CPU oracle pinned against the reference's golden vectors and kernel definitions.

Restates the reference's xunit suites (tests/Jevstral.Tests/DequantizerParityTests.cs,
KernelTests.cs, PanelGemmTests.cs, AttentionKernelTests.cs, RopeAndCacheTests.cs,
DeciderTests.cs, SystemPromptCacheTests.cs) against oracle/jv_oracle.cpp.
"""
from __future__ import annotations

import base64
import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import binding as ob
from small_model import SMALL_PROMPT, VERDICT_ROWS

TYPE_IDS = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11,
            "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
GEOMETRY = {"Q4_0": (32, 18), "Q4_1": (32, 20), "Q5_0": (32, 22), "Q5_1": (32, 24), "Q8_0": (32, 34), "F32": (1, 4),
            "F16": (1, 2), "Q2_K": (256, 84), "Q3_K": (256, 110), "Q4_K": (256, 144), "Q5_K": (256, 176),
            "Q6_K": (256, 210)}


def close(expected, actual, rel, what=""):
    """Numeric.Close (tests/Jevstral.Tests/Numeric.cs:14-41): relative to max(1, |expected|)."""
    e = np.asarray(expected, dtype=np.float64)
    a = np.asarray(actual, dtype=np.float64)
    err = np.abs(a - e) / np.maximum(1.0, np.abs(e))
    assert err.max(initial=0.0) <= rel, f"{what}: worst relative error {err.max():.3e} > {rel:.0e}"


def kat_cases():
    return json.loads((GOLDEN / "quant_kat.json").read_text())["cases"]


# --------------------------------------------------------------------- dequant


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c["type"])
def test_dequantize_matches_the_reference_fixture_bit_exactly(case):
    """DequantizerParityTests.Dequantize_MatchesReference (:39-84), tightened to bit equality."""
    bs, ts = GEOMETRY[case["type"]]
    assert (case["block_size"], case["type_size"]) == (bs, ts)
    compared = 0
    for kind in ("quantized", "synthetic"):
        if kind not in case:
            continue
        raw = np.frombuffer(base64.b64decode(case[kind]["bytes"]), dtype=np.uint8)
        expected = np.asarray(case[kind]["expected"], dtype=np.float32)
        got = ob.dequantize(TYPE_IDS[case["type"]], raw, expected.size)
        assert got.view(np.uint32).tolist() == expected.view(np.uint32).tolist(), f"{case['type']} {kind}"
        compared += 1
    assert compared > 0


def test_dequantize_rejects_partial_blocks():
    """DequantizerParityTests.RejectsPartialBlocks (:146-152)."""
    with pytest.raises(ob.OracleError):
        ob.dequantize(8, np.zeros(34, np.uint8), 31)


def test_row_bytes_rejects_unaligned_rows():
    """DequantizerParityTests.RowBytesRejectsUnalignedRows (:154-160)."""
    assert ob.lib.orc_row_bytes(8, 64) == 68
    assert ob.lib.orc_row_bytes(8, 33) == -1


# ------------------------------------------------------------------ kernels

LENGTHS = [1, 2, 3, 7, 8, 15, 16, 17, 31, 33, 64, 127, 3072, 9216]  # KernelTests.cs:26


def rand(n, seed, lo=-2.0, hi=2.0):
    return np.random.default_rng(seed).uniform(lo, hi, n).astype(np.float32)


@pytest.mark.parametrize("n", LENGTHS)
def test_rmsnorm_matches_the_definition(n):
    x, w = rand(n, 7), rand(n, 11)
    mean = np.sum(x.astype(np.float64) ** 2) / n
    scale = np.float32(1.0) / np.sqrt(np.float32(mean) + np.float32(1e-5))
    close(x * scale * w, ob.rmsnorm(x, w), 1e-5, f"rmsnorm({n})")


@pytest.mark.parametrize("n", LENGTHS)
def test_softmax_sums_to_one_and_is_shift_invariant(n):
    x = rand(n, 7)
    a = ob.softmax(x)
    close(1.0, a.sum(dtype=np.float64), 1e-5, "softmax total")
    assert ((a >= 0) & (a <= 1)).all()
    close(a, ob.softmax(x + np.float32(13.5)), 1e-5, "shift invariance")


@pytest.mark.parametrize("n", LENGTHS)
def test_swiglu_matches_the_definition(n):
    g, u = rand(n, 7), rand(n, 23)
    close(g / (1 + np.exp(-g)) * u, ob.swiglu(g, u), 1e-5, f"swiglu({n})")


@pytest.mark.parametrize("magnitude", [50.0, 95.0, 400.0])
def test_softmax_survives_large_logits(magnitude):
    """KernelTests.SoftmaxSurvivesLargeLogits (:112-135)."""
    x = (magnitude * np.arange(64) / 63).astype(np.float32)
    a = ob.softmax(x)
    assert np.isfinite(a).all() and a.argmax() == 63
    e = np.exp(x.astype(np.float64) - magnitude)
    close(e / e.sum(), a, 1e-5, "p")


def test_softmax_of_all_masked_positions_stays_finite():
    a = ob.softmax(np.full(8, -np.inf, np.float32))
    assert not np.isnan(a).any()


def naive(w, x):
    return (x.astype(np.float64) @ w.astype(np.float64).T)


@pytest.mark.parametrize("tokens", [1, 5, 400])
def test_quant_matmul_matches_naive_product(tokens):
    """KernelTests.QuantMatMulMatchesNaiveProduct (:152-178) — F32 weights, 64-row tiles."""
    rows, cols = 64, 64
    w, x = rand(rows * cols, 31).reshape(rows, cols), rand(tokens * cols, 41).reshape(tokens, cols)
    y = ob.matmul(0, w.view(np.uint8), rows, cols, x, tokens)
    close(naive(w, x), y, 1e-5, "C")


@pytest.mark.parametrize("rows,cols,tokens", [(128, 256, 1), (64, 3072, 5), (128, 3072, 13), (64, 4096, 6),
                                              (64, 9216, 7)])
def test_panel_gemm_matches_the_definition(rows, cols, tokens):
    """PanelGemmTests.MatchesTheDefinition (:38-59)."""
    w = rand(rows * cols, 1, -1, 1).reshape(rows, cols)
    x = rand(tokens * cols, 2, -1, 1).reshape(tokens, cols)
    close(naive(w, x), ob.matmul(0, w.view(np.uint8), rows, cols, x, tokens), 1e-4, "panel")


def test_a_tokens_result_does_not_depend_on_its_batch():
    """PanelGemmTests.ATokensResultDoesNotDependOnItsBatch (:61-74): bit equality."""
    rows, cols, tokens = 128, 3072, 17
    w = rand(rows * cols, 3, -1, 1).reshape(rows, cols)
    x = rand(tokens * cols, 4, -1, 1).reshape(tokens, cols)
    allr = ob.matmul(0, w.view(np.uint8), rows, cols, x, tokens)
    tail = ob.matmul(0, w.view(np.uint8), rows, cols, x[-5:], 5)
    assert allr[-5:].tobytes() == tail.tobytes()


def test_fan_out_does_not_change_the_result():
    """PanelGemmTests.FanOutDoesNotChangeTheResult (:76-89)."""
    rows, cols, tokens = 256, 3072, 11
    w = rand(rows * cols, 5, -1, 1).reshape(rows, cols)
    x = rand(tokens * cols, 6, -1, 1).reshape(tokens, cols)
    ob.set_threads(1)
    one = ob.matmul(0, w.view(np.uint8), rows, cols, x, tokens)
    ob.set_threads(8)
    many = ob.matmul(0, w.view(np.uint8), rows, cols, x, tokens)
    ob.set_threads(0)
    assert one.tobytes() == many.tobytes()


def test_quantized_matmul_agrees_with_dequantized_weights():
    """KernelTests.QuantMatMulAgreesWithDequantizedWeights (:224-261), float strategy."""
    rows, cols = 8, 256
    rng = np.random.default_rng(99)
    blocks = rng.integers(0, 256, rows * cols // 32 * 34, dtype=np.uint8)
    d = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    for b in range(rows * cols // 32):
        blocks[b * 34:b * 34 + 2] = d
    x = rand(cols, 12)
    deq = ob.dequantize(8, blocks, rows * cols).reshape(rows, cols)
    yq = ob.matmul(8, blocks, rows, cols, x, 1)
    yf = ob.matmul(0, deq.view(np.uint8), rows, cols, x, 1)
    close(yf, yq, 1e-6, "quantized vs dequantized")


# ------------------------------------------------------------------- model


def test_oracle_matches_the_reference_numpy_model(small_gguf, golden_small):
    """Every captured tensor of the reference's tools/reference_shieldstral.py on the same weights
    (the ActivationParityTests pattern, ActivationParityTests.cs:41-129)."""
    caps = {}
    with ob.OracleModel(small_gguf) as m:
        logits = m.forward(SMALL_PROMPT, sink=lambda n, a: caps.__setitem__(n, a))
    for key in golden_small.files:
        if not key.startswith("cap/"):
            continue
        ref, got = golden_small[key], caps[key[4:]]
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert rel < 1e-5, f"{key}: rel L2 {rel:.2e}"
    assert np.array_equal(caps["embeddings"], golden_small["cap/embeddings"])  # dequant is bit-exact
    close(golden_small["logits"], logits, 1e-5, "logits")


def _tokens(n, seed):
    return np.random.default_rng(seed).integers(1000, 16384, n).tolist()


def test_branches_match_running_each_continuation_alone(small_gguf):
    """DeciderTests.BranchesMatchRunningEachContinuationAlone (:54-91): bit-identical."""
    trunk = [1] + _tokens(40, 1)
    branches = [_tokens(n, 10 + i) for i, n in enumerate((5, 9, 3))]
    with ob.OracleModel(small_gguf) as m:
        tree = m.forward_tree(trunk, branches, VERDICT_ROWS)
        for b, br in enumerate(branches):
            m.kv_reset()
            m.forward(trunk, logits=False)
            alone = m.forward_selected(br, VERDICT_ROWS)
            assert alone.tobytes() == tree[b].tobytes(), f"branch {b}"


def test_cached_and_uncached_produce_identical_logits(small_gguf):
    """SystemPromptCacheTests.CachedAndUncachedProduceIdenticalLogits (:41-68)."""
    prompt = [1] + _tokens(60, 3)
    with ob.OracleModel(small_gguf) as m:
        whole = m.forward(prompt)
        m.kv_reset()
        m.forward(prompt[:37], logits=False)
        snap = m.kv_snapshot(37)
        m.kv_reset()
        m.kv_restore(snap, 37)
        cached = m.forward(prompt[37:])
    assert whole.tobytes() == cached.tobytes()


def test_a_row_after_the_prefix_is_a_causal_continuation(small_gguf):
    """TokenLayout.Rows (MinistralModel.cs:758-780): a row whose region starts right after the
    shared prefix sees exactly the causal context, so its last logits equal ForwardAsync's on the
    prompt plus the row (tolerance: the reference takes its sparse per-key attention for rows of
    fewer than 16 tokens)."""
    prefix = [1] + _tokens(30, 5)
    row = _tokens(4, 6)
    with ob.OracleModel(small_gguf) as m:
        whole = m.forward(prefix + row)
        m.kv_reset()
        m.forward(prefix, logits=False)
        rows = m.forward_rows(len(prefix), [len(prefix)], [0], [row])
    close(whole, rows[0], 1e-5, "row vs causal")


def test_rows_do_not_see_each_other(small_gguf):
    """Each row attends to the shared prefix and its own region only: a row's logits do not
    depend on which other rows share the pass (bit-identical while the head stays a GEMM, i.e.
    at least two rows: one output takes RunRowsFloat, QuantMatMul.cs:90-95,140-176)."""
    prefix = [1] + _tokens(30, 7)
    p = len(prefix)
    rows = [_tokens(n, 8 + i) for i, n in enumerate((3, 5, 2))]
    bases = [p + 32 * i for i in range(3)]
    with ob.OracleModel(small_gguf) as m:
        m.forward(prefix, logits=False)
        together = m.forward_rows(p, bases, [0, 0, 0], rows)
        m.kv_reset()
        m.forward(prefix, logits=False)
        pair = m.forward_rows(p, [bases[2], bases[1]], [0, 0], [rows[2], rows[1]])
    assert pair[0].tobytes() == together[2].tobytes()
    assert pair[1].tobytes() == together[1].tobytes()


def test_snapshot_rejects_more_than_is_cached(small_gguf):
    with ob.OracleModel(small_gguf) as m:
        m.forward([1, 2000], logits=False)
        with pytest.raises(ob.OracleError):
            m.kv_snapshot(3)
        snap = m.kv_snapshot(2)
        with pytest.raises(ob.OracleError):
            m.kv_restore(snap, 3)


def test_token_out_of_range_is_rejected(small_gguf):
    with ob.OracleModel(small_gguf) as m:
        with pytest.raises(ob.OracleError) as e:
            m.forward([1, 16384])
        assert e.value.code == 2


def test_truncated_gguf_is_rejected(small_gguf, tmp_path):
    """GgufReaderTests.RejectsATruncatedFile (:89-108)."""
    data = small_gguf.read_bytes()
    short = tmp_path / "short.gguf"
    short.write_bytes(data[: len(data) // 2])
    with pytest.raises(ob.OracleError) as e:
        ob.OracleModel(short)
    assert e.value.code == 4
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + data[4:100])
    with pytest.raises(ob.OracleError) as e:
        ob.OracleModel(bad)
    assert e.value.code == 3


def _rope_cs_freqs(base, dims, factor, orig, beta_fast, beta_slow, ext=1.0):
    """Rope() of the reference (src/Jevstral/Model/Rope.cs:33-66, YarnCorrectionDims :91-106) in
    float32, as MathF computes it: the frequency of every rotated pair with the YaRN ramp."""
    f32 = np.float32
    half = dims // 2
    base, factor, ext = f32(base), f32(factor), f32(ext)
    freq_scale = f32(1) / factor

    def corr(rot):
        return f32(dims) * np.log(f32(orig) / (f32(rot) * f32(2) * f32(np.pi)), dtype=f32) / (f32(2) * np.log(base, dtype=f32))

    low = max(f32(0), np.floor(corr(beta_fast)))
    high = min(f32(dims) / f32(2) - f32(1), np.ceil(corr(beta_slow)))
    out = np.empty(half, dtype=f32)
    for i in range(half):
        extrap = f32(1) / np.power(base, f32(2) * f32(i) / f32(dims), dtype=f32)
        interp = freq_scale * extrap
        y = (f32(i) - low) / max(f32(0.001), high - low)
        mix = (f32(1) - np.clip(y, f32(0), f32(1))) * ext
        out[i] = interp * (f32(1) - mix) + extrap * mix
    return out


def test_yarn_frequencies_follow_the_reference_formula(tmp_path):
    """The oracle's YaRN table (the real checkpoint's keys: factor 16 over 16384, beta 32/1,
    "apply_scale": false) against Rope.cs restated in float32, within float32 pow/log rounding; the
    magnitude scale cancels to exactly 1 and the query temperature is read (RopeAndCacheTests
    MagnitudeScaleIsOneWhenApplyScaleIsOff / YarnRampInterpolatesTheSlowBandsOnly)."""
    from jevstral_b200.synth import SynthConfig, write_random_gguf, yarn_metadata

    cfg = SynthConfig(layers=1, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=2048,
                      extra=yarn_metadata())
    path = write_random_gguf(tmp_path / "yarn.gguf", cfg, "Q8_0", seed=1, backend="fast")
    with ob.OracleModel(path) as o:
        assert o.config["yarn_active"] == 1
        assert o.config["rope_mscale"] == 1.0
        assert abs(o.config["temperature_scale"] - 0.1) < 1e-7
        assert o.config["rope_orig_ctx"] == 16384
        got = np.empty(64, dtype=np.float32)
        assert ob.lib.orc_rope_freqs(o._h, got.ctypes.data_as(ob.f32p)) == 64
    want = _rope_cs_freqs(1e6, 128, 16.0, 16384, 32.0, 1.0)
    assert np.allclose(got, want, rtol=4e-7, atol=0), np.abs(got / want - 1).max()
    base = np.float32(1) / np.power(np.float32(1e6), np.arange(64, dtype=np.float32) * 2 / 128, dtype=np.float32)
    # the fast bands keep the base frequency, the slow bands are divided by the factor
    assert np.allclose(got[:8], base[:8], rtol=1e-6)
    assert np.allclose(got[-4:], base[-4:] / 16, rtol=1e-6)


def test_the_avx512_tile_gives_the_avx2_tile_s_bits():
    """The panel GEMM's 16-lane tile (used where the host has AVX-512F, as the reference's
    Tile512x6 is) keeps each output's FMA chain, so it matches the 8-lane tile bit for bit."""
    rng = np.random.default_rng(8)
    raw = rng.integers(0, 256, 128 * 4096 // 32 * 34, dtype=np.uint8)
    for b in range(128 * 4096 // 32):  # finite fp16 scales
        raw[b * 34:b * 34 + 2] = np.frombuffer(np.float16(0.01 + 0.001 * (b % 7)).tobytes(), np.uint8)
    x = rng.normal(0, 1, (13, 4096)).astype(np.float32)
    try:
        ob.lib.orc_set_isa(1)
        narrow = ob.matmul(8, raw, 128, 4096, x, 13)
        ob.lib.orc_set_isa(0)
        wide = ob.matmul(8, raw, 128, 4096, x, 13)
    finally:
        ob.lib.orc_set_isa(0)
    assert narrow.tobytes() == wide.tobytes()

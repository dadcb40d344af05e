"""The random-weight GGUF writer's quantizer against the `gguf` package (0.19.0), the tool the
reference's converter quantizes with (tools/convert_shieldstral_to_gguf.py:285-292): the same fp32
values must give the same bytes. The benchmark and the full-depth tests write their 3B models
with the fast writer, so this is what ties those files to BASELINE.json's "quantised with
gguf.quants.quantize"."""
from __future__ import annotations

import gguf
import numpy as np
import pytest

from jevstral_b200.synth import (MINISTRAL_3B, QTYPES, SynthConfig, synth_normal, synth_quantize, tensor_plan,
                                 write_random_gguf)


def awkward_blocks(rng) -> np.ndarray:
    """Blocks that exercise the quantizers' edge cases: zeros, ties for the largest magnitude,
    a negative extreme, constant blocks, halves that round either way, large and tiny scales."""
    blocks = [np.zeros(32), np.full(32, 0.37), np.full(32, -1e-3)]
    b = rng.normal(0, 1, 32)
    b[5], b[17] = 4.0, -4.0          # equal magnitudes, opposite signs: the first one wins
    blocks.append(b)
    b = rng.normal(0, 1, 32)
    b[9] = -7.5                      # a negative extreme
    blocks.append(b)
    blocks.append(np.arange(32) / 2.0 - 8.0)   # exact halves after scaling
    blocks.append(rng.normal(0, 300.0, 32))
    blocks.append(rng.normal(0, 1e-6, 32))
    blocks.append(rng.uniform(-1, 1, 32) * 127 / 127.0)
    return np.concatenate(blocks).astype(np.float32)


@pytest.mark.parametrize("qtype", ["Q8_0", "Q4_0", "Q5_1"])
def test_quantizer_matches_the_gguf_package_bytes(qtype):
    rng = np.random.default_rng(11)
    normal = synth_normal(5, 3, 32 * 4096, 0.02)
    values = np.concatenate([normal, awkward_blocks(rng), rng.normal(0, 0.05, 32 * 512).astype(np.float32)])
    ours = synth_quantize(values, qtype)
    theirs = gguf.quants.quantize(values.reshape(-1, 32), getattr(gguf.GGMLQuantizationType, qtype))
    assert ours.tobytes() == np.ascontiguousarray(theirs).tobytes()


@pytest.mark.parametrize("qtype", ["Q8_0", "Q4_0", "Q5_1"])
def test_fast_writer_tensors_are_gguf_quantized_normals(tmp_path, qtype):
    """A file from the fast writer holds, for each matrix, gguf.quants.quantize of the counter-based
    N(0, 0.02) values of that tensor (checked on sampled rows of every matrix of a small model)."""
    cfg = SynthConfig(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=2048)
    path = write_random_gguf(tmp_path / "m.gguf", cfg, qtype, seed=9, backend="fast")
    reader = gguf.GGUFReader(str(path))
    tensors = {t.name: t for t in reader.tensors}
    qt = getattr(gguf.GGMLQuantizationType, qtype)
    for tid, (name, shape, is_mat) in enumerate(tensor_plan(cfg)):
        t = tensors[name]
        if not is_mat:
            assert np.array_equal(np.asarray(t.data, np.float32).reshape(-1), np.ones(shape[0], np.float32))
            continue
        assert int(t.tensor_type) == QTYPES[qtype]
        rows, cols = shape
        raw = np.asarray(t.data).reshape(rows, -1)
        for r in (0, 1, rows // 2, rows - 1):
            vals = synth_normal(9, tid, rows * cols, 0.02)[r * cols:(r + 1) * cols]
            want = gguf.quants.quantize(vals.reshape(1, cols), qt)
            assert raw[r].tobytes() == np.ascontiguousarray(want).tobytes(), (name, r)


def test_the_benchmark_model_shapes_are_the_3b_architecture():
    plan = {n: s for n, s, _ in tensor_plan(MINISTRAL_3B)}
    assert plan["token_embd.weight"] == (131072, 3072)
    assert plan["blk.25.attn_q.weight"] == (4096, 3072)
    assert plan["blk.25.attn_k.weight"] == (1024, 3072)
    assert plan["blk.25.ffn_down.weight"] == (3072, 9216)
    assert "blk.26.attn_q.weight" not in plan
    weights = sum(int(np.prod(s)) for n, s, m in tensor_plan(MINISTRAL_3B) if m and n.startswith("blk."))
    assert weights == 3_026_190_336


@pytest.mark.parametrize("qtype", ["Q8_0", "Q5_1"])
def test_the_standalone_writer_gives_the_same_file(tmp_path, qtype):
    """backend="exe" (the `jvsynth` program, used where no library of the package may be loaded)
    writes the same bytes as the in-process writer."""
    cfg = SynthConfig(layers=1, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=2048)
    a = write_random_gguf(tmp_path / "a.gguf", cfg, qtype, seed=4, backend="fast")
    b = write_random_gguf(tmp_path / "b.gguf", cfg, qtype, seed=4, backend="exe")
    assert a.read_bytes() == b.read_bytes()


@pytest.mark.parametrize("qtype", ["Q4_1", "Q5_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_random_block_files_decode_like_the_gguf_package(tmp_path, qtype):
    """The formats the writer fills with random blocks (there is no quantizer for them here): the
    file reads back through gguf.GGUFReader, and the oracle decodes each sampled matrix exactly as
    gguf.quants.dequantize does (the tool the reference's fixtures come from)."""
    from oracle import binding as ob

    cfg = SynthConfig(layers=1, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=2048)
    path = write_random_gguf(tmp_path / "k.gguf", cfg, qtype, seed=2, backend="fast")
    reader = gguf.GGUFReader(str(path))
    for t in reader.tensors:
        if not t.name.endswith(("attn_q.weight", "ffn_down.weight", "token_embd.weight")):
            continue
        assert t.tensor_type.name == qtype
        want = gguf.quants.dequantize(np.asarray(t.data), t.tensor_type).reshape(-1).astype(np.float32)
        got = ob.dequantize(QTYPES[qtype], np.asarray(t.data).reshape(-1), want.size)
        assert got.view(np.uint32).tobytes() == want.view(np.uint32).tobytes(), t.name
        assert 0.01 < float(want.std()) < 0.05


def test_per_tensor_types_make_a_mixed_k_quant_file(tmp_path):
    """type_overrides: a Q4_K file whose attn_v and ffn_down are Q6_K (the "Q4_K_M" mix), the same
    bytes from the in-process and the stand-alone writer."""
    mix = (("attn_v.weight", "Q6_K"), ("ffn_down.weight", "Q6_K"))
    cfg = SynthConfig(layers=1, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=2048, type_overrides=mix)
    a = write_random_gguf(tmp_path / "a.gguf", cfg, "Q4_K", seed=2, backend="fast")
    b = write_random_gguf(tmp_path / "b.gguf", cfg, "Q4_K", seed=2, backend="exe")
    assert a.read_bytes() == b.read_bytes()
    types = {t.name: t.tensor_type.name for t in gguf.GGUFReader(str(a)).tensors}
    assert types["blk.0.attn_v.weight"] == "Q6_K" and types["blk.0.ffn_down.weight"] == "Q6_K"
    assert types["blk.0.attn_q.weight"] == "Q4_K" and types["token_embd.weight"] == "Q4_K"

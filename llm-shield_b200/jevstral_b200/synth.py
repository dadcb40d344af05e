"""Random-init Ministral-3 GGUF files for the tests and the benchmark.

Two writers produce the same tensor set, metadata keys (llama.cpp's `mistral3` names, as
the reference's converter writes them: tools/convert_shieldstral_to_gguf.py:316-369) and
quantization rules (gguf.quants, the converter's quantizer):
  * backend="numpy": weights from numpy.random.default_rng(seed), quantized by
    gguf.quants.quantize and written by gguf.GGUFWriter — the standard tooling, used for
    the small test models;
  * backend="fast": weights from libjvsynth's counter-based generator, quantized by its
    restatement of the same rules, written straight into a memory-mapped file — seconds
    for the full 3B model instead of minutes;
  * backend="exe": the same bytes as "fast", filled by the stand-alone `jvsynth` program in a
    child process, so the calling process loads no library of this package (the benchmark's
    reference arm imports this file on its own, outside the package).
Norm gains are 1.0 in F32, the LM head is tied to token_embd, and the vocabulary is a
placeholder token list with "yes" at 13059 and "no" at 2649 (the real ids) when it fits.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Tuple

import numpy as np

PKG = Path(__file__).resolve().parent.parent
SYNTH_LIB = PKG / "libjvsynth.so"
SYNTH_EXE = PKG / "jvsynth"

QTYPES = {"F32": 0, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12,
          "Q5_K": 13, "Q6_K": 14}
# (weights, bytes) per block
BLOCKS = {0: (1, 4), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84), 11: (256, 110),
          12: (256, 144), 13: (256, 176), 14: (256, 210)}
# Formats the fast writer fills with random blocks (no quantizer; see gguf_synth.cpp).
RANDOM_BLOCK_TYPES = ("Q4_1", "Q5_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K")
YES_ID, NO_ID = 13059, 2649


@dataclass(frozen=True)
class SynthConfig:
    layers: int = 26
    hidden: int = 3072
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ff: int = 9216
    vocab: int = 131072
    rope_theta: float = 1e6
    eps: float = 1e-5
    context_length: int = 262144
    # Further `mistral3.*` metadata as (key after the architecture prefix, kind, value); kind is
    # "str", "u32" or "f32". yarn_metadata() gives the real checkpoint's RoPE scaling keys.
    extra: Tuple[Tuple[str, str, object], ...] = ()
    norm_gain: float = 1.0  # every RMSNorm gain (1.0 in the benchmark model)
    # Per-tensor weight types, as (tensor-name suffix, qtype): e.g. (("attn_v.weight", "Q6_K"),
    # ("ffn_down.weight", "Q6_K")) over a Q4_K file is the layout of a "Q4_K_M" checkpoint.
    type_overrides: Tuple[Tuple[str, str], ...] = ()


MINISTRAL_3B = SynthConfig()


def yarn_metadata(factor: float = 16.0, original_context: int = 16384, beta_fast: float = 32.0,
                  beta_slow: float = 1.0, temperature_scale: float = 0.1) -> Tuple[Tuple[str, str, object], ...]:
    """The RoPE-scaling and attention-temperature keys the reference's converter writes for a
    Mistral-format checkpoint with YaRN and llama-4 scaling (tools/convert_shieldstral_to_gguf.py:
    337-354): YaRN factor over an original window, beta fast/slow, "apply_scale": false (the
    magnitude terms cancel to 1), and the query temperature beta past the window."""
    return (("rope.scaling.type", "str", "yarn"),
            ("rope.scaling.factor", "f32", float(factor)),
            ("rope.scaling.original_context_length", "u32", int(original_context)),
            ("rope.scaling.yarn_beta_fast", "f32", float(beta_fast)),
            ("rope.scaling.yarn_beta_slow", "f32", float(beta_slow)),
            ("rope.scaling.yarn_ext_factor", "f32", 1.0),
            ("rope.scaling.mscale", "f32", 1.0),
            ("rope.scaling.yarn_log_multiplier", "f32", 1.0),
            ("rope.scaling.attn_factor", "f32", 1.0),
            ("attention.temperature_scale", "f32", float(temperature_scale)),
            ("attention.temperature_length", "u32", int(original_context)))


def tensor_plan(cfg: SynthConfig) -> List[Tuple[str, Tuple[int, ...], bool]]:
    """(name, numpy shape (rows, cols) or (n,), is_matrix) in file order."""
    q, kv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    plan = [("token_embd.weight", (cfg.vocab, cfg.hidden), True), ("output_norm.weight", (cfg.hidden,), False)]
    for l in range(cfg.layers):
        p = f"blk.{l}."
        plan += [(p + "attn_norm.weight", (cfg.hidden,), False),
                 (p + "attn_q.weight", (q, cfg.hidden), True),
                 (p + "attn_k.weight", (kv, cfg.hidden), True),
                 (p + "attn_v.weight", (kv, cfg.hidden), True),
                 (p + "attn_output.weight", (cfg.hidden, q), True),
                 (p + "ffn_norm.weight", (cfg.hidden,), False),
                 (p + "ffn_gate.weight", (cfg.ff, cfg.hidden), True),
                 (p + "ffn_up.weight", (cfg.ff, cfg.hidden), True),
                 (p + "ffn_down.weight", (cfg.hidden, cfg.ff), True)]
    return plan


def _token_list(vocab: int) -> List[str]:
    toks = [f"<t{i}>" for i in range(vocab)]
    if vocab > YES_ID:
        toks[YES_ID] = "yes"
    if vocab > NO_ID:
        toks[NO_ID] = "no"
    return toks


def _metadata(cfg: SynthConfig, qtype: int) -> Dict[str, tuple]:
    a = "mistral3"
    return {
        "general.architecture": ("str", a),
        "general.name": ("str", "random-init Ministral-3"),
        "general.alignment": ("u32", 32),
        "general.file_type": ("u32", qtype),
        f"{a}.context_length": ("u32", cfg.context_length),
        f"{a}.embedding_length": ("u32", cfg.hidden),
        f"{a}.block_count": ("u32", cfg.layers),
        f"{a}.feed_forward_length": ("u32", cfg.ff),
        f"{a}.attention.head_count": ("u32", cfg.heads),
        f"{a}.attention.head_count_kv": ("u32", cfg.kv_heads),
        f"{a}.attention.key_length": ("u32", cfg.head_dim),
        f"{a}.attention.value_length": ("u32", cfg.head_dim),
        f"{a}.attention.layer_norm_rms_epsilon": ("f32", cfg.eps),
        f"{a}.vocab_size": ("u32", cfg.vocab),
        f"{a}.rope.freq_base": ("f32", cfg.rope_theta),
        f"{a}.rope.dimension_count": ("u32", cfg.head_dim),
        "tokenizer.ggml.tokens": ("strs", _token_list(cfg.vocab)),
        "tokenizer.ggml.bos_token_id": ("u32", 1),
        "tokenizer.ggml.eos_token_id": ("u32", 2),
        **{f"{a}.{k}": (kind, v) for k, kind, v in cfg.extra},
    }


def _enc_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _enc_kv(key: str, kind: str, val) -> bytes:
    out = _enc_str(key)
    if kind == "str":
        return out + struct.pack("<I", 8) + _enc_str(val)
    if kind == "u32":
        return out + struct.pack("<II", 4, int(val))
    if kind == "f32":
        return out + struct.pack("<If", 6, float(val))
    if kind == "strs":
        body = b"".join(_enc_str(s) for s in val)
        return out + struct.pack("<IIQ", 9, 8, len(val)) + body
    raise ValueError(kind)


def _row_bytes(qtype: int, cols: int) -> int:
    w, b = BLOCKS[qtype]
    return cols // w * b


def _synth_lib():
    if not SYNTH_LIB.exists():
        raise ImportError(f"{SYNTH_LIB} is not built; run `python llm-shield_b200/build.py`")
    lib = C.CDLL(str(SYNTH_LIB))
    lib.jvs_fill.restype = C.c_int64
    lib.jvs_fill.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_uint64, C.c_uint32, C.c_float, C.c_int]
    lib.jvs_quantize.restype = C.c_int64
    lib.jvs_quantize.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_void_p]
    lib.jvs_normal.restype = None
    lib.jvs_normal.argtypes = [C.c_uint64, C.c_uint32, C.c_float, C.c_int64, C.c_void_p]
    return lib


def synth_normal(seed: int, tensor_id: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _synth_lib().jvs_normal(seed, tensor_id, std, n, out.ctypes.data)
    return out


def synth_quantize(values: np.ndarray, qtype: str) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    t = QTYPES[qtype]
    out = np.empty(_row_bytes(t, v.size), dtype=np.uint8)
    n = _synth_lib().jvs_quantize(v.ctypes.data, t, v.size, out.ctypes.data)
    if n < 0:
        raise ValueError("bad quantization request")
    return out


def write_random_gguf(path, cfg: SynthConfig = MINISTRAL_3B, qtype: str = "Q8_0", seed: int = 0,
                      backend: str = "fast", std: float = 0.02) -> Path:
    path = Path(path)
    if backend == "numpy":
        if qtype in RANDOM_BLOCK_TYPES:
            raise ValueError(f"{qtype} has no quantizer here; write it with backend='fast' (random blocks)")
        return _write_numpy(path, cfg, qtype, seed, std)
    t = QTYPES[qtype]
    plan = tensor_plan(cfg)
    kv = _metadata(cfg, t)
    header = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(plan), len(kv)))
    for k, (kind, v) in kv.items():
        header += _enc_kv(k, kind, v)
    def type_of(name: str) -> int:
        for suffix, q in cfg.type_overrides:
            if name.endswith(suffix):
                return QTYPES[q]
        return t

    offsets, off = [], 0
    for name, shape, is_mat in plan:
        tt = type_of(name) if is_mat else 0
        ne = list(reversed(shape))
        header += _enc_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        header += struct.pack("<IQ", tt, off)
        offsets.append(off)
        nbytes = _row_bytes(tt, shape[-1]) * (shape[0] if len(shape) == 2 else 1)
        off += (nbytes + 31) // 32 * 32
    data_start = (len(header) + 31) // 32 * 32
    total = data_start + off
    tmp = path.with_suffix(path.suffix + ".partial")
    with open(tmp, "wb") as f:
        f.write(header)
        f.truncate(total)
    mm = np.memmap(tmp, dtype=np.uint8, mode="r+")
    threads = os.cpu_count() or 1
    jobs = []
    for tid, ((name, shape, is_mat), o) in enumerate(zip(plan, offsets)):
        base = data_start + o
        if not is_mat:
            mm[base:base + 4 * shape[0]] = np.full(shape[0], cfg.norm_gain, dtype=np.float32).view(np.uint8)
            continue
        jobs.append((tid, base, shape[0], shape[1], name, type_of(name)))
    if backend == "exe":
        mm.flush()
        del mm
        if not SYNTH_EXE.exists():
            raise FileNotFoundError(f"{SYNTH_EXE} is not built; run `python llm-shield_b200/build.py`")
        for jt in sorted({j[5] for j in jobs}):  # the program fills one weight type per run
            plan_text = "".join(f"{tid} {base} {rows} {cols}\n" for tid, base, rows, cols, _, tt in jobs if tt == jt)
            r = subprocess.run([str(SYNTH_EXE), str(tmp), str(jt), str(seed), repr(float(std)), str(threads)],
                               input=plan_text, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"jvsynth failed ({r.returncode}): {r.stderr.strip()}")
    else:
        lib = _synth_lib()
        for tid, base, rows, cols, name, tt in jobs:
            n = lib.jvs_fill(C.c_void_p(mm.ctypes.data + base), tt, rows, cols, seed, tid, std, threads)
            if n != _row_bytes(tt, cols) * rows:
                raise RuntimeError(f"jvs_fill failed for {name}")
        mm.flush()
        del mm
    os.replace(tmp, path)
    return path


def _write_numpy(path: Path, cfg: SynthConfig, qtype: str, seed: int, std: float) -> Path:
    import gguf
    from gguf import GGMLQuantizationType as G

    qt = getattr(G, qtype)
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(str(path), "mistral3")
    for k, (kind, v) in _metadata(cfg, QTYPES[qtype]).items():
        if k in ("general.architecture", "general.alignment"):
            continue
        if kind == "str":
            w.add_string(k, v)
        elif kind == "u32":
            w.add_uint32(k, v)
        elif kind == "f32":
            w.add_float32(k, v)
        elif kind == "strs":
            w.add_array(k, v)
    for name, shape, is_mat in tensor_plan(cfg):
        if not is_mat:
            w.add_tensor(name, np.full(shape, cfg.norm_gain, dtype=np.float32))
            continue
        vals = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        w.add_tensor(name, gguf.quants.quantize(vals, qt), raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path

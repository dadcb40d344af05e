"""MinistralModel / KvCache over the C ABI, with the reference's member names.

Reference: src/Jevstral/Model/MinistralModel.cs (forward entry points, :128-294),
src/Jevstral/Model/KvCache.cs (cache state), src/Jevstral/Model/ModelConfig.cs.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import JvConfig, JvLayout, check, lib
from .layout import TokenLayout


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _p(a: np.ndarray, t=C.c_int32):
    return a.ctypes.data_as(C.POINTER(t))


@dataclass(frozen=True)
class ModelConfig:
    """ModelConfig (ModelConfig.cs:11-56), as the library resolved it."""
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ff: int
    vocab: int
    rope_dim: int
    context_length: int
    rope_orig_ctx: int
    yarn_active: bool
    weight_type: int
    eps: float
    rope_base: float
    rope_scale: float
    rope_mscale: float
    temperature_scale: float

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


def device_count() -> int:
    n = C.c_int32(0)
    check(lib.jv_device_count(C.byref(n)))
    return n.value


def kernel_launches() -> int:
    return int(lib.jv_kernel_launches())


class Model:
    """The weights of one GGUF resident on one GPU (the shareable half of MinistralModel)."""

    def __init__(self, path: str, device: int = 0, kv_pool_mb: int = 0):
        h = C.c_void_p()
        check(lib.jv_model_open(str(path).encode(), device, kv_pool_mb, C.byref(h)))
        self._h = h
        self.path = str(path)
        self.device = device
        cfg = JvConfig()
        check(lib.jv_model_config(h, C.byref(cfg)))
        self.config = ModelConfig(**{f: getattr(cfg, f) for f, _ in JvConfig._fields_})

    def close(self) -> None:
        if self._h:
            lib.jv_model_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Snapshot:
    """Refcounted KV pages holding a prefix (zero-copy SystemPromptCache / question LRU)."""

    def __init__(self, handle):
        self._h = handle

    @property
    def length(self) -> int:
        return int(lib.jv_snapshot_length(self._h))

    def release(self) -> None:
        if self._h:
            lib.jv_snapshot_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class KvCache:
    """KvCache (KvCache.cs:12-140) of one context, backed by device KV pages."""

    def __init__(self, ctx: "MinistralModel"):
        self._ctx = ctx

    @property
    def length(self) -> int:
        return int(lib.jv_kv_length(self._ctx._h))

    @property
    def capacity(self) -> int:
        return int(lib.jv_kv_capacity(self._ctx._h))

    @property
    def bytes_per_position(self) -> int:
        return int(lib.jv_kv_bytes_per_position(self._ctx._h))

    def reset(self) -> None:
        check(lib.jv_kv_reset(self._ctx._h))

    def truncate(self, length: int) -> None:
        check(lib.jv_kv_truncate(self._ctx._h, int(length)))

    def ensure_capacity(self, required: int) -> None:
        check(lib.jv_kv_ensure_capacity(self._ctx._h, int(required)))

    def snapshot(self, length: int) -> np.ndarray:
        """Snapshot (KvCache.cs:94-112): flat fp32, keys of all layers/heads then values."""
        n = int(lib.jv_kv_snapshot_floats(self._ctx._h, int(length)))
        out = np.empty(max(n, 0), dtype=np.float32)
        check(lib.jv_kv_snapshot(self._ctx._h, int(length), _p(out, C.c_float), n))
        return out

    def restore(self, snapshot: np.ndarray, length: int) -> None:
        """Restore (KvCache.cs:115-136)."""
        s = np.ascontiguousarray(snapshot, dtype=np.float32)
        check(lib.jv_kv_restore(self._ctx._h, _p(s, C.c_float), s.size, int(length)))

    def save_shkv(self, path, fingerprint: str, tokens: Sequence[int]) -> None:
        """SystemPromptCache.Save (SystemPromptCache.cs:110-127) of the first len(tokens) cached
        positions, written from the device pages in the reference's SHKV file format."""
        t = _i32(tokens)
        check(lib.jv_kv_save_shkv(self._ctx._h, str(path).encode(), fingerprint.encode(), _p(t), t.size))

    def load_shkv(self, path, fingerprint: str, max_tokens: int = 1 << 20) -> Optional[List[int]]:
        """SystemPromptCache.TryLoad + RestoreInto (SystemPromptCache.cs:65-74,133-164): the
        cache becomes the file's prefix and its tokens are returned; None on a miss (a file that
        is absent, unreadable, or not a snapshot of this model and prefix), cache untouched."""
        out = np.empty(max_tokens, dtype=np.int32)
        n = C.c_int32(0)
        rc = lib.jv_kv_load_shkv(self._ctx._h, str(path).encode(), fingerprint.encode(), _p(out), max_tokens,
                                 C.byref(n))
        if rc in (_lib.JV_ERR_IO, _lib.JV_ERR_FORMAT):
            return None
        check(rc)
        return out[: n.value].tolist()

    def share(self, length: int) -> Snapshot:
        h = C.c_void_p()
        check(lib.jv_kv_share(self._ctx._h, int(length), C.byref(h)))
        return Snapshot(h)

    def adopt(self, snap: Snapshot) -> None:
        check(lib.jv_kv_adopt(self._ctx._h, snap._h))


class MinistralModel:
    """One MinistralModel instance: a KV cache, a stream and buffers over shared weights.

    Not thread-safe, like the reference (MinistralModel.cs:21-22).
    """

    def __init__(self, model: Model, initial_capacity: int = 512):
        h = C.c_void_p()
        check(lib.jv_ctx_create(model._h, int(initial_capacity), C.byref(h)))
        self._h = h
        self.model = model
        self.config = model.config
        self.kv_cache = KvCache(self)
        self._sink_ref = None
        self._cancel = None

    # -- lifecycle
    def close(self) -> None:
        if self._h:
            lib.jv_ctx_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def cached_token_count(self) -> int:
        return self.kv_cache.length

    @property
    def stream(self) -> int:
        return int(lib.jv_ctx_stream(self._h) or 0)

    def reset_kv_cache(self) -> None:
        self.kv_cache.reset()

    PROFILE_KINDS = {"gemm": 0, "gemv": 1, "attention": 2, "other": 3}

    def profile(self, enable: bool = True) -> None:
        """Bracket GEMM / GEMV / attention launches with CUDA events on this context's stream."""
        check(lib.jv_ctx_profile(self._h, int(enable)))

    def profile_reset(self) -> None:
        check(lib.jv_ctx_profile_reset(self._h))

    def check_wait_timeout(self, bound_cycles: int = 20_000_000) -> None:
        """Run one device wait that nothing completes; raises DeviceTimeoutError once its bound
        (SM clock cycles) runs out, after which the context is usable again."""
        check(lib.jv_ctx_check_wait_timeout(self._h, int(bound_cycles)))

    def profile_read(self, kind: str) -> dict:
        ms, n, fl, by = C.c_double(), C.c_int64(), C.c_double(), C.c_double()
        check(lib.jv_ctx_profile_read(self._h, self.PROFILE_KINDS[kind], C.byref(ms), C.byref(n), C.byref(fl),
                                      C.byref(by)))
        return {"ms": ms.value, "launches": n.value, "flops": fl.value, "bytes": by.value}

    def set_activation_sink(self, sink: Optional[Callable[[str, np.ndarray], None]]) -> None:
        """IActivationSink: sink(name, array[rows, cols]) after every named sub-step."""
        if sink is None:
            self._sink_ref = None
            check(lib.jv_ctx_set_sink(self._h, _lib.SINK(), None))
            return

        def cb(user, name, values, rows, cols):
            arr = np.ctypeslib.as_array(values, shape=(rows * cols,)).reshape(rows, cols).copy()
            sink(name.decode(), arr)

        self._sink_ref = _lib.SINK(cb)
        check(lib.jv_ctx_set_sink(self._h, self._sink_ref, None))

    def set_cancellation(self, flag: Optional[np.ndarray]) -> None:
        """flag: an int32 numpy array of size 1; setting flag[0] != 0 cancels between layers."""
        self._cancel = flag
        check(lib.jv_ctx_set_cancel(self._h, _p(flag) if flag is not None else None))

    # -- forward passes (MinistralModel.cs:139-294)
    def forward(self, tokens: Sequence[int]) -> np.ndarray:
        """ForwardAsync(tokens): full-vocabulary logits of the last position."""
        t = _i32(tokens)
        out = np.empty(self.config.vocab, dtype=np.float32)
        check(lib.jv_forward(self._h, _p(t), t.size, _p(out, C.c_float)))
        return out

    def prefill(self, tokens: Sequence[int]) -> None:
        """PrefillAsync(tokens): KV only, no LM head."""
        t = _i32(tokens)
        check(lib.jv_forward(self._h, _p(t), t.size, None))

    def forward_selected(self, tokens: Sequence[int], vocab_rows: Sequence[int]) -> np.ndarray:
        t, r = _i32(tokens), _i32(vocab_rows)
        out = np.empty(r.size, dtype=np.float32)
        check(lib.jv_forward_selected(self._h, _p(t), t.size, _p(r), r.size, _p(out, C.c_float)))
        return out

    def forward_tree(self, trunk: Sequence[int], branches: Sequence[Sequence[int]],
                     vocab_rows: Sequence[int]) -> np.ndarray:
        """ForwardTreeAsync: [branches][rows] logits at each branch's last token."""
        tr = _i32(trunk)
        lens = _i32([len(b) for b in branches])
        flat = _i32(np.concatenate([np.asarray(b, dtype=np.int32) for b in branches]) if len(branches) else [])
        r = _i32(vocab_rows)
        out = np.empty((len(branches), r.size), dtype=np.float32)
        check(lib.jv_forward_tree(self._h, _p(tr), tr.size, _p(flat), _p(lens), len(branches), _p(r), r.size,
                                  _p(out, C.c_float)))
        return out

    def decide_batch(self, decisions: Sequence[Tuple[Sequence[int], Sequence[Sequence[int]]]],
                     vocab_rows: Sequence[int]) -> List[np.ndarray]:
        """Many independent tree decisions in one pass (jv_decide_batch): for each (trunk, branches)
        the [branches][rows] logits ForwardTreeAsync gives it on an empty cache. The cache is left
        as it was."""
        flat, trunks, counts, lens = [], [], [], []
        for trunk, branches in decisions:
            flat.extend(int(v) for v in trunk)
            trunks.append(len(trunk))
            counts.append(len(branches))
            for b in branches:
                flat.extend(int(v) for v in b)
                lens.append(len(b))
        t, tr, cn, ln, r = _i32(flat), _i32(trunks), _i32(counts), _i32(lens), _i32(vocab_rows)
        out = np.empty((len(lens), r.size), dtype=np.float32)
        check(lib.jv_decide_batch(self._h, len(decisions), _p(t), _p(tr), _p(cn), _p(ln), _p(r), r.size,
                                  _p(out, C.c_float)))
        res, i = [], 0
        for n in counts:
            res.append(out[i:i + n])
            i += n
        return res

    def forward_branches(self, branches, vocab_rows) -> np.ndarray:
        return self.forward_tree([], branches, vocab_rows)

    def forward_layout(self, tokens: Sequence[int], layout: Optional[TokenLayout], vocab_rows=None,
                       full_vocab: bool = False, compute_logits: bool = False):
        """The private ForwardAsync(tokens, ..., layout, selectedRows, selectedOut)."""
        t = _i32(tokens)
        keep = []
        lp = None
        n_out = 1
        if layout is not None:
            arrs = [_i32(a) for a in (layout.slot, layout.position, layout.shared, layout.segment, layout.outputs)]
            keep += arrs
            lay = JvLayout(_p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(arrs[3]), _p(arrs[4]), arrs[4].size, layout.end,
                           int(layout.sparse))
            lp = C.byref(lay)
            n_out = arrs[4].size
        r = _i32(vocab_rows) if vocab_rows is not None else None
        out = None
        if r is not None:
            out = np.empty((n_out, r.size), dtype=np.float32)
        elif full_vocab:
            out = np.empty((n_out, self.config.vocab), dtype=np.float32)
        logits = np.empty(self.config.vocab, dtype=np.float32) if compute_logits else None
        check(lib.jv_forward_layout(self._h, _p(t), t.size, lp, _p(r) if r is not None else None,
                                    r.size if r is not None else 0, int(full_vocab),
                                    _p(out, C.c_float) if out is not None else None, int(compute_logits),
                                    _p(logits, C.c_float) if logits is not None else None))
        return out, logits

    def forward_tree_logits(self, trunk, branches):
        """ForwardTreeLogitsAsync (MinistralModel.cs:227-255): full vocabulary at every branch token."""
        trunk = list(trunk)
        offsets, total = [], len(trunk)
        for b in branches:
            if len(b) == 0:
                raise _lib.ArgumentError(_lib.JV_ERR_ARG, "Branch is empty.")
            offsets.append(total)
            total += len(b)
        tokens = trunk + [x for b in branches for x in b]
        tree = TokenLayout.tree(self.kv_cache.length, len(trunk), offsets, total)
        lay = tree.with_outputs(list(range(len(trunk), total)))
        flat, _ = self.forward_layout(tokens, lay, None, full_vocab=True)
        res, k = [], 0
        for b in branches:
            res.append([flat[k + i] for i in range(len(b))])
            k += len(b)
        return res

    def forward_rows(self, shared: int, row_base, row_length, row_tokens, vocab_rows=None):
        """ForwardRowsAsync (MinistralModel.cs:282-294)."""
        counts = [len(r) for r in row_tokens]
        if any(c == 0 for c in counts):
            raise _lib.ArgumentError(_lib.JV_ERR_ARG, "Every row needs at least one token.")
        lay = TokenLayout.rows(shared, list(row_base), list(row_length), counts, sparse=max(counts) < 16)
        tokens = [x for r in row_tokens for x in r]
        out, _ = self.forward_layout(tokens, lay, vocab_rows, full_vocab=vocab_rows is None)
        return out

    def decode_greedy(self, first_token: int, steps: int) -> np.ndarray:
        out = np.empty(steps, dtype=np.int32)
        check(lib.jv_decode_greedy(self._h, int(first_token), int(steps), _p(out)))
        return out

"""ctypes binding of the CPU restatement (oracle/jv_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg, to check or time the CUDA path. Never by the product package.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Callable, Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libjvoracle.so"

i32, i64 = C.c_int32, C.c_int64
f32p, i32p, u8p = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.POINTER(C.c_uint8)
SINK = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, f32p, i32, i32)


class OrcConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ff", "vocab",
                                         "rope_dim")] + \
               [(n, C.c_float) for n in ("eps", "rope_base", "rope_mscale", "temperature_scale")] + \
               [("rope_orig_ctx", C.c_int32), ("yarn_active", C.c_int32)]


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _load():
    if not LIB_PATH.exists():
        build()
    lib = C.CDLL(str(LIB_PATH))
    sigs = [
        ("orc_last_error", C.c_char_p, []),
        ("orc_set_threads", None, [C.c_int]),
        ("orc_threads", C.c_int, []),
        ("orc_set_isa", None, [C.c_int]),
        ("orc_isa", C.c_int, []),
        ("orc_open", C.c_int, [C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]),
        ("orc_close", None, [C.c_void_p]),
        ("orc_config_get", C.c_int, [C.c_void_p, C.POINTER(OrcConfig)]),
        ("orc_rope_freqs", C.c_int, [C.c_void_p, f32p]),
        ("orc_forward", C.c_int, [C.c_void_p, i32p, i32, i32, f32p, SINK, C.c_void_p]),
        ("orc_forward_selected", C.c_int, [C.c_void_p, i32p, i32, i32p, i32, f32p]),
        ("orc_forward_tree", C.c_int, [C.c_void_p, i32p, i32, i32p, i32p, i32, i32p, i32, f32p, SINK, C.c_void_p]),
        ("orc_forward_rows", C.c_int, [C.c_void_p, i32, i32p, i32p, i32p, i32p, i32, i32p, i32, f32p]),
        ("orc_kv_length", i32, [C.c_void_p]),
        ("orc_kv_capacity", i32, [C.c_void_p]),
        ("orc_kv_reset", None, [C.c_void_p]),
        ("orc_kv_truncate", None, [C.c_void_p, i32]),
        ("orc_kv_snapshot_floats", i64, [C.c_void_p, i32]),
        ("orc_kv_snapshot", C.c_int, [C.c_void_p, i32, f32p]),
        ("orc_kv_restore", C.c_int, [C.c_void_p, f32p, i64, i32]),
        ("orc_dequantize", C.c_int, [C.c_uint32, u8p, f32p, i64]),
        ("orc_row_bytes", i64, [C.c_uint32, i64]),
        ("orc_matmul", C.c_int, [C.c_uint32, u8p, i32, i32, f32p, i32, f32p]),
        ("orc_rmsnorm", None, [f32p, f32p, i32, C.c_float, f32p]),
        ("orc_softmax", None, [f32p, i32]),
        ("orc_swiglu", None, [f32p, f32p, f32p, i32]),
        ("orc_dot", C.c_float, [f32p, f32p, i32]),
    ]
    for name, res, args in sigs:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(rc, (lib.orc_last_error() or b"").decode())


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(f32p)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(i32p)


def set_threads(n: int) -> None:
    lib.orc_set_threads(int(n))


def dequantize(type_id: int, raw: np.ndarray, count: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(count, dtype=np.float32)
    _check(lib.orc_dequantize(type_id, raw.ctypes.data_as(u8p), _fp(out), count))
    return out


def matmul(type_id: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, tokens: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(tokens * rows, dtype=np.float32)
    _check(lib.orc_matmul(type_id, w.ctypes.data_as(u8p), rows, cols, _fp(x), tokens, _fp(y)))
    return y.reshape(tokens, rows)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    lib.orc_rmsnorm(_fp(x), _fp(w), x.size, eps, _fp(y))
    return y


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib.orc_softmax(_fp(y), y.size)
    return y


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32).copy()
    d = np.empty_like(g)
    lib.orc_swiglu(_fp(g), _fp(u), _fp(d), g.size)
    return d


class OracleModel:
    """The restated MinistralModel: fp32 CPU, one KvCache."""

    def __init__(self, path, initial_capacity: int = 512):
        h = C.c_void_p()
        _check(lib.orc_open(str(path).encode(), initial_capacity, C.byref(h)))
        self._h = h
        c = OrcConfig()
        _check(lib.orc_config_get(h, C.byref(c)))
        self.config = {f: getattr(c, f) for f, _ in OrcConfig._fields_}

    def close(self):
        if self._h:
            lib.orc_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *e):
        self.close()

    def _sink(self, sink: Optional[Callable[[str, np.ndarray], None]]):
        if sink is None:
            return SINK(), None

        def cb(user, name, values, rows, cols):
            sink(name.decode(), np.ctypeslib.as_array(values, shape=(rows * cols,)).reshape(rows, cols).copy())

        f = SINK(cb)
        return f, f

    def forward(self, tokens: Sequence[int], logits: bool = True, sink=None):
        t = _i32(tokens)
        out = np.empty(self.config["vocab"], dtype=np.float32) if logits else None
        fn, keep = self._sink(sink)
        _check(lib.orc_forward(self._h, _ip(t), t.size, int(logits), _fp(out) if logits else None, fn, None))
        return out

    def forward_selected(self, tokens, rows):
        t, r = _i32(tokens), _i32(rows)
        out = np.empty(r.size, dtype=np.float32)
        _check(lib.orc_forward_selected(self._h, _ip(t), t.size, _ip(r), r.size, _fp(out)))
        return out

    def forward_tree(self, trunk, branches, rows, sink=None):
        tr = _i32(trunk)
        lens = _i32([len(b) for b in branches])
        flat = _i32(np.concatenate([np.asarray(b, dtype=np.int32) for b in branches]))
        r = _i32(rows) if rows is not None else None
        width = r.size if r is not None else self.config["vocab"]
        out = np.empty((len(branches), width), dtype=np.float32)
        fn, keep = self._sink(sink)
        _check(lib.orc_forward_tree(self._h, _ip(tr), tr.size, _ip(flat), _ip(lens), len(branches),
                                    _ip(r) if r is not None else None, r.size if r is not None else 0, _fp(out), fn,
                                    None))
        return out

    def forward_rows(self, shared, row_base, row_length, row_tokens, rows=None):
        counts = _i32([len(x) for x in row_tokens])
        flat = _i32(np.concatenate([np.asarray(x, dtype=np.int32) for x in row_tokens]))
        rb, rl = _i32(row_base), _i32(row_length)
        r = _i32(rows) if rows is not None else None
        width = r.size if r is not None else self.config["vocab"]
        out = np.empty((len(row_tokens), width), dtype=np.float32)
        _check(lib.orc_forward_rows(self._h, shared, _ip(rb), _ip(rl), _ip(flat), _ip(counts), len(row_tokens),
                                    _ip(r) if r is not None else None, r.size if r is not None else 0, _fp(out)))
        return out

    @property
    def kv_length(self) -> int:
        return int(lib.orc_kv_length(self._h))

    @property
    def kv_capacity(self) -> int:
        return int(lib.orc_kv_capacity(self._h))

    def kv_reset(self):
        lib.orc_kv_reset(self._h)

    def kv_truncate(self, n):
        lib.orc_kv_truncate(self._h, int(n))

    def kv_snapshot(self, n) -> np.ndarray:
        out = np.empty(int(lib.orc_kv_snapshot_floats(self._h, int(n))), dtype=np.float32)
        _check(lib.orc_kv_snapshot(self._h, int(n), _fp(out)))
        return out

    def kv_restore(self, snap: np.ndarray, n: int):
        s = np.ascontiguousarray(snap, dtype=np.float32)
        _check(lib.orc_kv_restore(self._h, _fp(s), s.size, int(n)))

"""ctypes binding of include/jv.h (libjv.so, built in-tree by llm-shield_b200/build.py).

There is no fallback: if the library is missing or cannot be loaded, importing this
module raises, so nothing can silently run without the CUDA path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
# JV_LIBRARY may name the bounds-checked build (libjv_checked.so) for a diagnostic run.
LIB_PATH = Path(os.environ["JV_LIBRARY"]) if os.environ.get("JV_LIBRARY") else PKG / "libjv.so"

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is not built; run `python llm-shield_b200/build.py` (nvcc, sm_100a)")

lib = C.CDLL(str(LIB_PATH))

i32 = C.c_int32
i64 = C.c_int64
f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)
vp = C.c_void_p


class JvConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ff", "vocab", "rope_dim",
                                         "context_length", "rope_orig_ctx", "yarn_active", "weight_type")] + \
               [(n, C.c_float) for n in ("eps", "rope_base", "rope_scale", "rope_mscale", "temperature_scale")]


class JvLayout(C.Structure):
    _fields_ = [("slot", i32p), ("position", i32p), ("shared", i32p), ("segment", i32p), ("outputs", i32p),
                ("n_outputs", i32), ("end", i32), ("sparse", i32)]


SINK = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, f32p, i32, i32)

# Every symbol include/jv.h declares, with its signature: (name, restype, argtypes).
SIGNATURES = [
    ("jv_last_error", C.c_char_p, []),
    ("jv_device_count", C.c_int, [i32p]),
    ("jv_kernel_launches", i64, []),
    ("jv_build_features", i32, []),
    ("jv_model_open", C.c_int, [C.c_char_p, i32, i32, C.POINTER(vp)]),
    ("jv_model_close", None, [vp]),
    ("jv_model_config", C.c_int, [vp, C.POINTER(JvConfig)]),
    ("jv_ctx_create", C.c_int, [vp, i32, C.POINTER(vp)]),
    ("jv_ctx_destroy", None, [vp]),
    ("jv_ctx_set_sink", C.c_int, [vp, SINK, vp]),
    ("jv_ctx_set_cancel", C.c_int, [vp, i32p]),
    ("jv_ctx_stream", vp, [vp]),
    ("jv_ctx_profile", C.c_int, [vp, i32]),
    ("jv_ctx_profile_read", C.c_int, [vp, i32, C.POINTER(C.c_double), C.POINTER(i64), C.POINTER(C.c_double),
                                      C.POINTER(C.c_double)]),
    ("jv_ctx_profile_reset", C.c_int, [vp]),
    ("jv_ctx_check_wait_timeout", C.c_int, [vp, i64]),
    ("jv_forward", C.c_int, [vp, i32p, i32, f32p]),
    ("jv_forward_selected", C.c_int, [vp, i32p, i32, i32p, i32, f32p]),
    ("jv_forward_tree", C.c_int, [vp, i32p, i32, i32p, i32p, i32, i32p, i32, f32p]),
    ("jv_decide_batch", C.c_int, [vp, i32, i32p, i32p, i32p, i32p, i32p, i32, f32p]),
    ("jv_forward_layout", C.c_int, [vp, i32p, i32, C.POINTER(JvLayout), i32p, i32, i32, f32p, i32, f32p]),
    ("jv_decode_greedy", C.c_int, [vp, i32, i32, i32p]),
    ("jv_qweight_bytes", i64, [i32, i32, i32]),
    ("jv_qweight_pack", C.c_int, [i32, vp, i32, i32, vp, vp]),
    ("jv_qmatvec", C.c_int, [i32, vp, i32, i32, vp, vp, vp]),
    ("jv_qmatvec_noalloc", C.c_int, [i32, vp, i32, i32, vp, vp, vp]),
    ("jv_kv_length", i32, [vp]),
    ("jv_kv_capacity", i32, [vp]),
    ("jv_kv_reset", C.c_int, [vp]),
    ("jv_kv_truncate", C.c_int, [vp, i32]),
    ("jv_kv_ensure_capacity", C.c_int, [vp, i32]),
    ("jv_kv_bytes_per_position", i64, [vp]),
    ("jv_kv_snapshot_floats", i64, [vp, i32]),
    ("jv_kv_snapshot", C.c_int, [vp, i32, f32p, i64]),
    ("jv_kv_restore", C.c_int, [vp, f32p, i64, i32]),
    ("jv_kv_save_shkv", C.c_int, [vp, C.c_char_p, C.c_char_p, i32p, i32]),
    ("jv_kv_load_shkv", C.c_int, [vp, C.c_char_p, C.c_char_p, i32p, i32, i32p]),
    ("jv_kv_share", C.c_int, [vp, i32, C.POINTER(vp)]),
    ("jv_kv_adopt", C.c_int, [vp, vp]),
    ("jv_snapshot_length", i32, [vp]),
    ("jv_snapshot_release", None, [vp]),
]

for _name, _res, _args in SIGNATURES:
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

# Status codes (enum jv_status).
JV_OK, JV_ERR_ARG, JV_ERR_RANGE, JV_ERR_FORMAT, JV_ERR_IO, JV_ERR_UNSUPPORTED, JV_ERR_CANCELLED, JV_ERR_DEVICE, \
    JV_ERR_DEVICE_TIMEOUT, JV_ERR_OOM, JV_ERR_NUMERIC = range(11)


class JvError(Exception):
    """A non-OK status from libjv; `code` is the JV_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


# The reference's exception types: ArgumentException, ArgumentOutOfRangeException,
# InvalidDataException, IOException, NotSupportedException, OperationCanceledException; a device
# failure, which has no counterpart in the managed reference; and ArithmeticException for an
# activation outside the fp16 range the device path computes in.
class ArgumentError(JvError, ValueError): ...
class ArgumentOutOfRangeError(JvError, IndexError): ...
class InvalidDataError(JvError): ...
class GgufIOError(JvError, OSError): ...
class NotSupportedError(JvError): ...
class OperationCanceledError(JvError): ...
class DeviceError(JvError, RuntimeError): ...
class DeviceTimeoutError(DeviceError): ...
class DeviceOutOfMemoryError(DeviceError, MemoryError): ...
class NumericError(JvError, ArithmeticError): ...


_BY_CODE = {JV_ERR_ARG: ArgumentError, JV_ERR_RANGE: ArgumentOutOfRangeError, JV_ERR_FORMAT: InvalidDataError,
            JV_ERR_IO: GgufIOError, JV_ERR_UNSUPPORTED: NotSupportedError, JV_ERR_CANCELLED: OperationCanceledError,
            JV_ERR_DEVICE: DeviceError, JV_ERR_DEVICE_TIMEOUT: DeviceTimeoutError, JV_ERR_OOM: DeviceOutOfMemoryError,
            JV_ERR_NUMERIC: NumericError}


def check(rc: int) -> None:
    if rc != JV_OK:
        msg = (lib.jv_last_error() or b"").decode(errors="replace")
        raise _BY_CODE.get(rc, JvError)(rc, msg)

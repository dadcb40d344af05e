"""The C ABI boundary without a GPU: the library loads, exports every declared symbol, and its
error paths return statuses instead of crashing."""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

from conftest import REPO

HEADER = REPO / "include" / "jv.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(jv_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import ctypes

    from jevstral_b200._lib import LIB_PATH

    lib = ctypes.CDLL(str(LIB_PATH))
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared in jv.h but not exported: {missing}"


def test_python_binding_covers_the_header():
    from jevstral_b200 import SIGNATURES

    bound = {s[0] for s in SIGNATURES}
    assert set(declared_functions()) <= bound


def test_build_targets_sm100a_only():
    import importlib.util

    spec = importlib.util.spec_from_file_location("jv_build", REPO / "llm-shield_b200" / "build.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    assert b.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_error_paths_return_statuses():
    import jevstral_b200 as jv

    assert jv.device_count() >= 0
    if jv.device_count() == 0:
        with pytest.raises(jv.JvError):
            jv.Model("/nonexistent.gguf")
    else:
        with pytest.raises(jv.GgufIOError):
            jv.Model("/nonexistent.gguf")
    # context entry points check their handle before touching a device
    from jevstral_b200._lib import JV_ERR_ARG, lib

    assert lib.jv_ctx_check_wait_timeout(None, 1000) == JV_ERR_ARG
    assert lib.jv_ctx_profile(None, 1) == JV_ERR_ARG
    assert b"NULL" in lib.jv_last_error()


def test_token_layout_restatement_matches_the_reference_rules():
    """TokenLayout.Tree / Rows (MinistralModel.cs:720-780) on a hand-checked case."""
    from jevstral_b200 import TokenLayout

    t = TokenLayout.tree(start_pos=10, trunk=3, offsets=[3, 5], tokens=8)
    assert t.slot == list(range(10, 18))
    assert t.position == [10, 11, 12, 13, 14, 13, 14, 15]
    assert t.shared == [10, 10, 10, 13, 13, 13, 13, 13]
    assert t.segment == [10, 10, 10, 13, 13, 15, 15, 15]
    assert t.outputs == [4, 7] and t.end == 18
    r = TokenLayout.rows(shared=4, row_base=[10, 20], row_length=[2, 0], row_tokens=[1, 2], sparse=True)
    assert r.slot == [12, 20, 21] and r.position == [6, 4, 5] and r.segment == [10, 20, 20]
    assert r.outputs == [0, 2] and r.end == 22


def test_decider_tail_matches_the_reference_formulas():
    """JevstralDecider.DecideAsync margins and softmax(z/T) (JevstralDecider.cs:306-313)."""
    from jevstral_b200 import decision_probs, margins_from_verdicts

    v = np.array([[1.0, 3.0, 0.5], [2.0, -1.0, -3.0]], np.float32)  # 2 yes rows, 1 no row
    z = margins_from_verdicts(v, n_yes=2)
    assert np.allclose(z, [2.5, 5.0])
    p = decision_probs(z, 2.0)
    e = np.exp(z / 2 - (z / 2).max())
    assert np.allclose(p, e / e.sum(), rtol=1e-6)


def test_struct_layouts_match_the_binding(tmp_path):
    """jv_config and jv_layout as a C compiler lays them out (the layout the C# structs mirror
    with LayoutKind.Sequential) against the ctypes mirror and the fixed sizes the library
    asserts at compile time (runtime.cu)."""
    import ctypes
    import subprocess

    from jevstral_b200._lib import JvConfig, JvLayout

    fields = {"jv_config": [f for f, _ in JvConfig._fields_], "jv_layout": [f for f, _ in JvLayout._fields_]}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "jv.h"', "int main(void) {"]
    for st, names in fields.items():
        lines.append(f'    printf("{st} sizeof %zu\\n", sizeof({st}));')
        for n in names:
            lines.append(f'    printf("{st} {n} %zu\\n", offsetof({st}, {n}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        st, name, val = line.split()
        got[(st, name)] = int(val)
    for st, cls in (("jv_config", JvConfig), ("jv_layout", JvLayout)):
        assert got[(st, "sizeof")] == ctypes.sizeof(cls), st
        for n in fields[st]:
            assert got[(st, n)] == getattr(cls, n).offset, (st, n)
    assert got[("jv_config", "sizeof")] == 68 and got[("jv_layout", "sizeof")] == 56


def test_status_codes_match_the_header():
    """Every JV_* status in include/jv.h has the same value in the Python binding (and so in a
    C# enum generated from the same header)."""
    import re as _re

    from jevstral_b200 import _lib

    text = HEADER.read_text()
    body = text[text.index("enum jv_status"):text.index("};", text.index("enum jv_status"))]
    body = _re.sub(r"/\*.*?\*/", "", body, flags=_re.S)
    codes = dict((n, int(v)) for n, v in _re.findall(r"(JV_[A-Z_]+)\s*=\s*(\d+)", body))
    assert codes["JV_ERR_NUMERIC"] == 10 and len(codes) == 11
    for name, value in codes.items():
        assert getattr(_lib, name) == value, name
    assert issubclass(_lib._BY_CODE[_lib.JV_ERR_NUMERIC], ArithmeticError)


def test_shkv_restatement_round_trips_and_encodes_lengths_like_binarywriter():
    import numpy as _np

    import shkv_format as shkv

    # .NET's documented 7-bit encoding examples
    assert shkv.encode_7bit(0) == b"\x00" and shkv.encode_7bit(127) == b"\x7f"
    assert shkv.encode_7bit(128) == b"\x80\x01" and shkv.encode_7bit(300) == b"\xac\x02"
    state = _np.arange(24, dtype=_np.float32) / 7
    fp = "ab" * 100  # a 200-byte string needs the two-byte length prefix
    blob = shkv.write(fp, [1, 5, 9], state)
    assert blob[:4] == bytes.fromhex("564b4853")  # "SHKV" little-endian
    got_fp, toks, st = shkv.read(blob)
    assert got_fp == fp and toks == [1, 5, 9] and _np.array_equal(st, state)


def test_shkv_entry_points_reject_bad_arguments_without_a_device():
    from jevstral_b200._lib import JV_ERR_ARG, lib

    n = ctypes_i32()
    assert lib.jv_kv_save_shkv(None, b"/tmp/x", b"fp", None, 0) == JV_ERR_ARG
    assert lib.jv_kv_load_shkv(None, b"/tmp/x", b"fp", None, 0, n) == JV_ERR_ARG


def ctypes_i32():
    import ctypes

    return ctypes.byref(ctypes.c_int32(0))


def test_the_bounds_checked_build_exports_the_same_api_and_says_so():
    """libjv_checked.so (built with -DJV_BOUNDS_CHECK) carries every declared symbol, and
    jv_build_features tells the two builds apart."""
    import ctypes

    from jevstral_b200._lib import LIB_PATH

    checked = LIB_PATH.parent / "libjv_checked.so"
    normal = ctypes.CDLL(str(LIB_PATH.parent / "libjv.so"))
    chk = ctypes.CDLL(str(checked))
    for lib in (normal, chk):
        assert not [n for n in declared_functions() if not hasattr(lib, n)]
        lib.jv_build_features.restype = ctypes.c_int32
    assert normal.jv_build_features() == 0
    assert chk.jv_build_features() == 1

"""The bounds-checked build (libjv_checked.so: every KV page-table lookup and GEMM work unit is
tested and a bad index fails the call with JV_ERR_RANGE instead of touching memory) runs the
parity tests that exercise the page tables — trees, reused trunks, decision batches, decode steps,
long contexts, snapshots and SHKV files, K-quant models — and none of them reports an index out
of range. It stands in for a memory checker, which this pool does not offer."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

SELECTION = ("tree_decision_matches or full_width_tree or decode_steps or decode_greedy or branches_match or "
             "cached_and_uncached or reusing_the_trunk or snapshot or verdict_scorer or decision_batch or "
             "long_context or batched_rows or tree_logits or k_quant_tree or mixed_k_quant or yarn")


def test_parity_tests_run_clean_on_the_bounds_checked_build():
    lib = REPO / "llm-shield_b200" / "libjv_checked.so"
    assert lib.exists(), "build it with llm-shield_b200/build.py"
    env = dict(os.environ, JV_LIBRARY=str(lib))
    probe = subprocess.run([sys.executable, "-c", "import sys; sys.path.insert(0, sys.argv[1]); import jevstral_b200 as jv;"
                            "print(jv._lib.lib.jv_build_features())", str(REPO / "llm-shield_b200")],
                           env=env, capture_output=True, text=True, timeout=120)
    assert probe.stdout.strip() == "1", probe.stderr
    r = subprocess.run([sys.executable, "-m", "pytest", str(REPO / "tests" / "test_gpu_parity.py"), "-m", "gpu", "-q",
                        "-x", "-p", "no:cacheprovider", "-k", SELECTION], env=env, capture_output=True, text=True,
                       timeout=1800, cwd=str(REPO))
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-2000:])
    assert " passed" in r.stdout and "failed" not in r.stdout

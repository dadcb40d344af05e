"""Shared fixtures. `-m gpu` marks the parity tests that need a B200; everything else runs on CPU."""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO / "llm-shield_b200", REPO, REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from small_model import SMALL_CFG, SMALL_QTYPE, SMALL_SEED, WIDE_CFG  # noqa: E402

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_small():
    return np.load(GOLDEN / "refnumpy_small.npz")


@pytest.fixture(scope="session")
def small_gguf(tmp_path_factory, golden_small):
    """The small model the reference NumPy golden was computed on (regenerated, hash-checked)."""
    from jevstral_b200.synth import write_random_gguf

    p = write_random_gguf(tmp_path_factory.mktemp("models") / "small.gguf", SMALL_CFG, SMALL_QTYPE, seed=SMALL_SEED,
                          backend="numpy")
    digest = hashlib.sha256(p.read_bytes()).digest()
    assert digest == golden_small["gguf_sha256"].tobytes(), "the regenerated small model differs from the golden's"
    return p


@pytest.fixture(scope="session")
def model_factory(tmp_path_factory):
    """Random GGUF files by (config, qtype, seed), written once per session."""
    from jevstral_b200.synth import write_random_gguf

    cache = {}
    root = tmp_path_factory.mktemp("synth")

    def make(cfg=WIDE_CFG, qtype="Q8_0", seed=7, backend="fast"):
        key = (cfg, qtype, seed, backend)
        if key not in cache:
            name = f"m_{len(cache)}_{qtype}.gguf"
            cache[key] = write_random_gguf(root / name, cfg, qtype, seed=seed, backend=backend)
        return cache[key]

    return make

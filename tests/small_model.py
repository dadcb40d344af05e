"""The small random models the tests run on (shared by the fixtures generator and the tests).

Shapes keep every constraint of the B200 kernels (head_dim 128, 4 query heads per KV
head, widths that tile into 128 x 64 chunks) and the verdict ids 13059/2649, at a size the
CPU oracle runs in well under a second."""
from __future__ import annotations

import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
if str(REPO / "llm-shield_b200") not in sys.path:
    sys.path.insert(0, str(REPO / "llm-shield_b200"))

from jevstral_b200.synth import SynthConfig  # noqa: E402

SMALL_CFG = SynthConfig(layers=2, hidden=256, heads=8, kv_heads=2, head_dim=128, ff=512, vocab=16384)
SMALL_SEED = 20261201
SMALL_QTYPE = "Q8_0"
SMALL_PROMPT = [1, 4017, 12001, 1500, 9001, 2222, 3333, 13000, 7777, 1234, 15000, 16000, 1001, 5555, 6666, 7070,
                8080, 9090, 10101, 11111, 12121, 13131, 14141, 15151]

# A full-width model with few layers: every real matrix shape of Ministral-3 3B
# (6144x3072 QKV, 3072x4096 O, 18432x3072 gate/up, 3072x9216 down).
WIDE_CFG = SynthConfig(layers=2, vocab=16384)

VERDICT_ROWS = [13059, 2649]

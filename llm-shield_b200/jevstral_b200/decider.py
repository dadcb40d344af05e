"""The decision logic around one tree pass, on token ids (JevstralDecider.DecideAsync,
reference src/Jevstral/JevstralDecider.cs:246-354). Tokenization and prompt rendering stay
with the host application; this is the part that drives the model and its KV cache."""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from .model import MinistralModel, Snapshot


def softmax(x: np.ndarray) -> np.ndarray:
    """Kernels.Softmax (Kernels.cs:102-121): max-shifted; uniform when the max is not finite."""
    x = np.asarray(x, dtype=np.float32).copy()
    if x.size == 0:
        return x
    mx = np.max(x)
    if not np.isfinite(mx):
        return np.full_like(x, 1.0 / x.size)
    e = np.exp(x - mx, dtype=np.float32)
    return (e / np.float32(e.sum(dtype=np.float32))).astype(np.float32)


def margins_from_verdicts(verdicts: np.ndarray, n_yes: int) -> np.ndarray:
    """z_i = max(yes rows) - max(no rows) (JevstralDecider.cs:306-308)."""
    v = np.asarray(verdicts, dtype=np.float32)
    return (v[:, :n_yes].max(axis=1) - v[:, n_yes:].max(axis=1)).astype(np.float32)


def decision_probs(margins: np.ndarray, temperature: float = 1.0) -> np.ndarray:
    """softmax(z / T) (JevstralDecider.cs:310-313)."""
    return softmax(np.asarray(margins, dtype=np.float32) / np.float32(temperature))


def common_prefix(a: Sequence[int], b: Optional[Sequence[int]]) -> int:
    if b is None:
        return 0
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


@dataclass
class DecisionResult:
    probabilities: np.ndarray
    margins: np.ndarray
    prefix_tokens: int
    suffix_tokens: int
    cached_tokens: int = 0


@dataclass
class _QuestionSnapshot:
    tokens: List[int]
    state: Snapshot


class TokenDecider:
    """DecideAsync on token ids: prefix reuse against the resident trunk, an LRU of question
    snapshots (zero-copy shared KV pages instead of float copies), the "never an empty
    trunk" rule, one tree pass, truncation back to the prefix, margins and softmax."""

    def __init__(self, model: MinistralModel, yes_rows: Sequence[int], no_rows: Sequence[int],
                 snapshots: int = 8):
        self.model = model
        self.yes = list(yes_rows)
        self.no = list(no_rows)
        self.verdict_rows = self.yes + self.no
        self._resident: Optional[List[int]] = None
        self._snaps: "OrderedDict[tuple, _QuestionSnapshot]" = OrderedDict()
        self._max_snaps = snapshots
        self.question_hits = 0

    def _find_snapshot(self, prefix: List[int], start: int) -> Optional[_QuestionSnapshot]:
        best = None
        for key, snap in self._snaps.items():
            n = len(snap.tokens)
            if start < n <= len(prefix) and prefix[:n] == snap.tokens and (best is None or n > len(best.tokens)):
                best = snap
        if best is not None:
            self._snaps.move_to_end(tuple(best.tokens))
        return best

    def _remember(self, prefix: List[int], question_length: int) -> None:
        if question_length <= 0 or question_length > self.model.kv_cache.length:
            return
        key = tuple(prefix[:question_length])
        if key in self._snaps:
            self._snaps.move_to_end(key)
            return
        self._snaps[key] = _QuestionSnapshot(list(key), self.model.kv_cache.share(question_length))
        while len(self._snaps) > self._max_snaps:
            _, old = self._snaps.popitem(last=False)
            old.state.release()

    def decide(self, prefix: Sequence[int], branches: Sequence[Sequence[int]], question_length: int = 0,
               temperature: float = 1.0) -> DecisionResult:
        if len(branches) < 2:
            raise ValueError("A decision needs at least two options.")
        prefix = list(prefix)
        kv = self.model.kv_cache
        start = common_prefix(prefix, self._resident)
        snap = self._find_snapshot(prefix, start) if start < question_length else None
        if snap is not None:
            kv.adopt(snap.state)
            start = len(snap.tokens)
            self.question_hits += 1
        elif start > 0:
            kv.truncate(start)
        else:
            kv.reset()
            start = 0
        if start == len(prefix):  # never an empty trunk (JevstralDecider.cs:287-289)
            start -= 1
            kv.truncate(start)
        verdicts = self.model.forward_tree(prefix[start:], branches, self.verdict_rows)
        kv.truncate(len(prefix))
        self._resident = prefix
        self._remember(prefix, question_length)
        margins = margins_from_verdicts(verdicts, len(self.yes))
        probs = decision_probs(margins, temperature)
        return DecisionResult(probs, margins, len(prefix), sum(len(b) for b in branches), start)

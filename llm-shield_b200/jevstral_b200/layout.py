"""TokenLayout (reference src/Jevstral/Model/MinistralModel.cs:703-780), restated for callers
that build layouts by hand (jv_forward_layout). The C library builds the Tree layout itself
for jv_forward_tree, with the same rules."""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import List


@dataclass
class TokenLayout:
    slot: List[int]
    position: List[int]
    shared: List[int]
    segment: List[int]
    outputs: List[int]
    end: int
    sparse: bool = False

    @staticmethod
    def tree(start_pos: int, trunk: int, offsets: List[int], tokens: int) -> "TokenLayout":
        """TokenLayout.Tree (MinistralModel.cs:720-745)."""
        slot, pos, sh, seg = [0] * tokens, [0] * tokens, [0] * tokens, [0] * tokens
        branch = -1
        for t in range(tokens):
            slot[t] = start_pos + t
            while branch + 1 < len(offsets) and t >= offsets[branch + 1]:
                branch += 1
            if t < trunk or branch < 0:
                pos[t], sh[t], seg[t] = start_pos + t, start_pos, start_pos
            else:
                pos[t] = start_pos + trunk + (t - offsets[branch])
                sh[t] = start_pos + trunk
                seg[t] = start_pos + offsets[branch]
        outputs = [(offsets[b + 1] if b + 1 < len(offsets) else tokens) - 1 for b in range(len(offsets))]
        return TokenLayout(slot, pos, sh, seg, outputs, start_pos + tokens)

    def with_outputs(self, outputs: List[int]) -> "TokenLayout":
        """TokenLayout.WithOutputs (MinistralModel.cs:748-751)."""
        return replace(self, outputs=list(outputs))

    @staticmethod
    def rows(shared: int, row_base: List[int], row_length: List[int], row_tokens: List[int],
             sparse: bool) -> "TokenLayout":
        """TokenLayout.Rows (MinistralModel.cs:758-780)."""
        total = sum(row_tokens)
        slot, pos, sh, seg = [0] * total, [0] * total, [0] * total, [0] * total
        outputs = [0] * len(row_tokens)
        t, end = 0, shared
        for r, n in enumerate(row_tokens):
            for i in range(n):
                slot[t] = row_base[r] + row_length[r] + i
                pos[t] = shared + row_length[r] + i
                sh[t] = shared
                seg[t] = row_base[r]
                end = max(end, slot[t] + 1)
                t += 1
            outputs[r] = t - 1
        return TokenLayout(slot, pos, sh, seg, outputs, end, sparse)

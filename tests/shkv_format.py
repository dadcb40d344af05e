"""The reference's system-prompt snapshot file ("SHKV", src/Jevstral/SystemPromptCache.cs:110-164),
restated in Python for the tests: .NET BinaryWriter's little-endian fields and its 7-bit-encoded
string length. Test infrastructure only."""
from __future__ import annotations

import struct
from typing import List, Optional, Tuple

import numpy as np

MAGIC, VERSION = 0x53484B56, 1


def encode_7bit(n: int) -> bytes:
    """BinaryWriter.Write7BitEncodedInt: seven bits a byte, low first, high bit = more follow."""
    out = bytearray()
    while n >= 0x80:
        out.append((n & 0x7F) | 0x80)
        n >>= 7
    out.append(n)
    return bytes(out)


def write(fingerprint: str, tokens: List[int], state: np.ndarray) -> bytes:
    fp = fingerprint.encode()
    head = struct.pack("<Ii", MAGIC, VERSION) + encode_7bit(len(fp)) + fp + struct.pack("<i", len(tokens))
    head += struct.pack(f"<{len(tokens)}i", *tokens) + struct.pack("<q", state.size)
    return head + np.ascontiguousarray(state, dtype="<f4").tobytes()


def read(data: bytes) -> Optional[Tuple[str, List[int], np.ndarray]]:
    magic, version = struct.unpack_from("<Ii", data, 0)
    if magic != MAGIC or version != VERSION:
        return None
    pos, n, shift = 8, 0, 0
    while True:
        b = data[pos]
        pos += 1
        n |= (b & 0x7F) << shift
        shift += 7
        if not b & 0x80:
            break
    fp = data[pos:pos + n].decode()
    pos += n
    (count,) = struct.unpack_from("<i", data, pos)
    pos += 4
    tokens = list(struct.unpack_from(f"<{count}i", data, pos))
    pos += 4 * count
    (floats,) = struct.unpack_from("<q", data, pos)
    pos += 8
    state = np.frombuffer(data, dtype="<f4", count=floats, offset=pos)
    return fp, tokens, state

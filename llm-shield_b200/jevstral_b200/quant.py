"""QuantMatMul on device buffers (reference src/Jevstral/Numerics/QuantMatMul.cs): re-tile GGUF
rows into this library's layout and run the single-token product. Arguments are device
pointers (ints), e.g. torch tensors' data_ptr(); `stream` is a cudaStream_t or 0."""
from __future__ import annotations

from ._lib import check, lib

TYPE_IDS = {"Q8_0": 8, "Q5_1": 7, "Q4_0": 2}
BLOCK_BYTES = {8: 34, 7: 24, 2: 18}


def qweight_bytes(qtype: str, rows: int, cols: int) -> int:
    n = int(lib.jv_qweight_bytes(TYPE_IDS[qtype], rows, cols))
    if n < 0:
        check(1)
    return n


def gguf_row_bytes(qtype: str, cols: int) -> int:
    return cols // 32 * BLOCK_BYTES[TYPE_IDS[qtype]]


def qweight_pack(qtype: str, gguf_rows_ptr: int, rows: int, cols: int, tiled_ptr: int, stream: int = 0) -> None:
    check(lib.jv_qweight_pack(TYPE_IDS[qtype], gguf_rows_ptr, rows, cols, tiled_ptr, stream))


def qmatvec(qtype: str, tiled_ptr: int, rows: int, cols: int, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
    """y[rows] = W x[cols] (fp32), QuantMatMul.ForwardAsync for one token."""
    check(lib.jv_qmatvec(TYPE_IDS[qtype], tiled_ptr, rows, cols, x_ptr, y_ptr, stream))

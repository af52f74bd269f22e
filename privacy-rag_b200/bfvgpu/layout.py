"""Public packing layout of the coefficient-packed matrix protocol.

Mirrors IV1/native/include/prag/bfv_layout.hpp:8-27 (``MatrixPacking``,
``matrix_packing``, ``matrix_packing_qk_reverse64``), IV1/native/src/bfv.cpp:112-116
(``packed_bfv_rows_per_ciphertext``) and the packing loops of
IV1/native/src/bfv_matrix.inc:25-29, :156-163.  All of it is public-dimension integer
logic; the same rule appears in the CPU oracle as an independent restatement.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

MASK59 = (1 << 59) - 1
MATRIX_BATCH_MAX = 16
MATRIX_INNER_MAX = 8192
MATRIX_COLUMNS_MAX = 155648
MATRIX_OUTPUT_COORDINATES = 512
DECODE_QK_REVERSE_BATCH_MAX = 64
INPUT_CT_BYTES = 1572960   # one [2][6][16384] input ciphertext plus framing, as costed
RETURN_BYTES = 786528      # one returned c1 [6][16384] plus framing


@dataclass(frozen=True)
class MatrixPacking:
    reduction: int
    columns: int
    returns: int
    inputs: int


def matrix_packing(b: int, k: int, o: int) -> MatrixPacking:
    """Cost-selected power-of-two reduction d: minimise inputs*1572960 + returns*786528;
    ties keep the smallest d.  Raises ValueError("E_MATRIX_SHAPE") outside the limits."""
    if not (0 < b <= 16 and 0 < k <= 8192 and 0 < o <= 155648):
        raise ValueError("E_MATRIX_SHAPE")
    gc = 512 // b
    best, cost = None, None
    d = 16
    while d <= 8192 // b:
        cap = min(gc, 8192 // (b * d))
        full, tail = divmod(o, gc)
        returns = full * ((gc + cap - 1) // cap) + ((tail + cap - 1) // cap if tail else 0)
        inputs = (k + d - 1) // d
        nbytes = inputs * INPUT_CT_BYTES + returns * RETURN_BYTES
        if cost is None or nbytes < cost:
            cost, best = nbytes, MatrixPacking(d, cap, returns, inputs)
        d *= 2
    return best


def matrix_packing_qk_reverse64(b: int) -> MatrixPacking:
    if not 0 < b <= 64:
        raise ValueError("E_QK_REVERSE64_SHAPE")
    return MatrixPacking(128, 1, 1, 1)


def packed_bfv_rows_per_ciphertext(d: int) -> int:
    if d == 0 or d > 8192:
        raise ValueError("E_BFV_PACKED_SHAPE")
    return min(16384 // (2 * d - 1), 8192 // d)


def pack_inputs(x: np.ndarray, d: int, blocks: int, n: int) -> np.ndarray:
    """x [B][K] ring-59 words -> packed input polys [blocks][n]:
    x[b][blk*d+j] at coefficient b*(2d-1)+j (bfv_matrix.inc:25-29)."""
    x = np.asarray(x, dtype=np.uint64)
    B, K = x.shape
    stride = 2 * d - 1
    out = np.zeros((blocks, n), dtype=np.uint64)
    for blk in range(blocks):
        width = min(d, K - blk * d)
        if width <= 0:
            continue
        for b in range(B):
            out[blk, b * stride: b * stride + width] = x[b, blk * d: blk * d + width] & np.uint64(MASK59)
    return out


def pack_weights(blocks_w: list, d: int, batch: int, n: int) -> np.ndarray:
    """Reader blocks -> weight ring polys [blocks][n]: row o of a block, column j, at
    coefficient o*B*(2d-1)+d-1-j (bfv_matrix.inc:156-160)."""
    stride = 2 * d - 1
    out = np.zeros((len(blocks_w), n), dtype=np.uint64)
    for blk, rows in enumerate(blocks_w):
        w = np.asarray(rows, dtype=np.uint64)
        if w.size == 0:
            continue
        count, actual = w.shape
        for o in range(count):
            base = o * batch * stride + d - 1
            out[blk, base - actual + 1: base + 1] = (w[o, ::-1] & np.uint64(MASK59))
    return out


def targets(count: int, batch: int, d: int) -> list[int]:
    """(o*B+b)*(2d-1)+d-1 for o < count, b < B (bfv_matrix.inc:162-163)."""
    stride = 2 * d - 1
    return [(o * batch + b) * stride + d - 1 for o in range(count) for b in range(batch)]

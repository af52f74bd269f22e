"""Matrix-protocol engine over the GPU backends: the BFV arithmetic of
``BfvEngine::matrix`` (IV1/native/src/bfv_matrix.inc:3-282) for both parties, with the
reference's operator API (``SecureOps::private_matrix`` / ``private_linear``,
IV1/native/include/prag/secure_ops.hpp:131-145) and public limits.

Out of this engine's scope, as in the rest of the repository: the two-party transport
(the ``send_data``/``recv_data`` calls become return values here) and the garbled-circuit
decode after the hand-off.  What crosses to the decoder is exactly what the reference
hands it: for every output coordinate the server's c0 value at the target coefficient
as an integer in [0, Q) (``rns_coefficient``, bfv.cpp:138-147, computed on the GPU) and
the client's c1*s value at the same coefficient.

Server side, per output group (bfv_matrix.inc:150-233): the reader callback returns the
weight block, the weights are packed into one ring polynomial per input block, the
server's local share x_S . W is accumulated on the host, and the GPU computes
W x Enc(x_C), subtracts the Delta-scaled mask, adds Enc(0), and returns c1 plus the
targets' c0.  Groups are batched into one ``Matrix.evaluate_groups`` call per chunk
instead of the reference's one-group-at-a-time pipeline (bfv_matrix.inc:77-120).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from .backend import Context, Matrix, NttBatch, PublicZero
from .layout import (MASK59, MATRIX_BATCH_MAX, MATRIX_COLUMNS_MAX, MATRIX_INNER_MAX, pack_inputs,
                     pack_weights, packed_bfv_rows_per_ciphertext, matrix_packing, targets as target_list)

Reader = Callable[[int, int, int, int], list]   # (input_begin, actual, first_row, rows) -> rows x actual
LINEAR_BLOCK = 8192
LINEAR_BLOCKS_MAX = 19


class ProtocolShapeError(ValueError):
    """Public shape rejected before any ciphertext is produced (the reference's E_SHAPE)."""


# --------------------------------------------------------------------------------------
# randomness (explicit buffers so parity is testable; the default draws from os.urandom)
# --------------------------------------------------------------------------------------
def _urandom_u64(count: int) -> np.ndarray:
    return np.frombuffer(os.urandom(8 * count), dtype=np.uint64).copy()


def urandom_masks(groups: int, n: int) -> np.ndarray:
    """Uniform ring-59 masks [groups][n] (the reference draws RAND_priv_bytes & MASK)."""
    return (_urandom_u64(groups * n) & np.uint64(MASK59)).reshape(groups, n)


def urandom_enc0_samples(primes: list[int], groups: int, n: int) -> np.ndarray:
    """Enc(0) randomness [groups][3][k][n]: ternary u, then e0, e1 from a centred binomial
    of 21 coin pairs (variance 10.5), as residues of every key-level prime."""
    k = len(primes)
    raw = _urandom_u64(groups * 3 * n)
    u = (raw[: groups * n] % np.uint64(3)).astype(np.int64) - 1
    bits = raw[groups * n:]
    lo = np.uint64((1 << 21) - 1)
    a = np.bitwise_count(bits & lo).astype(np.int64)
    b = np.bitwise_count((bits >> np.uint64(21)) & lo).astype(np.int64)
    e = (a - b).reshape(groups, 2, n)
    out = np.empty((groups, 3, k, n), dtype=np.uint64)
    signed = [u.reshape(groups, n), e[:, 0], e[:, 1]]
    for i, v in enumerate(signed):
        for p, q in enumerate(primes):
            out[:, i, p] = (v % q).astype(np.uint64)
    return out


# --------------------------------------------------------------------------------------
@dataclass
class TileReturn:
    """What the server hands to the peer / decoder for one tile of output columns."""
    first_column: int
    columns: int
    c1: np.ndarray              # [groups][dk][n]: sent to the client (bfv_matrix.inc:228)
    targets: list               # per group, the target coefficient indices
    c0_phase: list = field(default_factory=list)  # [columns*B] ints in [0,Q): server c0 at targets


class MatrixServer:
    """Server role of the coefficient-packed matrix protocol on one device."""

    def __init__(self, ctx: Context, pk: np.ndarray, group_chunk: int = 64,
                 masks: Callable[[int], np.ndarray] | None = None,
                 samples: Callable[[int], np.ndarray] | None = None):
        self.ctx = ctx
        self.pk = pk
        self.group_chunk = group_chunk
        self.masks = masks or (lambda g: urandom_masks(g, ctx.n))
        self.samples = samples or (lambda g: urandom_enc0_samples(ctx.primes, g, ctx.n))

    def run(self, encrypted: np.ndarray, x_local: np.ndarray, outputs: int, reader: Reader,
            d: int, cap: int, batch: int, tile_columns: int):
        """encrypted [I][2][dk][n]; x_local [B][K] the server's shares.  Returns
        (result [B][outputs] local shares, list of TileReturn)."""
        ctx = self.ctx
        n = ctx.n
        x_local = np.asarray(x_local, dtype=np.uint64)
        B, K = x_local.shape
        blocks = encrypted.shape[0]
        result = np.zeros((B, outputs), dtype=np.uint64)
        m = Matrix(ctx, encrypted)
        try:
            m.bind_public_key(self.pk)
            tiles = []
            for tile in range(0, outputs, tile_columns):
                tile_count = min(tile_columns, outputs - tile)
                groups = [(first, min(cap, tile + tile_count - first)) for first in range(tile, tile + tile_count, cap)]
                ret = TileReturn(tile, tile_count, np.zeros((len(groups), ctx.dk, n), dtype=np.uint64), [])
                for g0 in range(0, len(groups), self.group_chunk):
                    chunk = groups[g0:g0 + self.group_chunk]
                    ring = np.zeros((len(chunk), blocks, n), dtype=np.uint64)
                    tg = []
                    for gi, (first, count) in enumerate(chunk):
                        wblocks = []
                        for blk in range(blocks):
                            begin = blk * d
                            actual = min(d, K - begin)
                            w = reader(begin, actual, first, count)
                            if len(w) != count or any(len(row) != actual for row in w):
                                raise RuntimeError("E_BFV_WEIGHT_BLOCK_SHAPE")
                            w = np.asarray(w, dtype=np.uint64).reshape(count, actual) & np.uint64(MASK59)
                            wblocks.append(w)
                            # local share: x_S . W (mod 2^59), bfv_matrix.inc:158-159
                            result[:, first:first + count] += x_local[:, begin:begin + actual] @ w.T
                        ring[gi] = pack_weights(wblocks, d, batch, n)
                        tg.append(target_list(count, batch, d))
                    masks = self.masks(len(chunk))
                    samples = self.samples(len(chunk))
                    c1, c0, crt = m.evaluate_groups(ring, tg, mask=masks, samples=samples, crt=True)
                    for gi, (first, count) in enumerate(chunk):
                        ret.c1[g0 + gi] = c1[gi]
                        ret.targets.append(tg[gi])
                        for i, t in enumerate(tg[gi]):
                            o, b = divmod(i, batch)
                            result[b, first + o] += masks[gi, t]
                            ret.c0_phase.append(sum(int(crt[gi, i, l]) << (64 * l) for l in range(ctx.dk)))
                tiles.append(ret)
            result &= np.uint64(MASK59)
            return result, tiles
        finally:
            c = m.close()
            if not c["closed"] or c["first_cuda_error"]:
                raise RuntimeError("E_MATRIX_GPU_CLEANUP")


class MatrixClient:
    """Client role: encrypts the packed input blocks (PublicZero + Delta-scaled plaintext)
    and computes c1*s at the targets of each returned c1 (the client phase)."""

    def __init__(self, ctx: Context, pk: np.ndarray, sk_ntt: np.ndarray,
                 samples: Callable[[int], np.ndarray] | None = None):
        self.ctx = ctx
        self.pk = pk
        self.sk_ntt = np.ascontiguousarray(np.asarray(sk_ntt, dtype=np.uint64)[: ctx.dk])
        self.samples = samples or (lambda g: urandom_enc0_samples(ctx.primes, g, ctx.n))

    def encrypt_inputs(self, packed: np.ndarray) -> np.ndarray:
        pz = PublicZero(self.ctx, self.pk)
        try:
            s = self.samples(packed.shape[0])
            return np.stack([pz.encrypt(s[b], packed[b]) for b in range(packed.shape[0])])
        finally:
            pz.close()

    def phases(self, tiles: list) -> list:
        """For every target of every returned c1: (c1*s)[target] as an integer in [0,Q)."""
        ctx = self.ctx
        primes = ctx.primes[: ctx.dk]
        Q = 1
        for q in primes:
            Q *= q
        inv = [pow(Q // q % q, -1, q) for q in primes]
        out = []
        nb = NttBatch(ctx, key_level=False, batches=1)
        try:
            nb.bind_client_key(self.sk_ntt)
            for t in tiles:
                vals = []
                for g in range(t.c1.shape[0]):
                    u = nb.client_phase(t.c1[g][None])[0]
                    for tg in t.targets[g]:
                        acc = 0
                        for p, q in enumerate(primes):
                            acc += (int(u[p, tg]) * inv[p] % q) * (Q // q)
                        vals.append(acc % Q)
                out.append(vals)
            return out
        finally:
            nb.close()


def plan(batch: int, inner: int, outputs: int):
    """(d, cap, input blocks, tile columns) of a private_matrix / private_linear call."""
    if inner <= MATRIX_INNER_MAX:
        p = matrix_packing(batch, inner, outputs)
        return p.reduction, p.columns, p.inputs, 512 // batch
    if batch != 1:
        raise ProtocolShapeError("E_SHAPE")
    blocks = 1 + (inner - 1) // LINEAR_BLOCK
    if blocks > LINEAR_BLOCKS_MAX:
        raise ProtocolShapeError("E_SHAPE")
    d = LINEAR_BLOCK
    return d, packed_bfv_rows_per_ciphertext(d), blocks, 512


def validate(x_shape, outputs: int, fx: int, fw: int, linear: bool = False) -> None:
    """The public checks of private_matrix_impl / private_linear_streamed
    (bfv.cpp:598-603, :598-601) before any material is produced."""
    B, K = x_shape
    if fx > 58 or fw > 58 or fx + fw > 58 or not outputs or outputs > MATRIX_COLUMNS_MAX or not K or not B:
        raise ProtocolShapeError("E_SHAPE")
    if linear:
        if B != 1 or K > LINEAR_BLOCKS_MAX * LINEAR_BLOCK:
            raise ProtocolShapeError("E_SHAPE")
    elif B > MATRIX_BATCH_MAX or K > MATRIX_INNER_MAX:
        raise ProtocolShapeError("E_SHAPE")


def pack_client_inputs(x_client: np.ndarray, d: int, blocks: int, n: int) -> np.ndarray:
    """The client's packed input polynomials (bfv_matrix.inc:25-29; merged blocks of
    bfv.cpp:640-646 are the same rule with d = 8192, B = 1)."""
    return pack_inputs(np.asarray(x_client, dtype=np.uint64), d, blocks, n)

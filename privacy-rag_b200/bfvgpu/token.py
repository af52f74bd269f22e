"""Token lookup tile on the device (the reference's `token_packed_many`,
bfv_token_batch.inc:126-304, server side).

Per 512-coordinate tile the reference evaluates each coordinate's raw product
(`TokenWeights::evaluate_device`: the 19 input blocks times that coordinate's weight rows,
INTT, local share added at coefficient 8191, shifted by X^(2n-8191)) and folds it into a
binary-counter stack of `pack_pair` merges (bfv_acyclic_pack.hpp:45-54): 511 merges, two
keyswitches each, one coordinate at a time.  The merges form a fixed binary tree -- level l
merges pairs of 2^l-coordinate blocks with that level's two keys -- so here the raw products
of many coordinates run as one batched launch pair and the tree runs level by level, every
merge of a level in one launch sequence.  The result is the same ciphertext, bit for bit.
"""
from __future__ import annotations

from .backend import Context

TILE = 512
LEVELS = 9


def packed_target(coordinate: int) -> int:
    """Coefficient of coordinate's value in the packed tile (bfv_acyclic_pack.hpp:55-58): the
    9-bit reversal of the coordinate, times 32."""
    r = 0
    for j in range(LEVELS):
        r = (r << 1) | ((coordinate >> j) & 1)
    return r * 32


class TokenTile:
    """inputs_ntt [19][slots][2][dk][n] (device, NTT form), keys_one / keys_level: per level the
    device keys [dk][2][k][n] for elements 1 and 2^(level+1)+1.  run() takes a tile's weight
    rows ring [coords][19 * 8192] and local shares [coords][slots] (device) and returns the
    packed tile [slots][2][dk][n].  Allocations and launches go to the context stream."""

    def __init__(self, torch, ctx: Context, inputs_ntt, slots: int, keys_one, keys_level, coords: int = TILE,
                 chunk: int = 64):
        if coords & (coords - 1) or coords < 2 or coords > TILE:
            raise ValueError("E_TOKEN_BATCH_SHAPE")
        self.torch, self.ctx = torch, ctx
        self.inputs, self.slots, self.coords = inputs_ntt, slots, coords
        self.keys_one, self.keys_level = list(keys_one), list(keys_level)
        self.levels = coords.bit_length() - 1
        if len(self.keys_one) < self.levels or len(self.keys_level) < self.levels:
            raise ValueError("E_TOKEN_KEYS")
        self.chunk = min(chunk, coords)
        t, n, dk = torch, ctx.n, ctx.dk
        dev = inputs_ntt.device
        self.stream = torch.cuda.ExternalStream(ctx.stream())
        with torch.cuda.stream(self.stream):
            self.raw = t.empty((coords, slots, 2, dk, n), dtype=t.int64, device=dev)
            self.tscratch = t.empty(ctx.token_many_scratch_words(self.chunk, slots), dtype=t.int64, device=dev)
            self.pscratch = t.empty(ctx.packing_level_scratch_words((coords // 2) * slots), dtype=t.int64,
                                    device=dev)
            self.levels_out = [t.empty((coords >> (l + 1), slots, 2, dk, n), dtype=t.int64, device=dev)
                               for l in range(self.levels)]

    def finish(self, packed, masks, samples, pk):
        """The tile return (bfv_token_batch.inc:266-283): packed [slots][2][dk][n] from run(),
        masks [slots][n] ring-59 words, samples [slots][3][k][n] Enc(0) randomness, pk
        [2][k][n] (NTT form).  Returns (out, c0_crt): out [slots][2][dk][n] = packed - Delta
        masks + Enc(0) (c1 is what the reference sends) and c0_crt [slots][512][dk] the CRT of
        c0 at packed_target(coordinate) for coordinates 0..511 (device tensors; the masks at
        those targets stay with the caller)."""
        if self.coords != TILE:
            raise ValueError("E_TOKEN_BATCH_SHAPE: the tile return needs the full 512-coordinate tree")
        t, ctx = self.torch, self.ctx
        with t.cuda.stream(self.stream):
            if not hasattr(self, "fscratch"):
                dev = self.inputs.device
                self.fscratch = t.empty(ctx.token_finish_scratch_words(self.slots), dtype=t.int64, device=dev)
                self.fout = t.empty((self.slots, 2, ctx.dk, ctx.n), dtype=t.int64, device=dev)
                self.fcrt = t.empty((self.slots, TILE, ctx.dk), dtype=t.int64, device=dev)
            ctx.token_finish_device(packed, self.slots, masks, samples, pk, self.fscratch, self.fout, self.fcrt,
                                    stream=ctx.stream())
        return self.fout, self.fcrt

    def run(self, ring, local):
        ctx, s = self.ctx, self.ctx.stream()
        for c0 in range(0, self.coords, self.chunk):
            m = min(self.chunk, self.coords - c0)
            ctx.token_evaluate_many_device(self.inputs, self.slots, ring[c0:c0 + m], m, local[c0:c0 + m],
                                           self.tscratch, self.raw[c0:c0 + m], stream=s)
        cur = self.raw
        for level in range(self.levels):
            out = self.levels_out[level]
            ctx.packing_level_device(cur, out.shape[0], self.slots, level, self.keys_one[level],
                                     self.keys_level[level], self.pscratch, out, stream=s)
            cur = out
        return cur[0]

"""Device-resident server pipeline for the linear layers of one decoder layer.

``Transformer::layer_from_shares`` (IV1/compute/model.hpp:173-238) runs four
``private_matrix`` calls per 16-token tile -- q/k/v joint, o, gate/up joint, down
(``project_joint_many`` / ``project_many``, model.hpp:66-126) -- each packed by
``matrix_packing(B, K, O)``.  This module runs the server side of those calls with every
buffer resident in HBM: the layer's weights are packed into ring polynomials on the
device and transformed once per layer (the reference transforms them again in every
call, bfv_matrix.inc:186-193), then each tile's inputs are transformed once and every
projection runs as one multi-tile product (each NTT-form weight word read once for all
tiles), the INTT with the mask and Enc(0) folded in, and the target gather with CRT.
Torch provides device memory; all arithmetic is the library's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

from .backend import Context
from .layout import MASK59, matrix_packing

QWEN3_06B_LAYER = (("qkv", 1024, 4096), ("o", 2048, 1024), ("gate_up", 1024, 6144), ("down", 3072, 1024))


@dataclass(frozen=True)
class Projection:
    name: str
    inner: int        # K
    outputs: int      # O
    batch: int        # B
    d: int
    cap: int
    inputs: int       # I: input ciphertexts
    groups: int       # G: returned ciphertexts

    @property
    def stride(self) -> int:
        return 2 * self.d - 1


def plan(name: str, batch: int, inner: int, outputs: int) -> Projection:
    p = matrix_packing(batch, inner, outputs)
    groups = (outputs + p.columns - 1) // p.columns
    # one tile of 512/B columns holds whole groups for these shapes (cap divides 512/B)
    return Projection(name, inner, outputs, batch, p.reduction, p.columns, p.inputs, groups)


def pack_weights_device(torch, w_ring, pr: Projection, n: int):
    """w_ring: int64 [O][K] ring-59 words (device) -> ring polys [G][I][n] (device):
    row o of group g, column j of block b at coefficient o*B*(2d-1)+d-1-j."""
    G, I, cap, d = pr.groups, pr.inputs, pr.cap, pr.d
    O_pad, K_pad = G * cap, I * d
    w = torch.zeros((O_pad, K_pad), dtype=torch.int64, device=w_ring.device)
    w[: pr.outputs, : pr.inner] = w_ring & MASK59
    w = w.view(G, cap, I, d).permute(0, 2, 1, 3).reshape(G, I, cap * d)
    o = torch.arange(cap, device=w_ring.device).view(cap, 1)
    j = torch.arange(d, device=w_ring.device).view(1, d)
    pos = (o * pr.batch * pr.stride + d - 1 - j).reshape(-1)
    ring = torch.zeros((G, I, n), dtype=torch.int64, device=w_ring.device)
    ring[:, :, pos] = w
    return ring


def targets_device(torch, pr: Projection, device, tiles: int = 1):
    """[tiles*G][cap*B] target coefficients and [tiles*G] counts (int64 / int32 tensors)."""
    cnt = [min(pr.cap, pr.outputs - g * pr.cap) * pr.batch for g in range(pr.groups)] * tiles
    mx = pr.cap * pr.batch
    idx = torch.arange(mx, device=device)
    tg = (idx * pr.stride + pr.d - 1).repeat(tiles * pr.groups, 1).contiguous()  # (o*B+b)*(2d-1)+d-1
    counts = torch.tensor(cnt, dtype=torch.int32, device=device)
    return tg, counts, mx


class LayerServer:
    """Server-side linear protocol of one layer on one device (ART-002 context), for
    `tiles` token tiles at a time: the tiles of a prefill share every weight matrix, so
    each projection runs as one multi-tile product that reads the NTT-form weights once."""

    def __init__(self, torch, ctx: Context, pk_device, projections=QWEN3_06B_LAYER, batch: int = 16,
                 tiles: int = 1):
        """projections: (name, K, O) triples planned here with matrix_packing(batch, K, O), or
        Projection records (a shard of a larger call keeps the call's packing)."""
        self.torch = torch
        self.ctx = ctx
        self.pk = torch.empty((2, ctx.k, ctx.n, 2), dtype=torch.int64, device=pk_device.device)
        ctx.matrix_tiles_prepare_pk_device(pk_device, self.pk)
        self.proj = [p if isinstance(p, Projection) else plan(p[0], batch, p[1], p[2]) for p in projections]
        self.batch = batch
        self.tiles = tiles
        t, n, dk = torch, ctx.n, ctx.dk
        dev = pk_device.device
        maxg = max(p.groups for p in self.proj)
        maxi = max(p.inputs for p in self.proj)
        self.w_ntt = {}
        self.inp = t.empty(tiles * maxi * 2 * dk * n, dtype=t.int64, device=dev)  # transformed inputs
        self.scratch_words = max(1, ctx.matrix_tiles_scratch_words(tiles, maxg))
        self.scratch = t.empty(self.scratch_words, dtype=t.int64, device=dev)
        self.protect_slots = None  # two more scratch buffers, allocated by the first prepare_protection
        self.out = t.empty(tiles * maxg * 2 * dk * n, dtype=t.int64, device=dev)
        self.targets = {p.name: targets_device(t, p, dev, tiles) for p in self.proj}
        mx = max(v[2] for v in self.targets.values())
        self.selected = t.empty((tiles * maxg, dk, mx), dtype=t.int64, device=dev)
        self.crt = t.empty((tiles * maxg, mx, dk), dtype=t.int64, device=dev)

    def prepare_weights(self, ring_by_name: dict, stream=None) -> None:
        """Lift + NTT every weight block of the layer once (reused by all tiles)."""
        for p in self.proj:
            ring = ring_by_name[p.name]
            w = self.w_ntt.get(p.name)
            if w is None:
                w = self.torch.empty((p.groups, p.inputs, self.ctx.dk, self.ctx.n), dtype=self.torch.int64,
                                     device=ring.device)
                self.w_ntt[p.name] = w
            self.ctx.weights_ntt_device(ring, p.groups * p.inputs, w, stream=stream)

    def prepare_weights_from(self, weights, layer: int, rows_of=None, stream=None) -> None:
        """Lift + NTT the calls of decoder layer `layer` from a QuantizedWeights set (the
        reference's quantized f12 directory).  rows_of(projection) -> (lo, hi) selects a shard
        of each call's stacked rows (default: all of them)."""
        from .weights import ring_words
        rings = {}
        calls = dict(weights.layer_calls(layer))
        for p in self.proj:
            mats = calls[p.name]
            rows = rows_of(p) if rows_of else None
            w = self.torch.from_numpy(ring_words(mats, rows)).to(self.pk.device)
            if w.shape != (p.outputs, p.inner):
                raise ValueError("BAD_SHAPE")
            rings[p.name] = pack_weights_device(self.torch, w, p, self.ctx.n)
        self.prepare_weights(rings, stream=stream)

    def output(self, p: Projection):
        """[tiles][G][2][dk][n] view of the last run of projection p."""
        n, dk = self.ctx.n, self.ctx.dk
        return self.out[: self.tiles * p.groups * 2 * dk * n].view(self.tiles, p.groups, 2, dk, n)

    def gathered(self, p: Projection):
        """Views of the last run of projection p: target c0 residues [tiles*G][dk][cap*B] and
        their CRT limbs [tiles*G][cap*B][dk] (entries past a group's count are unset)."""
        e, dk, mx = self.tiles * p.groups, self.ctx.dk, self.targets[p.name][2]
        return (self.selected.view(-1)[: e * dk * mx].view(e, dk, mx),
                self.crt.view(-1)[: e * mx * dk].view(e, mx, dk))

    def prepare_protection(self, p: Projection, masks, samples, slot: int, stream=None) -> None:
        """The Enc(0) preparation and additive output term of a later run of projection p
        into protection slot `slot` (0/1), on `stream` -- ahead of the call's inputs, which
        they do not depend on.  The caller orders it after the previous reader of the slot and
        before the run that consumes it (run_projection(..., protected=slot))."""
        if self.protect_slots is None:
            self.protect_slots = [self.torch.empty(self.scratch_words, dtype=self.torch.int64,
                                                   device=self.scratch.device) for _ in range(2)]
        self.ctx.matrix_tiles_protect_device(self.tiles, p.groups, self.protect_slots[slot], masks=masks,
                                             samples=samples, pk_prep=self.pk, stream=stream)

    def run_projection(self, p: Projection, cts, masks, samples, stream=None, transformed=None, protected=None):
        """One private_matrix call for every tile: cts [tiles][I][2][dk][n] client ciphertexts
        in coefficient form (left unchanged; their transform goes to self.inp), or None with
        `transformed` holding them already in the product's operand form (InputExchange);
        masks [tiles][G][n], samples [tiles][G][3][k][n].  With `protected` = a slot filled by
        prepare_protection, the call reads that slot instead of preparing Enc(0) and the mask
        itself.  Leaves the re-randomised results in output(p) (c1 goes to the client) and the
        targets' c0 residues / CRT limbs in self.selected / self.crt."""
        ctx = self.ctx
        I, G, T = p.inputs, p.groups, self.tiles
        if transformed is None:
            transformed = self.inp
            ctx.matrix_tiles_inputs_device(cts, T * I, out=transformed, stream=stream)
        if protected is None:
            ctx.matrix_tiles_device(transformed, T, I, self.w_ntt[p.name], G, self.out, masks=masks, samples=samples,
                                    pk_prep=self.pk, scratch=self.scratch, stream=stream)
        else:  # masks / samples only say which parts prepare_protection had
            ctx.matrix_tiles_prepared_device(transformed, T, I, self.w_ntt[p.name], G, self.out,
                                             enc0=samples is not None, masked=masks is not None, pk_prep=self.pk,
                                             scratch=self.protect_slots[protected], stream=stream)
        tg, counts, mx = self.targets[p.name]
        ctx.gather_targets_device(self.out, T * G, tg, counts, mx, self.selected, self.crt, stream=stream)

"""Output-group sharding of the matrix protocol across the GPUs of one node.

In one ``private_matrix`` call (IV1/native/src/bfv_matrix.inc:150-233) every output group
-- one returned ciphertext and its targets -- depends only on the shared input
ciphertexts and its own rows of the weight matrix, so the groups of a call split into
contiguous ranges, one per rank, with no exchange during the computation.  Each rank packs
and transforms only its rows, evaluates its groups for every tile, and the results (c1 for
the client and the targets' c0 as CRT limbs) are gathered to the protocol rank over NCCL,
the only collective on the path.  The packing is the whole call's (``matrix_packing`` of
the full shape), so a shard's groups are exactly the unsharded call's groups lo..hi-1.
"""
from __future__ import annotations

import dataclasses

from .layer import Projection


def group_range(groups: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced range [lo, hi) of the groups that `rank` evaluates."""
    return groups * rank // world, groups * (rank + 1) // world


def shard_projection(p: Projection, rank: int, world: int) -> tuple[Projection, int, int]:
    """The rank's part of projection p (same packing; rows lo*cap .. min(hi*cap, O)) and the
    range of global groups it covers."""
    lo, hi = group_range(p.groups, rank, world)
    rows = max(0, min(hi * p.cap, p.outputs) - lo * p.cap)
    return dataclasses.replace(p, outputs=rows, groups=hi - lo), lo, hi


def weight_rows(w, p: Projection, rank: int, world: int):
    """Rows of the [O][K] weight matrix that the rank's groups use."""
    lo, hi = group_range(p.groups, rank, world)
    return w[lo * p.cap: min(hi * p.cap, p.outputs)]


def gather_groups(torch, dist, local, groups: int, world: int, dst: int = 0, async_op: bool = False,
                  group=None):
    """Gather per-rank results [tiles][g_local][...] into the protocol rank's
    [tiles][groups][...] in global group order (over `group`, default the world; dst is a
    global rank).  Blocks are padded to the widest shard so
    that every rank takes the same collective step (ranks without groups send an empty
    block).  Returns the assembled tensor on `dst` (None elsewhere), or (work, finish) if
    async_op, where finish() assembles after the work completes."""
    tiles = local.shape[0]
    tail = tuple(local.shape[2:])
    per = [group_range(groups, r, world) for r in range(world)]
    width = max(hi - lo for lo, hi in per)
    if local.shape[1] == width and local.is_contiguous():
        pad = local
    else:
        pad = torch.zeros((tiles, width) + tail, dtype=local.dtype, device=local.device)
        pad[:, : local.shape[1]] = local
    rank = dist.get_rank()
    bufs = [torch.empty_like(pad) for _ in range(world)] if rank == dst else None
    work = dist.gather(pad, gather_list=bufs, dst=dst, async_op=async_op, group=group)

    def finish():
        if rank != dst:
            return None
        return torch.cat([bufs[r][:, : hi - lo] for r, (lo, hi) in enumerate(per)], dim=1)

    if async_op:
        return work, finish
    return finish()


class GroupGather:
    """gather_groups with its buffers allocated once, for calls repeated with one shape: the
    padded send block `send` [tiles][width][...] (width = the widest shard; a rank writes its
    groups into send[:, :g_local], e.g. from a captured CUDA graph) and, on the protocol rank,
    one receive block per rank.  start() issues the same collective step as gather_groups;
    result() assembles [tiles][groups][...] in global group order once it has completed."""

    def __init__(self, torch, dist, tiles: int, groups: int, tail: tuple, dtype, device, dst: int = 0,
                 group=None):
        self.torch, self.dist, self.dst, self.group = torch, dist, dst, group
        world = dist.get_world_size(group)
        self.per = [group_range(groups, r, world) for r in range(world)]
        width = max(hi - lo for lo, hi in self.per)
        self.send = torch.zeros((tiles, width) + tuple(tail), dtype=dtype, device=device)
        self.rank = dist.get_rank()
        self.recv = [torch.empty_like(self.send) for _ in range(world)] if self.rank == dst else None

    def start(self, async_op: bool = True):
        return self.dist.gather(self.send, gather_list=self.recv, dst=self.dst, async_op=async_op, group=self.group)

    def result(self):
        if self.rank != self.dst:
            return None
        return self.torch.cat([self.recv[r][:, : hi - lo] for r, (lo, hi) in enumerate(self.per)], dim=1)


class InputExchange:
    """One call's client ciphertexts from the protocol rank to every rank in the product's
    operand form, with the transform itself sharded: the protocol rank scatters equal slices
    of the batch, each rank transforms its slice, and an all-gather assembles the whole
    transformed batch on every rank (the same bytes on the links as a broadcast, a 1/world
    share of the transform).  `count` ciphertexts of `words` words each are padded to a
    multiple of world; the padding slots carry no data anyone reads."""

    def __init__(self, torch, dist, group, count: int, words: int, device, src: int = 0):
        self.torch, self.dist, self.group, self.src = torch, dist, group, src
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.per = -(-count // self.world)
        self.count, self.words = count, words
        self.slice_in = torch.empty((self.per, words), dtype=torch.int64, device=device)
        self.slice_out = torch.empty((self.per, words), dtype=torch.int64, device=device)
        self.full = torch.empty((self.per * self.world, words), dtype=torch.int64, device=device)

    def scatter(self, source, async_op: bool = True):
        """source [count][words] on the protocol rank (ignored elsewhere) -> this rank's slice."""
        chunks = None
        if self.rank == self.src:
            flat = source.reshape(-1, self.words)
            if flat.shape[0] != self.count:
                raise ValueError("BAD_SHAPE")
            chunks = [flat[r * self.per:(r + 1) * self.per] for r in range(self.world)]
            if chunks[-1].shape[0] < self.per:  # pad the last chunk
                pad = self.torch.zeros((self.per, self.words), dtype=flat.dtype, device=flat.device)
                pad[: chunks[-1].shape[0]] = chunks[-1]
                chunks[-1] = pad
            chunks = [c.contiguous() for c in chunks]
        return self.dist.scatter(self.slice_in, chunks, src=self.src, group=self.group, async_op=async_op)

    def gather(self, transform, async_op: bool = True):
        """transform(slice_in, slice_out, slots) on this rank's slice, then the all-gather into
        self.full ([per*world][words]; rows past `count` are padding)."""
        transform(self.slice_in, self.slice_out, self.per)
        return self.dist.all_gather_into_tensor(self.full, self.slice_out, group=self.group, async_op=async_op)

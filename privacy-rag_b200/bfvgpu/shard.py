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

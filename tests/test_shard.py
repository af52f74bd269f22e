"""Output-group sharding (bfvgpu.shard) on CPU: the shards of a call are exactly the
unsharded call's groups -- packing, weight polynomials and targets -- and the gather to the
protocol rank reassembles the global group order.  The gather runs as world_size-2 and
world_size-3 `gloo` process groups on 127.0.0.1 (the NCCL path on the GPUs takes the same
collective steps)."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "privacy-rag_b200"))

from bfvgpu import layer as L  # noqa: E402
from bfvgpu import shard as S  # noqa: E402


@pytest.mark.parametrize("groups,world", [(32, 8), (16, 3), (5, 8), (192, 7)])
def test_group_ranges_partition(groups, world):
    seen = []
    for r in range(world):
        lo, hi = S.group_range(groups, r, world)
        assert 0 <= lo <= hi <= groups
        seen.extend(range(lo, hi))
    assert seen == list(range(groups))


@pytest.mark.parametrize("batch,K,O,world", [(16, 1024, 4096, 8), (1, 3072, 1024, 3), (16, 300, 200, 2)])
def test_shard_packing_matches_whole_call(batch, K, O, world):
    """Each shard's weight polynomials and targets are the corresponding slices of the
    unsharded call's (CPU torch tensors, n = 16384)."""
    import torch
    n = 16384
    p = L.plan("x", batch, K, O)
    rng = np.random.default_rng(K + O)
    w = torch.from_numpy(rng.integers(-127, 128, size=(O, K)).astype(np.int64))
    full = L.pack_weights_device(torch, w, p, n)
    tg_full, cnt_full, mx = L.targets_device(torch, p, "cpu")
    rows = 0
    for r in range(world):
        sp, lo, hi = S.shard_projection(p, r, world)
        assert (sp.d, sp.cap, sp.inputs, sp.batch) == (p.d, p.cap, p.inputs, p.batch)
        wr = S.weight_rows(w, p, r, world)
        assert wr.shape[0] == sp.outputs
        rows += sp.outputs
        if sp.groups == 0:
            continue
        assert torch.equal(L.pack_weights_device(torch, wr, sp, n), full[lo:hi])
        tg, cnt, mxs = L.targets_device(torch, sp, "cpu")
        assert mxs == mx and torch.equal(tg, tg_full[lo:hi]) and torch.equal(cnt, cnt_full[lo:hi])
    assert rows == O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, groups, tiles, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = S.group_range(groups, rank, world)
        t = torch.arange(tiles).view(tiles, 1, 1)
        g = torch.arange(lo, hi).view(1, -1, 1)
        e = torch.arange(3).view(1, 1, 3)
        local = (t * 100000 + g * 10 + e).to(torch.int64).contiguous()   # [tiles][g_local][3]
        got = S.gather_groups(torch, dist, local, groups, world)
        work, finish = S.gather_groups(torch, dist, local * 2, groups, world, async_op=True)
        work.wait()
        got2 = finish()
        if rank == 0:
            tt = torch.arange(tiles).view(tiles, 1, 1)
            gg = torch.arange(groups).view(1, -1, 1)
            want = (tt * 100000 + gg * 10 + e).to(torch.int64)
            q.put(bool(torch.equal(got, want)) and bool(torch.equal(got2, want * 2)))
        else:
            q.put(got is None and got2 is None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,groups", [(2, 7), (3, 2)])
def test_gather_groups_gloo(world, groups):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, groups, 2, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert all(res)


def _exchange_worker(rank, world, port, count, words, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex = S.InputExchange(torch, dist, None, count, words, "cpu")
        source = (torch.arange(count * words, dtype=torch.int64).view(count, words) * 7 + 5) if rank == 0 else None
        seen = []

        def transform(si, so, slots):
            seen.append(int(slots))
            so.copy_(si * 3 + 1)

        w = ex.scatter(source)
        w.wait()
        g = ex.gather(transform)
        g.wait()
        want = (torch.arange(count * words, dtype=torch.int64).view(count, words) * 7 + 5) * 3 + 1
        q.put(bool(torch.equal(ex.full[:count], want)) and seen == [ex.per])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,count", [(2, 8), (3, 7)])
def test_input_exchange_gloo(world, count):
    """Scatter from the protocol rank, per-rank transform of the slice, all-gather: every
    rank ends with the transform of the whole batch (count not a multiple of world: the
    padding is ignored)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, count, 5, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert all(res)

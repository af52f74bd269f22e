"""Output-group sharding over NCCL on two GPUs: the sharded call equals the 1-GPU call.

The config-5 multi-GPU design splits every private_matrix call's output groups into
contiguous ranges, one per rank (bfvgpu.shard).  Here two ranks run, over NCCL:

* one prefill call (the o projection of a 128-token group: B = 16, K = 2048, O = 1024, 8 tiles
  x 64 inputs x 64 groups) whose inputs travel through InputExchange -- rank 0 scatters the
  raw ciphertexts, each rank transforms its slice, an all-gather assembles the operand -- and
* one decode call (the qkv projection of one token: B = 1, K = 1024, O = 4096, 16 inputs x 32
  groups) whose inputs are broadcast and transformed locally, with its output protection
  prepared ahead in a protection slot, as the bench's decode calls run.

Each rank packs and transforms only its rows of the weights and evaluates only its groups;
gather_groups brings c1 and the targets' CRT limbs to rank 0, where they must equal, bit for
bit, the unsharded call run by a single LayerServer on rank 0's GPU with the same inputs,
masks and Enc(0) randomness.  Kernels read only their own GPU's memory; NCCL moves the data.
Needs two GPUs (skipped otherwise).
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(HERE, "..", "privacy-rag_b200")
CALLS = (("prefill", 16, 8, ("o", 2048, 1024)), ("decode", 1, 1, ("qkv", 1024, 4096)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch
    import torch.distributed as dist
    sys.path.insert(0, PKG)
    import bfvgpu
    from bfvgpu import layer as L
    from bfvgpu import shard as S
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    result = {}
    try:
        ctx = bfvgpu.Context.art002(rank)
        # torch's allocations, copies and collectives ordered with the library's kernels
        with torch.cuda.stream(torch.cuda.ExternalStream(ctx.stream())):
            _calls(torch, dist, L, S, ctx, rank, world, result)
        q.put((rank, result))
    except Exception as e:  # report, so the parent fails with the cause instead of a timeout
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _calls(torch, dist, L, S, ctx, rank, world, result):
    n, k, dk = ctx.n, ctx.k, ctx.dk
    qd = torch.tensor(ctx.primes, dtype=torch.int64, device="cuda")
    rng = np.random.default_rng(77)  # the same stream on every rank
    residues = lambda a, m: torch.remainder(torch.from_numpy(a).cuda(), qd[:m].view(m, 1))
    pk = residues(rng.integers(0, 1 << 62, size=(2, k, n), dtype=np.int64), k)
    for phase, B, T, (name, K, O) in CALLS:
        full = L.plan(name, B, K, O)
        sp, lo, hi = S.shard_projection(full, rank, world)
        W = torch.from_numpy(rng.integers(-127, 128, size=(O, K), dtype=np.int64)).cuda()
        masks = torch.from_numpy(rng.integers(0, 1 << 59, size=(T, full.groups, n), dtype=np.int64)).cuda()
        small = np.concatenate([rng.integers(-1, 2, size=(T, full.groups, 1, n)),
                                rng.integers(-5, 6, size=(T, full.groups, 2, n))], axis=2)
        samples = torch.remainder(torch.from_numpy(small).cuda().unsqueeze(-2), qd.view(k, 1)).contiguous()
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1000 + len(name))
        cts = torch.remainder(torch.randint(0, 2 ** 62, (T, full.inputs, 2, dk, n), dtype=torch.int64,
                                            device="cuda", generator=gen), qd[:dk].view(dk, 1))
        if rank != 0:
            cts.zero_()  # only the protocol rank holds the client's ciphertexts
        srv = L.LayerServer(torch, ctx, pk, [sp], B, T)
        srv.crt.zero_()
        srv.prepare_weights({name: L.pack_weights_device(torch, S.weight_rows(W, full, rank, world), sp, n)})
        m_loc, s_loc = masks[:, lo:hi].contiguous(), samples[:, lo:hi].contiguous()
        if phase == "prefill":
            ex = S.InputExchange(torch, dist, None, T * full.inputs, 2 * dk * n, "cuda")
            ex.scatter(cts).wait()
            ex.gather(lambda si, so, slots: ctx.matrix_tiles_inputs_device(si, slots, out=so)).wait()
            srv.run_projection(sp, None, m_loc, s_loc, transformed=ex.full)
        else:
            dist.broadcast(cts, src=0)
            srv.prepare_protection(sp, m_loc, s_loc, 0)
            srv.run_projection(sp, cts, m_loc, s_loc, protected=0)
        torch.cuda.synchronize()
        c1 = srv.output(sp)[:, :, 1].contiguous()
        crt = srv.gathered(sp)[1].view(T, sp.groups, -1, dk).contiguous()
        got_c1 = S.gather_groups(torch, dist, c1, full.groups, world)
        got_crt = S.gather_groups(torch, dist, crt, full.groups, world)
        if rank == 0:
            one = L.LayerServer(torch, ctx, pk, [full], B, T)
            one.crt.zero_()
            one.prepare_weights({name: L.pack_weights_device(torch, W, full, n)})
            one.run_projection(full, cts, masks, samples)
            torch.cuda.synchronize()
            want_c1 = one.output(full)[:, :, 1]
            want_crt = one.gathered(full)[1].view(T, full.groups, -1, dk)
            result[phase] = (bool(torch.equal(got_c1, want_c1)), bool(torch.equal(got_crt, want_crt)),
                             ctx.check())
            del one
        del srv
        torch.cuda.empty_cache()


def test_sharded_calls_equal_single_gpu():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    assert res[1] == {}, res[1]
    assert res[0] == {"prefill": (True, True, 0), "decode": (True, True, 0)}, res[0]

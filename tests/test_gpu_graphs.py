"""Decode calls replayed as captured CUDA graphs equal the same calls issued eagerly.

The config-5 decode calls (one token, B = 1) are short chains of small launches; the bench
captures each (layer, projection) call once and replays it.  A captured call has two branches:
on the side stream, the next call's output protection (Enc(0) preparation and additive term)
into the other protection slot; on the context stream, this call's input transform, product,
protected output transform and target gather.  Two projections alternate slots 0 and 1 the way
consecutive decode calls do.  Every replay's c1 and target CRT limbs must equal an eager
LayerServer call on the same inputs, masks and Enc(0) randomness, over two rounds of replays
(the second round reads protections prepared by the first).
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

PROJ = (("qkv", 1024, 4096), ("o", 2048, 1024))


def test_decode_call_graphs_equal_eager_calls(bfv):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bfvgpu import layer as L
    hc = bfv.Context.art002(0)
    n, k, dk = hc.n, hc.k, hc.dk
    stream = torch.cuda.ExternalStream(hc.stream())
    aux = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        q = torch.tensor(hc.primes, dtype=torch.int64, device="cuda")
        gen = torch.Generator(device="cuda")
        gen.manual_seed(3)
        res = lambda shape, m: torch.remainder(
            torch.randint(0, 2 ** 62, shape, dtype=torch.int64, device="cuda", generator=gen), q[:m].view(m, 1))
        pk = res((2, k, n), k)
        srv = L.LayerServer(torch, hc, pk, PROJ, 1, 1)
        ps = srv.proj
        rings, cts, masks, samples = {}, {}, {}, {}
        for p in ps:
            w = torch.randint(-127, 128, (p.outputs, p.inner), dtype=torch.int64, device="cuda", generator=gen)
            rings[p.name] = L.pack_weights_device(torch, w, p, n)
            cts[p.name] = res((1, p.inputs, 2, dk, n), dk)
            masks[p.name] = torch.randint(0, 2 ** 59, (1, p.groups, n), dtype=torch.int64, device="cuda", generator=gen)
            small = torch.cat([torch.randint(-1, 2, (1, p.groups, 1, n), device="cuda", generator=gen),
                               torch.randint(-5, 6, (1, p.groups, 2, n), device="cuda", generator=gen)], dim=2)
            samples[p.name] = torch.remainder(small.unsqueeze(-2), q.view(k, 1)).contiguous()
        srv.prepare_weights(rings)

        def results(p):
            return (srv.output(p)[:, :, 1].clone(), srv.gathered(p)[1].clone())

        eager = {}
        for p in ps:
            srv.crt.zero_()
            srv.run_projection(p, cts[p.name], masks[p.name], samples[p.name])
            eager[p.name] = results(p)
        # protection slots exist before capture (allocated by the first prepare_protection)
        srv.prepare_protection(ps[0], masks[ps[0].name], samples[ps[0].name], 0)
        torch.cuda.synchronize()

        def call(i):
            p, nxt = ps[i], ps[1 - i]
            fork = torch.cuda.Event()
            fork.record(stream)
            aux.wait_event(fork)
            srv.prepare_protection(nxt, masks[nxt.name], samples[nxt.name], 1 - i, stream=aux.cuda_stream)
            join = torch.cuda.Event()
            join.record(aux)
            srv.run_projection(p, cts[p.name], masks[p.name], samples[p.name], stream=hc.stream(), protected=i)
            stream.wait_event(join)

        graphs = []
        for i in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                call(i)
            graphs.append(g)
        # slot 0 holds ps[0]'s protection; each replay prepares the other projection's
        srv.prepare_protection(ps[0], masks[ps[0].name], samples[ps[0].name], 0)
        for rnd in range(2):
            for i, p in enumerate(ps):
                srv.crt.zero_()
                graphs[i].replay()
                got = results(p)
                torch.cuda.synchronize()
                assert torch.equal(got[0], eager[p.name][0]), (rnd, p.name, "c1")
                assert torch.equal(got[1], eager[p.name][1]), (rnd, p.name, "crt")
        assert hc.check() == 0
        del graphs

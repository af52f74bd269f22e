"""The matrix protocol end to end on the GPU path: the reference's plaintext known answers.

Each case of tests/golden/kat_linear.json (dev_bfv_packed_probe.cpp, dev_bfv_merged_probe.cpp,
dev_tile_long_probe.cpp) runs as the reference runs it: the client encrypts its packed
shares (GPU PublicZero + Delta-scaled plaintext), the server evaluates every output group
with masking and Enc(0) re-randomisation (GPU Matrix.evaluate_groups), the client computes
c1*s at the targets (GPU client phase); the decode that the garbled circuit performs is
done here in the clear (test-only), and the two parties' shares must add up to the
expected ring-59 values.  The reader callback counts are the probes' pins (26 and 1046).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def operands(case):
    cols, rows = case["columns"], case["rows"]
    j = np.arange(cols, dtype=np.int64)
    if case["generator"] == "packed":
        whole = ((j * 13 + 7) % 101) - 50
        w = np.stack([np.zeros(cols, dtype=np.int64) if r in (1, rows - 1) else ((j * (r + 3) + 5) % 17) - 8
                      for r in range(rows)])
    else:
        cid = case["case_id"]
        if cid == 1:
            whole = np.where((j == 0) | (j == 8192), 7, 0)
            w = np.zeros((rows, cols), dtype=np.int64)
            w[0, 0], w[0, 8192] = 11, -11
            w[2:, 0], w[2:, 8192] = 3, -5
        else:
            whole = ((j * 13 + 7) % 101) - 50
            w = np.stack([np.zeros(cols, dtype=np.int64) if (cid < 2 and r == 1) else ((j * (r + 3) + 5) % 17) - 8
                          for r in range(rows)])
    mask = (1 << 59) - 1
    client = ((0x1928abcdef + j.astype(np.uint64) * np.uint64(125939)) & np.uint64(mask)).astype(np.uint64)
    whole_u = (whole.astype(np.int64).astype(np.uint64)) & np.uint64(mask)
    server = (whole_u - client) & np.uint64(mask)
    w_u = w.astype(np.int64).astype(np.uint64) & np.uint64(mask)
    return client, server, w_u


@pytest.fixture(scope="module")
def setup(bfv, oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hc = bfv.Context.art002(0)
    oc = oracle.art002()
    tb = oracle.TestBfv(oc, seed=2024)
    return hc, oc, tb


def run_case(bfv, oracle, setup, case, seed):
    from bfvgpu import engine
    hc, oc, tb = setup
    rng = np.random.default_rng(seed)
    client_x, server_x, w = operands(case)
    K, rows = case["columns"], case["rows"]
    d, cap, blocks, tile = engine.plan(1, K, rows)
    calls = []

    def reader(begin, actual, first, count):
        calls.append((begin, actual, first, count))
        return w[first:first + count, begin:begin + actual]

    q = np.array(hc.primes, dtype=np.int64).reshape(1, 1, -1, 1)

    def samples(g):
        """Seeded Enc(0) randomness [g][3][k][n]: ternary u, small e0/e1."""
        u = rng.integers(-1, 2, size=(g, 1, 1, hc.n))
        e = rng.integers(-5, 6, size=(g, 2, 1, hc.n))
        return (np.concatenate([u, e], axis=1) % q).astype(np.uint64)

    client = engine.MatrixClient(hc, tb.pk, tb.sk_ntt, samples=samples)
    server = engine.MatrixServer(hc, tb.pk, masks=lambda g: rng.integers(0, 1 << 59, size=(g, hc.n), dtype=np.uint64),
                                 samples=samples)
    packed = engine.pack_client_inputs(client_x[None, :], d, blocks, hc.n)
    encrypted = client.encrypt_inputs(packed)
    result, tiles = server.run(encrypted, server_x[None, :], rows, reader, d, cap, 1, tile)
    u = client.phases(tiles)
    Q = oc.Q
    out = [int(v) for v in result[0]]
    for t, ut in zip(tiles, u):
        for i, (c0v, uv) in enumerate(zip(t.c0_phase, ut)):
            col = t.first_column + i  # B = 1: one target per output column
            out[col] = (out[col] + oracle.decode((c0v + uv) % Q, Q)) & ((1 << 59) - 1)
    assert out == case["expected"], case["probe"]
    return len(calls), blocks


def test_packed_probe_cases(bfv, oracle, setup):
    with open(os.path.join(GOLD, "kat_linear.json")) as f:
        cases = [c for c in json.load(f)["cases"] if c["probe"] == "dev_bfv_packed_probe"]
    for i, case in enumerate(cases):
        run_case(bfv, oracle, setup, case, 100 + i)


def test_merged_probe_cases_and_callback_pin(bfv, oracle, setup):
    with open(os.path.join(GOLD, "kat_linear.json")) as f:
        cases = [c for c in json.load(f)["cases"] if c["probe"] == "dev_bfv_merged_probe"]
    total = sum(run_case(bfv, oracle, setup, case, 200 + i)[0] for i, case in enumerate(cases))
    assert total == 26  # dev_bfv_merged_probe.cpp: server_callback_calls


def test_tile_long_probe_cases_and_callback_pin(bfv, oracle, setup):
    with open(os.path.join(GOLD, "kat_linear.json")) as f:
        cases = [c for c in json.load(f)["cases"] if c["probe"] == "dev_tile_long_probe"]
    total = sum(run_case(bfv, oracle, setup, case, 300 + i)[0] for i, case in enumerate(cases))
    assert total == 1046  # dev_tile_long_probe.cpp: server_callback_calls


def test_public_shape_rejections(bfv):
    from bfvgpu import engine
    for shape, outputs, fx, fw, linear in [((17, 8), 1, 12, 12, False), ((1, 8193), 1, 12, 12, False),
                                           ((1, 8), 0, 12, 12, False), ((1, 8), 155649, 12, 12, False),
                                           ((1, 8), 1, 40, 20, False), ((1, 19 * 8192 + 1), 1, 12, 12, True)]:
        with pytest.raises(engine.ProtocolShapeError):
            engine.validate(shape, outputs, fx, fw, linear=linear)


@pytest.mark.parametrize("tiles,batch,projections", [
    (3, 2, (("a", 300, 200), ("b", 130, 600))),
    (8, 2, (("a", 300, 200), ("b", 130, 600))),
    # one head's attention pair (BatchOps::matrix shapes): 16 x 128 . 128 x 1280, 16 x 1280 . 1280 x 128
    (1, 16, (("scores", 128, 1280), ("values", 1280, 128))),
])
def test_layer_server_tiles_decrypt(bfv, oracle, setup, tiles, batch, projections):
    """LayerServer (multi-tile product, folded Enc(0), mask, target gather with CRT) on small
    projections over 3 and 8 token tiles (8: the tensor-core product) and on one attention
    head pair: every target decrypts to sum_j x.w minus the mask at that coefficient (mod
    2^59), and the gathered c0 residues and CRT limbs are the output ciphertext's own."""
    import torch
    from bfvgpu import layer as L
    from bfvgpu.layout import MASK59, pack_inputs
    hc, oc, tb = setup
    n, k, dk = oc.n, oc.k, oc.data_k
    rng = np.random.default_rng(77)
    pk = torch.from_numpy(tb.pk.view(np.int64)).cuda()
    srv = L.LayerServer(torch, hc, pk, projections, batch, tiles)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()
    rings, w_int = {}, {}
    for p in srv.proj:
        w_int[p.name] = rng.integers(-127, 128, size=(p.outputs, p.inner))
        rings[p.name] = L.pack_weights_device(torch, dev(w_int[p.name].astype(np.int64).astype(np.uint64)), p, n)
    srv.prepare_weights(rings)
    for p in srv.proj:
        x = rng.integers(0, 1 << 59, size=(tiles, batch, p.inner), dtype=np.uint64)
        cts = np.stack([np.stack([tb.encrypt(poly) for poly in pack_inputs(x[t], p.d, p.inputs, n)])
                        for t in range(tiles)])
        masks = rng.integers(0, 1 << 59, size=(tiles, p.groups, n), dtype=np.uint64)
        samples = np.stack([np.stack([tb.samples() for _ in range(p.groups)]) for _ in range(tiles)])
        srv.run_projection(p, dev(cts), dev(masks), dev(samples))
        assert hc.check() == 0
        out = srv.output(p).cpu().numpy().view(np.uint64)
        tg, counts, mx = srv.targets[p.name]
        tg, counts = tg.cpu().numpy(), counts.cpu().numpy()
        sel, crt = (a.cpu().numpy().view(np.uint64) for a in srv.gathered(p))
        w_u = w_int[p.name].astype(np.int64).astype(np.uint64) & np.uint64(MASK59)
        for t in range(tiles):
            for g in range(p.groups):
                e = t * p.groups + g
                u = oc.client_phase(out[t, g, 1], tb.sk_data_ntt())
                for i in range(counts[e]):
                    z = int(tg[e, i])
                    o, b = divmod(i, batch)
                    row = g * p.cap + o
                    expect = (int((x[t, b].astype(object) * w_u[row].astype(object)).sum()) - int(masks[t, g, z])) \
                        % (1 << 59)
                    res = [(int(out[t, g, 0, q, z]) + int(u[q, z])) % oc.primes[q] for q in range(dk)]
                    assert oracle.decode(oracle.crt(res, oc.primes[:dk]), oc.Q) == expect, (p.name, t, g, i)
                    assert np.array_equal(sel[e, :, i], out[t, g, 0, :, z])
                    v = sum(int(crt[e, i, l]) << (64 * l) for l in range(dk))
                    assert v == oracle.crt(out[t, g, 0, :, z], oc.primes[:dk])


def test_layer_weights_from_quantized_directory(bfv, oracle, setup, tmp_path):
    """LayerServer.prepare_weights_from: a quantized f12 layer (the reference's checkpoint
    format) stacked per joint call, packed, lifted and transformed on the GPU equals the
    oracle's lift + NTT of the reference packing (layout.pack_weights of the reader blocks)
    for sampled (call, group, block) pairs."""
    import torch
    import test_weights as TW
    from bfvgpu import layer as L
    from bfvgpu import weights as W
    from bfvgpu.layout import pack_weights
    hc, oc, tb = setup
    n, dk = oc.n, oc.data_k
    TW.write_layer(str(tmp_path), seed=11)
    qw = W.QuantizedWeights(str(tmp_path))
    pk = torch.from_numpy(tb.pk.view(np.int64)).cuda()
    srv = L.LayerServer(torch, hc, pk, L.QWEN3_06B_LAYER, 16, 1)
    srv.prepare_weights_from(qw, 0)
    torch.cuda.synchronize()
    calls = dict(qw.layer_calls(0))
    for p, g, b in [(srv.proj[0], 0, 0), (srv.proj[0], 127, 63), (srv.proj[2], 64, 17), (srv.proj[3], 5, 47)]:
        rows = W.ring_words(calls[p.name], (g * p.cap, min((g + 1) * p.cap, p.outputs))).astype(np.uint64)
        block = rows[:, b * p.d:(b + 1) * p.d]
        ring = pack_weights([block], p.d, p.batch, n)
        lifted = oc.lift(ring)[0]
        expect = oc.ntt(lifted, prime_count=dk)
        got = srv.w_ntt[p.name][g, b].cpu().numpy().view(np.uint64)
        assert np.array_equal(got, expect), (p.name, g, b)

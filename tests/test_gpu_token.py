"""The token lookup tile at the benchmark's shape, end to end on the GPU, with real keys.

One 512-coordinate tile of one slot at ART-002, as `token_packed_many` builds it
(bfv_token_batch.inc:126-304): the client's 19 input blocks encrypted under s_0, each
coordinate's 19 x 8192 weight rows (|w| <= 2^20) and local share, the nine-level packing
tree whose level l switches s_l -> s_(l+1) with the keys of elements 1 and 2^(l+1)+1
(acyclic_keys, bfv_acyclic_pack.hpp:23-36), then the tile return (mask, Enc(0) under s_9,
CRT of c0 at the packed targets, :271-283).  Decrypting the returned tile under s_9 gives,
at packed_target(j), 512 * (x . w_j + local_j) - mask[packed_target(j)] mod 2^59: the value
the reference's decoder unscales by 2^9 (bfv_token_decoder.inc).  The returned ciphertext
also equals the oracle's sub_plain + Enc(0) + add of the packed tile word for word, and the
CRT limbs equal the CRT of its c0 residues.

The level-batched tree itself is compared with the reference's binary-counter stack of
pairwise merges at 64 coordinates (6 levels) in test_gpu_parity.py.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MASK59 = (1 << 59) - 1


def test_token_tile_decrypts_at_packed_targets(bfv, oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bfvgpu import token as TK
    hc, oc = bfv.Context.art002(0), oracle.art002()
    n, k, dk = oc.n, oc.k, oc.data_k
    rng = np.random.default_rng(2026)
    keys = [oracle.TestBfv(oc, seed=500 + l) for l in range(TK.LEVELS + 1)]  # s_0 .. s_9
    # client: 19 input blocks of ring words (a share of the one-hot row), encrypted under s_0
    x = rng.integers(0, 1 << 59, size=19 * 8192, dtype=np.uint64)
    x[:3] = [0, 1, MASK59]
    blocks = []
    for b in range(19):
        plain = np.zeros(n, dtype=np.uint64)
        plain[:8192] = x[b * 8192:(b + 1) * 8192]
        blocks.append(keys[0].encrypt(plain))
    cts = np.stack(blocks)  # [19][2][dk][n], coefficient form
    # server: weights and local shares of the 512 coordinates
    bound = 1 << 20
    w = rng.integers(-bound, bound + 1, size=(TK.TILE, 19 * 8192), dtype=np.int64)
    w[0, :4] = [bound, -bound, 0, -1]
    ring = (w & MASK59).astype(np.uint64)
    local = rng.integers(0, 1 << 59, size=(TK.TILE, 1), dtype=np.uint64)
    mask = rng.integers(0, 1 << 59, size=n, dtype=np.uint64)
    samples = keys[-1].samples()
    key_one = [keys[l].galois_key(1, target=keys[l + 1]) for l in range(TK.LEVELS)]
    key_lev = [keys[l].galois_key((2 << l) + 1, target=keys[l + 1]) for l in range(TK.LEVELS)]

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()
    stream = torch.cuda.ExternalStream(hc.stream())
    with torch.cuda.stream(stream):
        inputs = dev(cts)
        hc.ntt_device(inputs, 19 * 2 * dk, dk, stream=hc.stream())
        inputs = inputs.view(19, 1, 2, dk, n)
        tile = TK.TokenTile(torch, hc, inputs, 1, [dev(a) for a in key_one], [dev(a) for a in key_lev])
        packed = tile.run(dev(ring), dev(local))
        out, crt = tile.finish(packed, dev(mask).view(1, n), dev(samples).view(1, 3, k, n), dev(keys[-1].pk))
    torch.cuda.synchronize()
    assert hc.check() == 0
    packed_h = packed[0].cpu().numpy().view(np.uint64)  # slot 0: [2][dk][n]
    out_h = out[0].cpu().numpy().view(np.uint64)
    crt_h = crt[0].cpu().numpy().view(np.uint64)

    # the tile return equals the oracle's sub_plain + Enc(0) + add, word for word
    want = packed_h.copy()
    want[0] = oc.sub_plain(want[0], mask)
    assert np.array_equal(out_h, oc.add(want, oc.enc0(samples, keys[-1].pk)))
    # decryption under s_9 at the packed targets
    targets = [TK.packed_target(j) for j in range(TK.TILE)]
    u = oc.client_phase(out_h[1], keys[-1].sk_data_ntt())
    primes = oc.primes[:dk]
    # x . w_j mod 2^59 in wrapping 64-bit arithmetic (2^59 divides 2^64), 64 rows at a time
    dot = np.concatenate([(w[r:r + 64].astype(np.uint64) * x[None, :]).sum(axis=1, dtype=np.uint64)
                          for r in range(0, TK.TILE, 64)]) & np.uint64(MASK59)
    for j, tg in enumerate(targets):
        residues = [(int(out_h[0][p][tg]) + int(u[p][tg])) % primes[p] for p in range(dk)]
        got = oracle.decode(oracle.crt(residues, primes), oc.Q, 1 << 59)
        expect = (512 * (int(dot[j]) + int(local[j, 0])) - int(mask[tg])) & MASK59
        assert got == expect, j
        c0 = oracle.crt([int(out_h[0][p][tg]) for p in range(dk)], primes)
        assert sum(int(crt_h[j][i]) << (64 * i) for i in range(dk)) == c0, j

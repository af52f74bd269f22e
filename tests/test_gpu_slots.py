"""The slot-packed matvec (bfvgpu.SlotMatvec, C ABI bfvgpu_slots_*) on the GPU at the
config-2 parameters (n = 8192, 4 x 50-bit + 60-bit special prime, t = 65537) with real
keys: the decrypted, decoded result is W x mod t, and the ciphertext equals, word for
word, the oracle running the same steps (keyswitches, multi-block product, sums)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T = 65537


@pytest.fixture(scope="module")
def setup(bfv, oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    primes = oracle.coeff_modulus(8192, [50, 50, 50, 50, 60])
    hc = bfv.Context(8192, primes, 4, 1, T, device=0)
    pc = bfv.Context(8192, [T], 1, 0, 2, device=0)
    oc = oracle.Ctx(8192, primes, data_k=4, t=T)
    tc = oracle.Ctx(8192, [T], data_k=1, t=2)
    return hc, pc, oc, tc


def _decode(S, tc, coeffs):
    ev = tc.ntt_one(np.asarray(coeffs, dtype=np.uint64), 0, canonical=True)
    return ev[S.slot_positions(tc.n)]


@pytest.mark.parametrize("K,O", [(64, 128), (16, 40), (1024, 2048)])
def test_slot_matvec(bfv, oracle, setup, K, O):
    """(1024, 2048) is the benchmark's config-3 shape: W 2048 x 1024 int8, baby 32 x giant 16,
    47 keys, 31 baby-step elements in one multi-element rotation launch pair."""
    import torch
    import bfvgpu.slots as S
    hc, pc, oc, tc = setup
    n = hc.n
    lay = S.SlotLayout(n, K, O)
    baby, giant = lay.steps
    elts = S.rotation_elements(n, baby, giant)
    tb = oracle.TestBfv(oc, seed=K + O)
    keys = np.stack([tb.galois_key(e) for e in elts])
    rng = np.random.default_rng(K)
    W = rng.integers(-127, 128, size=(O, K))
    W[0, :4] = [-127, 127, 0, -1]
    x = rng.integers(0, T, size=K)
    x[:3] = [0, T - 1, 1]
    plain = lay.encode_device(torch, pc, lay.diagonals_device(torch, torch.from_numpy(W).cuda()))
    xs = lay.encode_device(torch, pc, torch.from_numpy(lay.pack_input(x)).cuda()).cpu().numpy().view(np.uint64)
    ct = tb.encrypt(xs)
    sm = bfv.SlotMatvec(hc, keys, baby, giant, plain)
    try:
        out = sm.apply(ct)
        again = sm.apply(ct)
        d_ct = torch.from_numpy(np.ascontiguousarray(ct).view(np.int64)).cuda()
        d_out = torch.empty_like(d_ct)
        sm.apply_device(d_ct, d_out)
        torch.cuda.synchronize()
        dev = d_out.cpu().numpy().view(np.uint64)
    finally:
        assert sm.close()["closed"]
    assert np.array_equal(out, again) and np.array_equal(out, dev)
    y = _decode(S, tc, tb.decrypt(out))[:O]
    want = (W.astype(object) @ x.astype(object)) % T
    assert np.array_equal(y.astype(object), want)
    # the same steps on the oracle
    pt = plain.cpu().numpy().view(np.uint64)
    R = [ct] + [oc.keyswitch(ct, keys[b - 1], elts[b - 1]) for b in range(1, baby)]
    cn = oc.matrix_open(np.stack(R), threads=8)
    parts = [oc.matrix_evaluate(cn, pt[g], threads=8) for g in range(giant)]
    acc = parts[0]
    for g in range(1, giant):
        acc = oc.add(acc, oc.keyswitch(parts[g], keys[baby - 2 + g], elts[baby - 2 + g]))
    res = oc.add(acc, oc.keyswitch(acc, keys[-1], elts[-1]))
    assert np.array_equal(out, res)

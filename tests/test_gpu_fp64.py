"""The FP64-pipe arithmetic (primes below 2^50) against the integer pipe and the oracle.

Contexts of config 1 (n = 4096, 36/36/37-bit primes) and config 2 (n = 8192, 4 x 50-bit data
primes + a 60-bit special prime) compute their batched NTTs and Galois keyswitch rotations on
the FP64 pipe by default (bfvgpu_ctx_set_fp64); a second context with it switched off runs the
integer kernels.  Both must give the same words, and the oracle's, on the same seeded inputs
(boundary residues 0, 1, q-1 included, and a ciphertext with zero c1 words for the exact
path).  Once a context has prepared keys its mode is fixed (BFVGPU_E_STATE).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG1 = dict(n=4096, bits=[36, 36, 37], dk=3, special=0, t=65537)
CFG2 = dict(n=8192, bits=[50, 50, 50, 50, 60], dk=4, special=1, t=65537)


@pytest.fixture(scope="module")
def gpu(bfv):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return bfv


def _pair(bfv, oracle, cfg):
    primes = oracle.coeff_modulus(cfg["n"], cfg["bits"])
    f = bfv.Context(cfg["n"], primes, cfg["dk"], cfg["special"], cfg["t"], device=0)
    i = bfv.Context(cfg["n"], primes, cfg["dk"], cfg["special"], cfg["t"], device=0)
    i.set_fp64(False)
    oc = oracle.Ctx(cfg["n"], primes, data_k=cfg["dk"], t=cfg["t"])
    return f, i, oc


@pytest.mark.parametrize("cfg", [CFG1, CFG2], ids=["cfg1", "cfg2"])
def test_ntt_fp64_equals_integer_and_oracle(gpu, oracle, cfg):
    import torch
    f, i, oc = _pair(gpu, oracle, cfg)
    k, n = oc.k, oc.n
    polys = 4 * k
    data = oc.uniform(91, polys, prime_count=k).reshape(polys, n)
    for r in range(polys):
        q = oc.primes[r % k]
        data[r, ::13] = 0
        data[r, 1::13] = q - 1
        data[r, 2::13] = 1
    outs = []
    for ctx in (f, i):
        d = torch.from_numpy(data.view(np.int64).copy()).cuda()
        torch.cuda.synchronize()
        ctx.ntt_device(d, polys, k, 0, False)
        torch.cuda.synchronize()
        fwd = d.cpu().numpy().view(np.uint64).copy()
        ctx.ntt_device(d, polys, k, 0, True)
        torch.cuda.synchronize()
        assert np.array_equal(d.cpu().numpy().view(np.uint64), data)
        outs.append(fwd)
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(outs[0], oc.ntt(data, prime_count=k))


def test_rotations_fp64_equals_integer_and_oracle(gpu, oracle):
    """The pipelined rotations (hoisted digits, FP64 key product, transform and special-prime
    finish for the data primes) equal the integer kernels and the oracle keyswitch."""
    import torch
    f, i, oc = _pair(gpu, oracle, CFG2)
    n, k, dk = oc.n, oc.k, oc.data_k
    count = 4
    cts = oc.uniform(93, count * 2 * dk).reshape(count, 2, dk, n)
    cts[1, 1, 2, ::5] = 0  # zero c1 words: the exact path
    cts[3, 0, :, :7] = 0
    elts = [3, pow(3, 11, 2 * n), 2 * n - 1]
    keys = np.stack([oc.uniform(95 + e, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n) for e in range(len(elts))])
    results = []
    for ctx in (f, i):
        d_cts = torch.from_numpy(cts.view(np.int64)).cuda()
        d_keys = torch.from_numpy(keys.view(np.int64)).cuda()
        hoisted = torch.empty(ctx.keyswitch_hoist_words(count), dtype=torch.int64, device="cuda")
        pw = ctx.keyswitch_prepared_words()
        prepared = torch.empty(len(elts) * pw, dtype=torch.int64, device="cuda")
        scratch = torch.empty(ctx.keyswitch_rotate_many_scratch_words(count), dtype=torch.int64, device="cuda")
        outs = [torch.full_like(d_cts, -1) for _ in elts]
        one = torch.empty_like(d_cts)
        torch.cuda.synchronize()
        ctx.keyswitch_hoist_device(d_cts, count, hoisted)
        ctx.keyswitch_prepare_device(d_keys, elts, prepared)
        ctx.keyswitch_rotate_many_device(d_cts, count, hoisted, prepared, elts, scratch, outs)
        torch.cuda.synchronize()
        assert ctx.check() == 0
        # the launch-pair form (rotate + finish kernels) agrees too
        ctx.keyswitch_rotate_device(d_cts, count, hoisted, prepared[:pw], elts[0], scratch, one)
        torch.cuda.synchronize()
        assert torch.equal(one, outs[0])
        results.append([o.cpu().numpy().view(np.uint64).copy() for o in outs])
    for e in range(len(elts)):
        assert np.array_equal(results[0][e], results[1][e]), elts[e]
    want = oc.keyswitch_many(cts, keys[1], [elts[1]], threads=8)[0]
    assert np.array_equal(results[0][1], want)


def test_fp64_mode_fixed_once_keys_are_prepared(gpu, oracle):
    import torch
    f, i, oc = _pair(gpu, oracle, CFG2)
    n, k, dk = oc.n, oc.k, oc.data_k
    keys = oc.uniform(97, dk * 2 * k, prime_count=k).reshape(1, dk, 2, k, n)
    prepared = torch.empty(f.keyswitch_prepared_words(), dtype=torch.int64, device="cuda")
    f.set_fp64(False)  # no keys yet: either mode
    f.set_fp64(True)
    f.keyswitch_prepare_device(torch.from_numpy(keys.view(np.int64)).cuda(), [3], prepared)
    torch.cuda.synchronize()
    f.set_fp64(True)  # the same mode stays allowed
    with pytest.raises(gpu.BfvGpuError) as err:
        f.set_fp64(False)
    assert err.value.code == 11 and err.value.name == "BFVGPU_E_STATE"

"""Slot packing for the slot-variant matvec (bfvgpu.slots), on the CPU: the slot positions
against the oracle's NTT mod t and Galois map (rotations and the row swap act on slots as
the layout says), and the baby-step giant-step diagonal schedule simulated on plaintext
slot vectors gives W x mod t.  The encrypted product runs in tests/test_gpu_slots.py."""
from __future__ import annotations

import numpy as np
import pytest

T = 65537


@pytest.fixture(scope="module")
def S():
    import bfvgpu.slots as S
    return S


@pytest.fixture(scope="module")
def tctx(oracle):
    """One-prime oracle context for the plaintext modulus (n = 8192)."""
    return oracle.Ctx(8192, [T], data_k=1, t=2)


def encode(S, tctx, slots):
    n = tctx.n
    poly_ntt = np.zeros(n, dtype=np.uint64)
    poly_ntt[S.slot_positions(n)] = np.asarray(slots, dtype=np.uint64) % T
    return tctx.ntt_one(poly_ntt, 0, inverse=True, canonical=True)


def decode(S, tctx, poly):
    ev = tctx.ntt_one(np.asarray(poly, dtype=np.uint64), 0, canonical=True)
    return ev[S.slot_positions(tctx.n)]


def rows_roll(v, r):
    half = v.size // 2
    return np.concatenate([np.roll(v[:half], -r), np.roll(v[half:], -r)])


def test_slot_positions_permutation(S):
    for n in (32, 4096, 8192):
        p = S.slot_positions(n)
        assert np.array_equal(np.sort(p), np.arange(n))


def test_encode_decode_round_trip_and_galois(S, tctx):
    n = tctx.n
    rng = np.random.default_rng(7)
    v = rng.integers(0, T, size=n, dtype=np.uint64)
    poly = encode(S, tctx, v)
    assert np.array_equal(decode(S, tctx, poly), v)
    for r in (1, 5, 100, n // 2 - 1):
        rot = tctx.galois(poly.reshape(1, n), pow(3, r, 2 * n), prime_count=1)[0]
        assert np.array_equal(decode(S, tctx, rot), rows_roll(v, r)), r
    sw = tctx.galois(poly.reshape(1, n), 2 * n - 1, prime_count=1)[0]
    half = n // 2
    assert np.array_equal(decode(S, tctx, sw), np.concatenate([v[half:], v[:half]]))
    # slotwise product = negacyclic product of the encoded polynomials
    w = rng.integers(0, T, size=n, dtype=np.uint64)
    prod_ntt = (tctx.ntt_one(poly, 0, canonical=True).astype(object) *
                tctx.ntt_one(encode(S, tctx, w), 0, canonical=True).astype(object)) % T
    prod = tctx.ntt_one(np.array(list(prod_ntt), dtype=np.uint64), 0, inverse=True, canonical=True)
    assert np.array_equal(decode(S, tctx, prod), (v.astype(object) * w.astype(object) % T).astype(np.uint64))


@pytest.mark.parametrize("K,O", [(64, 128), (1024, 2048), (32, 20)])
def test_bsgs_schedule_on_slots(S, K, O):
    """The evaluation order of SlotMatvec, run on plaintext slot vectors (rotations as
    row rolls): row 0 of the result is W x mod t at slots < O."""
    import torch
    n = 8192
    lay = S.SlotLayout(n, K, O)
    baby, giant = lay.steps
    assert baby * giant == K // 2
    rng = np.random.default_rng(K + O)
    W = rng.integers(-127, 128, size=(O, K))
    x = rng.integers(0, T, size=K)
    pt = lay.diagonals_device(torch, torch.from_numpy(W)).numpy().astype(object)
    xs = lay.pack_input(x).astype(object)
    rot = [rows_roll(xs, b) for b in range(baby)]
    acc = np.zeros(n, dtype=object)
    for g in range(giant):
        part = sum(pt[g, b] * rot[b] for b in range(baby)) % T
        acc = (acc + rows_roll(part, g * baby)) % T
    half = n // 2
    res = (acc + np.concatenate([acc[half:], acc[:half]])) % T
    want = (W.astype(object) @ x.astype(object)) % T
    assert np.array_equal(res[:O], want)


def test_rotation_elements(S):
    n = 8192
    el = S.rotation_elements(n, 4, 3)
    assert el == [3, 9, 27, pow(3, 4, 2 * n), pow(3, 8, 2 * n), 2 * n - 1]


def test_layout_rejects_bad_shapes(S):
    with pytest.raises(ValueError):
        S.SlotLayout(8192, 33, 64)      # odd K
    with pytest.raises(ValueError):
        S.SlotLayout(8192, 64, 8192)    # O beyond a row
    with pytest.raises(ValueError):
        S.SlotLayout(8192, 64, 64, t=65539)  # t not 1 mod 2n

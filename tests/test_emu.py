"""CPU pre-check of the CUDA kernel bodies (no GPU).

tests/emu/libemu.so compiles privacy-rag_b200/csrc/block_ops.cuh with the host compiler
and runs each thread block's work units in turn, with the constants and twiddle tables
of the product library's host-only context.  Every kernel's pass schedule, index
arithmetic, prologue and epilogue is compared bit for bit with the CPU oracle at the
sizes the kernels are instantiated for (n = 32, 64, 4096, 8192, 16384).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "emu"))
import emu_api  # noqa: E402

p = emu_api.p

SETS = {
    5: (lambda O: O.ART002_PRIMES, 6, 1 << 59),
    6: (lambda O: O.ART002_PRIMES, 6, 1 << 59),
    12: (lambda O: O.coeff_modulus(4096, [36, 36, 37]), 3, 65537),
    13: (lambda O: O.coeff_modulus(8192, [50, 50, 50, 50, 60]), 4, 65537),
    14: (lambda O: O.ART002_PRIMES, 6, 1 << 59),
}


def make(bfv, oracle, logn, fp64=True):
    """Host-only context, oracle and the kernels' constants.  fp64=False: the integer-pipe
    records (the FP64 path is taken for primes below 2^50 only when f64 is set)."""
    primes_fn, dk, t = SETS[logn]
    primes = primes_fn(oracle)
    n = 1 << logn
    hc = bfv.Context(n, primes, dk, len(primes) - dk, t, device=-1)
    hc.set_fp64(fp64)
    oc = oracle.Ctx(n, primes, data_k=dk, t=t)
    mods = np.ascontiguousarray(hc.moduli())
    fwd = np.ascontiguousarray(np.stack([hc.tables(i)[0] for i in range(hc.k)]))
    inv = np.ascontiguousarray(np.stack([hc.tables(i)[1] for i in range(hc.k)]))
    return hc, oc, mods, fwd, inv


@pytest.fixture(scope="module")
def E(emu):
    return emu_api.bind(emu)


@pytest.mark.parametrize("logn", [5, 6, 12, 13, 14])
def test_tables_match_oracle(bfv, oracle, logn):
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn)
    ofwd, oinv, oinvn = oc.tables()
    assert np.array_equal(fwd, ofwd) and np.array_equal(inv, oinv)
    assert np.array_equal(mods[:, 3:5], oinvn)
    for i, q in enumerate(oc.primes):
        r = ((1 << 128) - 1) // q
        assert int(mods[i, 0]) == q and int(mods[i, 1]) == r & ((1 << 64) - 1) and int(mods[i, 2]) == r >> 64
    for i in range(oc.data_k):
        assert int(mods[i, 8]) == oc.delta[i]


# (logn, fp64): the FP64 path applies to the 36/37-bit (n = 4096) and 50-bit (n = 8192)
# data primes; the integer path is kept covered at those degrees with fp64 off
ARITH = [(5, True), (6, True), (12, True), (12, False), (13, True), (13, False), (14, True)]


@pytest.mark.parametrize("logn,fp64", ARITH)
def test_ntt_kernel_body(bfv, oracle, E, logn, fp64):
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn, fp64)
    assert bool(int(mods[0, 10])) == (fp64 and oc.primes[0] < 2 ** 50)
    k = hc.k
    data = oc.uniform(logn, 2 * k, prime_count=k)
    n = 1 << logn
    data[0, :13] = 0
    data[1, :13] = oc.primes[1] - 1
    got = data.copy()
    assert E.emu_ntt(logn, k, p(mods), p(fwd), p(inv), p(got), data.shape[0], k, 0, 0) == 0
    assert np.array_equal(got, oc.ntt(data, prime_count=k))
    back = got.copy()
    E.emu_ntt(logn, k, p(mods), p(fwd), p(inv), p(back), data.shape[0], k, 0, 1)
    assert np.array_equal(back, data)
    # prime offset / count selection (polys on primes 1..k-1 only)
    if k > 2:
        sub = data[: k - 1].copy()
        E.emu_ntt(logn, k, p(mods), p(fwd), p(inv), p(sub), k - 1, k - 1, 1, 0)
        exp = np.stack([oc.ntt_one(data[i], 1 + i) for i in range(k - 1)])
        assert np.array_equal(sub, exp)


@pytest.mark.parametrize("logn", [6, 12, 13, 14])
def test_ntt_split_between_two_blocks(bfv, oracle, E, logn):
    """A limb split between the two blocks of a cluster (each holds half; the level whose
    pairs straddle the halves runs as a cross step through the other block's shared memory,
    the rest as a half-size schedule with the full transform's twiddles) transforms exactly
    as the one-block kernel and the oracle, forward and inverse, with boundary residues."""
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn)
    k, n = hc.k, 1 << logn
    data = oc.uniform(700 + logn, 2 * k, prime_count=k).reshape(2 * k, n)
    data[0, :3] = [0, 1, oc.primes[0] - 1]
    f = data.copy()
    E.emu_ntt_pair(logn, k, p(mods), p(fwd), p(inv), p(f), 2 * k, k, 0, 0)
    assert np.array_equal(f, oc.ntt(data, prime_count=k)), logn
    back = f.copy()
    E.emu_ntt_pair(logn, k, p(mods), p(fwd), p(inv), p(back), 2 * k, k, 0, 1)
    assert np.array_equal(back, data), logn


@pytest.mark.parametrize("logn,elts,fp64", [(5, [1, 3, 63], True), (6, [5, 127, 9], True),
                                            (13, [3, 2 ** 13 + 1, 16383], True), (13, [3, 16383], False),
                                            (14, [1, 3, 1025], True)])
def test_keyswitch_kernel_body(bfv, oracle, E, logn, elts, fp64):
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn, fp64)
    k, dk, n = hc.k, hc.dk, 1 << logn
    count = 2
    cts = oc.uniform(100 + logn, count * 2 * dk, prime_count=dk).reshape(count, 2, dk, n)
    cts[0, 1, :, ::5] = 0  # zero digits: the automorphism must keep them zero
    key = oc.uniform(200 + logn, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n)
    for elt in elts:
        out = np.zeros_like(cts)
        E.emu_keyswitch(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), count, p(key), elt, p(out))
        for c in range(count):
            assert np.array_equal(out[c], oc.keyswitch(cts[c], key, elt)), (logn, elt, c)


@pytest.mark.parametrize("logn,elts,fp64", [(5, [1, 3, 63], True), (6, [5, 127, 9], True),
                                            (13, [3, 2 ** 13 + 1, 16383], True), (13, [2 ** 13 + 1], False),
                                            (14, [3, 1025], True)])
def test_hoisted_keyswitch_kernel_bodies(bfv, oracle, E, logn, elts, fp64):
    """Hoist + key preparation + rotate + finish equals the reference keyswitch; the
    ciphertext with zero c1 words is flagged and takes the exact path."""
    import ctypes
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn, fp64)
    k, dk, n = hc.k, hc.dk, 1 << logn
    count = 3
    cts = oc.uniform(300 + logn, count * 2 * dk, prime_count=dk).reshape(count, 2, dk, n)
    cts[1, 1, 2, ::3] = 0
    key = oc.uniform(400 + logn, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n)
    for elt in elts:
        out = np.zeros_like(cts)
        flags = (ctypes.c_uint32 * count)()
        E.emu_keyswitch_hoisted(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), count, p(key), elt, p(out), flags)
        assert list(flags) == [0, 1, 0]
        for c in range(count):
            assert np.array_equal(out[c], oc.keyswitch(cts[c], key, elt)), (logn, elt, c)


@pytest.mark.parametrize("logn,elts,fp64", [(5, [3, 63, 1, 9], True), (6, [5, 127, 9], True),
                                            (13, [3, 2 ** 13 + 1, 16383], True), (13, [3, 16383], False)])
def test_pipelined_rotation_kernel_bodies(bfv, oracle, E, logn, elts, fp64):
    """The software-pipelined rotations (launch r: special-prime blocks of element r beside
    the data-prime blocks of element r - 1, which finish the keyswitch in shared memory) run
    on the host with the device's buffers and indexing, against the reference keyswitch for
    every element, including a ciphertext whose c1 holds zero words (the exact path)."""
    import ctypes
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn, fp64)
    k, dk, n = hc.k, hc.dk, 1 << logn
    count = 3
    cts = oc.uniform(500 + logn, count * 2 * dk, prime_count=dk).reshape(count, 2, dk, n)
    cts[2, 1, 1, ::4] = 0
    keys = np.stack([oc.uniform(600 + logn + e, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n)
                     for e in range(len(elts))])
    outs = np.zeros((len(elts), count, 2, dk, n), dtype=np.uint64)
    el = (ctypes.c_uint32 * len(elts))(*elts)
    E.emu_keyswitch_pipe(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), count, p(keys), el, len(elts), p(outs))
    for e, elt in enumerate(elts):
        for c in range(count):
            assert np.array_equal(outs[e, c], oc.keyswitch(cts[c], keys[e], elt)), (logn, elt, c)


@pytest.mark.parametrize("logn", [6, 14])
def test_matrix_mask_enc0_kernel_bodies(bfv, oracle, E, logn):
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn)
    k, dk, n = hc.k, hc.dk, 1 << logn
    tb = oracle.TestBfv(oc, seed=logn)
    rng = np.random.default_rng(logn)
    I, G = 3, 2
    cts = np.stack([tb.encrypt(rng.integers(0, 1 << 59, size=n, dtype=np.uint64)) for _ in range(I)])
    ring = rng.integers(0, 1 << 59, size=(G, I, n), dtype=np.uint64)
    ring[0, 0, :4] = [(1 << 59) - 1, 1 << 58, (1 << 58) - 1, 0]
    mask = rng.integers(0, 1 << 59, size=(G, n), dtype=np.uint64)
    samples = np.stack([tb.samples() for _ in range(G)])
    out = np.zeros((G, 2, dk, n), dtype=np.uint64)
    E.emu_matrix(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), I, p(ring), G, p(mask), p(samples), p(tb.pk),
                 oc.q_mod_t, oc.upper_half, 1 << 59, 59, p(out))
    cn = oc.matrix_open(cts)
    for g in range(G):
        e = oc.matrix_evaluate(cn, ring[g])
        e[0] = oc.sub_plain(e[0], mask[g])
        e = oc.add(e, oc.enc0(samples[g], tb.pk))
        assert np.array_equal(out[g], e), g
    # unprotected product
    out2 = np.zeros((1, 2, dk, n), dtype=np.uint64)
    E.emu_matrix(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), I, p(ring[0]), 1, None, None, None,
                 oc.q_mod_t, oc.upper_half, 1 << 59, 59, p(out2))
    assert np.array_equal(out2[0], oc.matrix_evaluate(cn, ring[0]))


@pytest.mark.parametrize("tiles,I,G,path", [(1, 3, 2, 0), (3, 3, 2, 0), (8, 3, 2, 1), (2, 20, 19, 0),
                                             (1, 264, 3, 0), (8, 3, 2, 0), (9, 40, 33, 0), (8, 64, 3, 0)])
def test_matrix_tiles_kernel_bodies(bfv, oracle, E, tiles, I, G, path):
    """Layer pipeline (split-operand NTT, multi-tile product over 30-bit halves with its
    shared-memory staging, Enc(0) prep, INTT with folded Enc(0) and mask) against the
    oracle's per-tile matrix evaluation + sub_plain + Enc(0) add.  Cases cover partial and
    several input chunks, more groups than one block holds, and more than 256 inputs (the
    periodic reduction of the 128-bit sums); with path 0, launches of 8 tiles take the
    tcgen05 product (K padded to 32 and 64, a partial group chunk), emulated from its
    shared-memory operand layouts, TMEM drain and shuffle recombination."""
    logn = 5
    hc, oc, mods, fwd, inv = make(bfv, oracle, logn)
    k, dk, n = hc.k, hc.dk, 1 << logn
    tb = oracle.TestBfv(oc, seed=40 + tiles)
    rng = np.random.default_rng(tiles + I)
    cts = np.stack([np.stack([tb.encrypt(rng.integers(0, 1 << 59, size=n, dtype=np.uint64)) for _ in range(I)])
                    for _ in range(tiles)])
    ring = rng.integers(0, 1 << 59, size=(G, I, n), dtype=np.uint64)
    ring[0, 0, :4] = [(1 << 59) - 1, 1 << 58, (1 << 58) - 1, 0]
    masks = rng.integers(0, 1 << 59, size=(tiles, G, n), dtype=np.uint64)
    samples = np.stack([np.stack([tb.samples() for _ in range(G)]) for _ in range(tiles)])
    out = np.zeros((tiles, G, 2, dk, n), dtype=np.uint64)
    E.emu_matrix_tiles(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), tiles, I, p(ring), G, p(masks), p(samples),
                       p(tb.pk), oc.q_mod_t, oc.upper_half, 1 << 59, 59, p(out), path)
    plain = np.zeros_like(out)
    E.emu_matrix_tiles(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), tiles, I, p(ring), G, None, None, None,
                       oc.q_mod_t, oc.upper_half, 1 << 59, 59, p(plain), path)
    masked = np.zeros_like(out)  # masks without Enc(0): the additive term is -Delta mask alone
    E.emu_matrix_tiles(logn, k, dk, p(mods), p(fwd), p(inv), p(cts), tiles, I, p(ring), G, p(masks), None, None,
                       oc.q_mod_t, oc.upper_half, 1 << 59, 59, p(masked), path)
    for t in range(tiles):
        cn = oc.matrix_open(cts[t])
        for g in range(G):
            e = oc.matrix_evaluate(cn, ring[g])
            assert np.array_equal(plain[t, g], e), (t, g)
            e[0] = oc.sub_plain(e[0], masks[t, g])
            assert np.array_equal(masked[t, g], e), (t, g)
            e = oc.add(e, oc.enc0(samples[t, g], tb.pk))
            assert np.array_equal(out[t, g], e), (t, g)


def test_client_phase_kernel_body(bfv, oracle, E):
    hc, oc, mods, fwd, inv = make(bfv, oracle, 14)
    tb = oracle.TestBfv(oc, seed=2)
    c1 = oc.uniform(5, 2 * 6).reshape(2, 6, oc.n)
    got = c1.copy()
    E.emu_client_phase(14, 7, 6, p(mods), p(fwd), p(inv), p(got), p(tb.sk_data_ntt()), 2)
    for b in range(2):
        assert np.array_equal(got[b], oc.client_phase(c1[b], tb.sk_data_ntt()))


def test_crt_body(bfv, oracle, E):
    primes = oracle.ART002_PRIMES[:6]
    Q = 1
    for q in primes:
        Q *= q
    vals = [0, 1, Q - 1, Q // 2, 2 ** 359, 12345678901234567890123456789 ** 3 % Q]
    res = np.array([[v % q for q in primes] for v in vals], dtype=np.uint64)
    hc = bfv.Context(64, oracle.ART002_PRIMES, 6, 1, 1 << 59, device=-1)
    mods = np.ascontiguousarray(hc.moduli())
    part = np.array([[((Q // q) >> (64 * l)) & ((1 << 64) - 1) for l in range(6)] for q in primes], dtype=np.uint64)
    cinv = np.array([[pow(Q // q % q, -1, q), (pow(Q // q % q, -1, q) << 64) // q] for q in primes], dtype=np.uint64)
    ql = np.array([(Q >> (64 * l)) & ((1 << 64) - 1) for l in range(6)], dtype=np.uint64)
    limbs = np.zeros_like(res)
    E.emu_crt(7, 6, p(mods), p(res), len(vals), p(part), p(cinv), p(ql), p(limbs))
    for i, v in enumerate(vals):
        assert sum(int(limbs[i, l]) << (64 * l) for l in range(6)) == v


def test_token_kernel_bodies(bfv, oracle, E):
    hc, oc, mods, fwd, inv = make(bfv, oracle, 14)
    rng = np.random.default_rng(8)
    slots = 1
    cts = oc.uniform(77, 19 * slots * 2 * 6).reshape(19, slots, 2, 6, oc.n)
    cts_ntt = oc.ntt(cts.reshape(-1, oc.n), prime_count=6).reshape(cts.shape)
    bound = 1 << 20
    ring = (rng.integers(-bound, bound + 1, size=19 * 8192) & ((1 << 59) - 1)).astype(np.uint64)
    scaled = np.array([oc.scale_plain(int(rng.integers(0, 1 << 59)))], dtype=np.uint64)
    out = np.zeros((slots, 2, 6, oc.n), dtype=np.uint64)
    E.emu_token(7, 6, p(mods), p(fwd), p(inv), p(cts_ntt), slots, p(ring), p(scaled), p(out))
    assert np.array_equal(out, oc.token_evaluate(cts_ntt, slots, ring, scaled))

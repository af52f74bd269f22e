"""CPU oracle pinned against the reference's known answers (no GPU).

* parameter KAT: IV1/artifacts/bfv_context.json (primes, Q and bit sizes of all levels)
* prime search reproduces the locked ART-002 chain (bfv.cpp:91-105)
* NTT = its evaluation definition; lazy (SEAL-style) = canonical (reference GPU stage form)
* Barrett limb sequence (matrix.cu:37-43) = exact 128-bit reduction
* packing decisions (bfv_layout.hpp:14-27) = the per-shape values the survey derives
* decode/CRT = the locked decode arithmetic (bfv.cpp:138-147, :328-356)
* end-to-end plaintext KATs of the reference probes through oracle encryption, the
  oracle ct-pt product, masking and Enc(0), then decryption
"""
from __future__ import annotations

import json
import os
import random

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_art002_context_kat(oracle):
    with open(os.path.join(GOLD, "art002_context.json")) as f:
        ctx = json.load(f)
    assert ctx["polynomial_degree"] == 16384 and int(ctx["plaintext_modulus"]) == 1 << 59
    key = [lv for lv in ctx["levels"] if lv["key_level"]][0]
    assert [int(p) for p in key["primes"]] == oracle.ART002_PRIMES
    for lv in ctx["levels"]:
        q = 1
        for p in lv["primes"]:
            q *= int(p)
        assert q == int(lv["Q"]) and q.bit_length() == lv["Q_bits"]
    assert oracle.coeff_modulus(16384, [60] * 7) == oracle.ART002_PRIMES
    oc = oracle.art002()
    data_q = [lv for lv in ctx["levels"] if lv["chain_index"] == 5][0]
    assert oc.Q == int(data_q["Q"])


def test_baseline_prime_chains(oracle):
    c1 = oracle.coeff_modulus(4096, [36, 36, 37])
    c2 = oracle.coeff_modulus(8192, [50, 50, 50, 50, 60])
    assert [p.bit_length() for p in c1] == [36, 36, 37]
    assert [p.bit_length() for p in c2] == [50, 50, 50, 50, 60]
    for p in c1:
        assert oracle.is_prime(p) and (p - 1) % 8192 == 0
    for p in c2:
        assert oracle.is_prime(p) and (p - 1) % 16384 == 0


@pytest.mark.parametrize("n", [16, 64, 256])
def test_ntt_definition_and_round_trip(oracle, n):
    oc = oracle.Ctx(n, oracle.ART002_PRIMES, data_k=6)
    rng = np.random.default_rng(n)
    for p in range(7):
        a = (rng.integers(0, 1 << 62, size=n, dtype=np.uint64) % np.uint64(oc.primes[p])).astype(np.uint64)
        f = oc.ntt_one(a, p)
        assert np.array_equal(f, oc.ntt_naive(a, p))
        assert np.array_equal(f, oc.ntt_one(a, p, canonical=True))
        assert np.array_equal(oc.ntt_one(f, p, inverse=True), a)
        assert np.array_equal(oc.ntt_one(f, p, inverse=True, canonical=True), a)


def test_minimal_root(oracle):
    for q in oracle.ART002_PRIMES[:2]:
        psi = oracle.minimal_root(q, 64)
        assert pow(psi, 32, q) == q - 1
        # no smaller element is a primitive 64th root
        assert all(pow(x, 32, q) != q - 1 for x in range(2, min(psi, 20000)))


def test_barrett_matches_exact(oracle):
    L = oracle.lib()
    rnd = random.Random(5)
    for q in oracle.ART002_PRIMES + oracle.coeff_modulus(8192, [50, 50, 50, 50, 60]):
        r = ((1 << 128) - 1) // q
        for a, b in [(0, 0), (q - 1, q - 1), (1, q - 1)] + [(rnd.randrange(q), rnd.randrange(q)) for _ in range(300)]:
            assert L.or_mul_barrett(a, b, q, r & ((1 << 64) - 1), r >> 64) == a * b % q


SHAPE_PACKING = {
    # (B, K, O): (d, cap, returns, inputs) -- the per-shape decisions quoted for the
    # reference rule (q_proj at B=1; the four 16-token tile calls; the decode calls)
    (1, 1024, 2048): (64, 128, 16, 16),
    (16, 1024, 4096): (16, 32, 128, 64),
    (16, 2048, 1024): (32, 16, 64, 64),
    (16, 1024, 6144): (16, 32, 192, 64),
    (16, 3072, 1024): (64, 8, 128, 48),
    (1, 1024, 4096): (64, 128, 32, 16),
    (1, 2048, 1024): (128, 64, 16, 16),
    (1, 1024, 6144): (64, 128, 48, 16),
    (1, 3072, 1024): (256, 32, 32, 12),
}


def test_packing_decisions(oracle, bfv):
    for (b, k, o), want in SHAPE_PACKING.items():
        p = oracle.matrix_packing(b, k, o)
        assert (p.reduction, p.columns, p.returns, p.inputs) == want, (b, k, o)
        q = bfv.matrix_packing(b, k, o)
        assert (q.reduction, q.columns, q.returns, q.inputs) == want, (b, k, o)
    with open(os.path.join(GOLD, "packing_kats.json")) as f:
        for c in json.load(f)["cases"]:
            q = bfv.matrix_packing(c["b"], c["k"], c["o"])
            assert (q.reduction, q.columns, q.returns, q.inputs) == (c["reduction"], c["columns"], c["returns"],
                                                                       c["inputs"])
    for bad in ((0, 1, 1), (17, 1, 1), (1, 0, 1), (1, 8193, 1), (1, 1, 0), (1, 1, 155649)):
        with pytest.raises(ValueError):
            bfv.matrix_packing(*bad)
    assert bfv.packed_bfv_rows_per_ciphertext(4096) == 2
    assert bfv.packed_bfv_rows_per_ciphertext(2730) == 3
    assert bfv.packed_bfv_rows_per_ciphertext(3) == 2730


def test_crt_and_decode(oracle):
    primes = oracle.ART002_PRIMES[:6]
    Q = 1
    for p in primes:
        Q *= p
    for v in (0, 1, Q - 1, Q // 2, Q // 2 + 1, 123456789 ** 5):
        assert oracle.crt([v % p for p in primes], primes) == v
    t = 1 << 59
    for m in (0, 1, t - 1, 12345):
        delta_m = (Q * m + (t + 1) // 2) // t  # what the scaled plaintext encodes
        assert oracle.decode(delta_m % Q, Q, t) == m


def test_scale_plain_matches_definition(oracle):
    oc = oracle.art002()
    Q, t = oc.Q, oc.t
    for m in (0, 1, t - 1, 987654321987):
        want = ((Q // t) * m + ((Q % t) * m + (t + 1) // 2) // t)
        assert oc.scale_plain(m) == [want % p for p in oc.primes[:6]]


def test_small_bfv_keyswitch_decrypts(oracle):
    oc = oracle.Ctx(64, oracle.ART002_PRIMES, data_k=6)
    tb = oracle.TestBfv(oc, seed=3)
    m = np.array([random.Random(1).randrange(1 << 59) for _ in range(64)], dtype=np.uint64)
    ct = tb.encrypt(m)
    assert tb.decrypt(ct) == [int(v) for v in m]
    for elt in (3, 5, 127):
        out = oc.keyswitch(ct, tb.galois_key(elt), elt)
        exp = [0] * 64
        for j in range(64):
            d = (j * elt) % 128
            if d >= 64:
                exp[d - 64] = (-int(m[j])) % (1 << 59)
            else:
                exp[d] = int(m[j])
        assert tb.decrypt(out) == exp


def _kat_operands(case):
    mask = (1 << 59) - 1
    cols, rows = case["columns"], case["rows"]
    j = np.arange(cols, dtype=np.int64)
    if case["generator"] == "packed":
        whole = (((j * 13 + 7) % 101) - 50)
        w = np.stack([np.zeros(cols, dtype=np.int64) if r in (1, rows - 1) else (((j * (r + 3) + 5) % 17) - 8)
                      for r in range(rows)])
    else:
        cid = case["case_id"]
        if cid == 1:
            whole = np.where((j == 0) | (j == 8192), 7, 0)
            w = np.zeros((rows, cols), dtype=np.int64)
            w[0, 0], w[0, 8192] = 11, -11  # row 0 cancels across ciphertexts
            w[2:, 0], w[2:, 8192] = 3, -5   # row 1 zero, rows >= 2 negative
        else:
            whole = (((j * 13 + 7) % 101) - 50)
            w = np.stack([np.zeros(cols, dtype=np.int64) if (cid < 2 and r == 1) else (((j * (r + 3) + 5) % 17) - 8)
                          for r in range(rows)])
    client = (0x1928abcdef + j.astype(object) * 125939) % (1 << 59)
    whole_u = (whole.astype(object)) % (1 << 59)
    server = (whole_u - client) % (1 << 59)
    return ([int(v) for v in client], [int(v) for v in server], (w.astype(object) % (1 << 59)).tolist(), mask)


def test_linear_kat_expected_values(oracle):
    """The committed expected values equal the plaintext dot product of the restated
    operands (independent numpy computation)."""
    with open(os.path.join(GOLD, "kat_linear.json")) as f:
        cases = json.load(f)["cases"]
    for case in cases:
        client, server, w, mask = _kat_operands(case)
        whole = [(c + s) & mask for c, s in zip(client, server)]
        exp = [sum(int(a) * int(b) for a, b in zip(whole, row)) & mask for row in w]
        assert exp == case["expected"], case["probe"]


def test_linear_kat_through_oracle_bfv(oracle):
    """dev_bfv_packed_probe case d=2730, rows=4 end to end at ART-002 through the oracle:
    pack (B=1), encrypt, product, mask, Enc(0), client phase, CRT, decode, add shares."""
    with open(os.path.join(GOLD, "kat_linear.json")) as f:
        case = [c for c in json.load(f)["cases"] if c["probe"] == "dev_bfv_packed_probe" and c["columns"] == 2730][0]
    client, server, w, mask = _kat_operands(case)
    oc = oracle.art002()
    tb = oracle.TestBfv(oc, seed=9)
    K, O = case["columns"], case["rows"]
    pk = oracle.matrix_packing(1, K, O)
    d, cap = pk.reduction, pk.columns
    x_poly = oracle.pack_inputs([client], d, pk.inputs, oc.n)
    cts = np.stack([tb.encrypt(x_poly[b]) for b in range(pk.inputs)])
    cn = oc.matrix_open(cts, threads=8)
    result = [0] * O
    rng = np.random.default_rng(4)
    for first in range(0, O, cap):
        count = min(cap, O - first)
        blocks = []
        for blk in range(pk.inputs):
            begin, actual = blk * d, min(d, K - blk * d)
            rows = [[w[first + o][begin + j] for j in range(actual)] for o in range(count)]
            blocks.append(rows)
            for o in range(count):
                result[first + o] = (result[first + o] + sum(server[begin + j] * rows[o][j] for j in range(actual))) & mask
        ring = oracle.pack_weights(blocks, d, 1, oc.n)
        tg = oracle.targets(count, 1, d)
        out = oc.matrix_evaluate(cn, ring, threads=8)
        m = rng.integers(0, 1 << 59, size=oc.n, dtype=np.uint64)
        out[0] = oc.sub_plain(out[0], m)
        out = oc.add(out, oc.enc0(tb.samples(), tb.pk))
        for o, t in enumerate(tg):
            result[first + o] = (result[first + o] + int(m[t])) & mask
            phase = tb.phase_at(out, t)
            result[first + o] = (result[first + o] + oracle.decode(phase, oc.Q)) & mask
    assert result == case["expected"]

"""Exactness of the FP64-pipe modular arithmetic (privacy-rag_b200/csrc/f64mod.cuh), run on
the host build of the same header (IEEE double operations with std::fma, no contraction).

mulmod_f64(y, w) must return a representative of y*w mod q with |r| <= 0.75 q for every
|y| < 2^52 and centred |w| <= q/2, q < 2^50; reduce_f64(v) one with |r| <= (q + 1)/2;
canon_f64 the canonical residue; mulmod_f64_barrett(y, w) (quotient from fl(1/q), for key
words that carry no quotient) a representative with |r| <= 0.75 q for |y| <= (q + 1)/2 and
0 <= w < q.  (The NTT passes rely on the (q + 1)/2 bound: eight
reduced values summed stay below 4q + 4 < 2^52.)  The cases include the range limits
(|y| = 2^52 - 1, |w| = floor(q/2), q just below 2^50) and random values for several moduli.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "emu"))
import emu_api  # noqa: E402

p = emu_api.p


@pytest.fixture(scope="module")
def E(emu):
    return emu_api.bind(emu)


def _cases(q: int, rng: np.random.Generator, count: int):
    lim = (1 << 52) - 1
    half = q // 2
    edge_y = [0, 1, -1, lim, -lim, q, -q, 4 * q - 1, -(4 * q - 1), lim - 1, 3 * q + half]
    edge_w = [v for v in (0, 1, -1, half, -half, half - 1, -(half - 1), 2, 12345) if abs(v) <= half]
    ys = [y for y in edge_y for _ in edge_w]
    ws = [w for _ in edge_y for w in edge_w]
    ys += [int(v) for v in rng.integers(-lim, lim, size=count, dtype=np.int64)]
    ws += [int(v) for v in rng.integers(-half, half + 1, size=count, dtype=np.int64)]
    return ys, ws


@pytest.mark.parametrize("q", [(1 << 50) - 27, (1 << 50) - 1, 1125899906826241, (1 << 49) + 1, 68719403009, 97])
def test_mulmod_reduce_exact(E, q):
    rng = np.random.default_rng(q & 0xFFFF)
    ys, ws = _cases(q, rng, 20000)
    y = np.array(ys, dtype=np.int64)
    w = np.array(ws, dtype=np.int64)
    n = len(ys)
    r = np.zeros(n, dtype=np.int64)
    c = np.zeros(n, dtype=np.uint64)
    red = np.zeros(n, dtype=np.int64)
    assert E.emu_f64_mulmod(p(y.view(np.uint64)), p(w.view(np.uint64)), n, q, p(r.view(np.uint64)), p(c),
                            p(red.view(np.uint64))) == 0
    for i in range(n):
        want = ys[i] * ws[i] % q
        ri = int(r[i])
        assert ri % q == want, (ys[i], ws[i])
        assert 4 * abs(ri) <= 3 * q
        assert int(c[i]) == want
        rd = int(red[i])
        assert rd % q == ys[i] % q
        assert 2 * abs(rd) <= q + 1


@pytest.mark.parametrize("q", [(1 << 50) - 27, 1125899906826241, (1 << 49) + 1, 68719403009, 97])
def test_mulmod_barrett_exact(E, q):
    rng = np.random.default_rng((q & 0xFFFF) + 1)
    hy = (q + 1) // 2
    ys = [0, 1, -1, hy, -hy, hy - 1, -(hy - 1)] * 4
    ws = [0] * 7 + [1] * 7 + [q - 1] * 7 + [q // 2] * 7
    ys += [int(v) for v in rng.integers(-hy, hy + 1, size=20000, dtype=np.int64)]
    ws += [int(v) for v in rng.integers(0, q, size=20000, dtype=np.uint64)]
    y = np.array(ys, dtype=np.int64)
    w = np.array(ws, dtype=np.uint64)
    r = np.zeros(len(ys), dtype=np.int64)
    assert E.emu_f64_mulmod_barrett(p(y.view(np.uint64)), p(w), len(ys), q, p(r.view(np.uint64))) == 0
    for yi, wi, ri in zip(ys, ws, r.tolist()):
        assert ri % q == yi * wi % q, (yi, wi)
        assert 4 * abs(ri) <= 3 * q


def test_convert_round_trip(E):
    rng = np.random.default_rng(7)
    x = np.concatenate([np.array([0, 1, (1 << 52) - 1, (1 << 50) - 1, 1 << 51], dtype=np.uint64),
                        rng.integers(0, 1 << 52, size=5000, dtype=np.uint64)])
    out = np.zeros_like(x)
    assert E.emu_f64_convert(p(x), len(x), p(out)) == 0
    assert np.array_equal(out, x)

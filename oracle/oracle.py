"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker or the timed CPU baseline.  The product
path (``privacy-rag_b200``) never imports it.

It wraps ``liboracle.so`` (``bfv_oracle.c``) and adds the multi-precision pieces
that the reference does with GMP, written with Python integers:

* ``crt`` -- ``rns_coefficient`` (IV1/native/src/bfv.cpp:138-147): CRT of one
  coefficient's residues to an integer in [0, Q).
* ``decode`` -- the locked BFV decode the garbled circuit evaluates
  (IV1/native/src/bfv.cpp:308-357): round(t * phase / Q) mod t.
* a test-only BFV key generation / encryption / decryption over the oracle's
  arithmetic, used to turn the reference's plaintext known answers
  (dev_bfv_packed_probe.cpp:35-80, dev_bfv_merged_probe.cpp, dev_tile_long_probe.cpp)
  into end-to-end checks.  The production samplers (Blake2xb, CBD) are SEAL's and
  are not restated; the key material here is seeded and only self-consistent.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

U64 = ctypes.c_uint64
U64P = ctypes.POINTER(ctypes.c_uint64)
MAX_PRIMES = 16

# ART-002 (IV1/native/src/bfv.cpp:97-100; IV1/artifacts/bfv_context.json)
ART002_PRIMES = [
    1152921504599080961, 1152921504600260609, 1152921504604979201,
    1152921504605962241, 1152921504606584833, 1152921504606683137,
    1152921504606748673,
]
ART002_N = 16384
ART002_T = 1 << 59
MASK59 = (1 << 59) - 1


class _OrCtx(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_size_t), ("logn", ctypes.c_size_t), ("k", ctypes.c_size_t),
        ("data_k", ctypes.c_size_t), ("t", U64),
        ("q", U64 * MAX_PRIMES), ("r0", U64 * MAX_PRIMES), ("r1", U64 * MAX_PRIMES),
        ("fwd", U64P), ("inv", U64P), ("invn", (U64 * 2) * MAX_PRIMES),
        ("psi", U64 * MAX_PRIMES), ("inv_special", (U64 * 2) * MAX_PRIMES),
        ("delta", U64 * MAX_PRIMES), ("q_mod_t", U64), ("upper_half", U64),
    ]


class _OrPacking(ctypes.Structure):
    _fields_ = [("reduction", U64), ("columns", U64), ("returns", U64), ("inputs", U64)]


def build() -> str:
    """Compile liboracle.so with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "bfv_oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER(_OrCtx)
        sz = ctypes.c_size_t
        sig = {
            "or_is_prime": (ctypes.c_int, [U64]),
            "or_get_primes": (sz, [U64, ctypes.c_int, sz, U64P]),
            "or_coeff_modulus": (ctypes.c_int, [sz, ctypes.POINTER(ctypes.c_int), sz, U64P]),
            "or_minimal_root": (U64, [U64, U64]),
            "or_shoup_quotient": (U64, [U64, U64]),
            "or_ctx_new": (P, [sz, sz, U64P, sz, U64]),
            "or_ctx_free": (None, [P]),
            "or_mul_barrett": (U64, [U64, U64, U64, U64, U64]),
            "or_mul_shoup": (U64, [U64, U64, U64, U64]),
            "or_mulmod": (U64, [U64, U64, U64]),
            "or_ntt_forward": (None, [P, sz, U64P]),
            "or_ntt_inverse": (None, [P, sz, U64P]),
            "or_ntt_forward_canonical": (None, [P, sz, U64P]),
            "or_ntt_inverse_canonical": (None, [P, sz, U64P]),
            "or_ntt_batch": (None, [P, U64P, sz, sz, sz, ctypes.c_int, ctypes.c_int]),
            "or_ntt_naive": (None, [P, sz, U64P, U64P]),
            "or_matrix_packing": (ctypes.c_int, [sz, sz, sz, ctypes.POINTER(_OrPacking)]),
            "or_matrix_packing_qk_reverse64": (ctypes.c_int, [sz, ctypes.POINTER(_OrPacking)]),
            "or_packed_rows_per_ciphertext": (sz, [sz]),
            "or_lift": (None, [P, U64P, sz, U64P]),
            "or_matrix_open": (None, [P, U64P, sz, ctypes.c_int]),
            "or_matrix_evaluate": (None, [P, U64P, sz, U64P, U64P, sz, U64P, ctypes.c_int]),
            "or_scale_plain": (None, [P, U64, U64P]),
            "or_sub_plain": (None, [P, U64P, U64P]),
            "or_add_plain": (None, [P, U64P, U64P, sz]),
            "or_enc0": (None, [P, U64P, U64P, U64P]),
            "or_moddown": (None, [P, U64P, U64P]),
            "or_add_inplace": (None, [P, U64P, U64P, sz]),
            "or_galois": (None, [P, U64P, U64P, sz, sz, ctypes.c_uint32]),
            "or_keyswitch_galois": (None, [P, U64P, U64P, ctypes.c_uint32, U64P]),
            "or_keyswitch_many": (None, [P, U64P, sz, U64P, ctypes.POINTER(ctypes.c_uint32), sz,
                                         U64P, ctypes.c_int]),
            "or_monomial_shift": (None, [P, U64P, sz]),
            "or_packing_pair": (None, [P, U64P, U64P, U64P, U64P, ctypes.c_uint, U64P]),
            "or_client_phase": (None, [P, U64P, U64P, U64P]),
            "or_token_evaluate": (None, [P, U64P, sz, U64P, U64P, U64P]),
            "or_token_local_scaled": (None, [P, U64P, sz, U64P, U64P]),
            "or_fill_uniform": (None, [U64, U64P, sz, sz, sz, U64P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(U64P)


def u64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint64))


# --------------------------------------------------------------------------------
# primes
# --------------------------------------------------------------------------------
def is_prime(n: int) -> bool:
    return bool(lib().or_is_prime(n))


def coeff_modulus(n: int, bits: list[int]) -> list[int]:
    out = (U64 * len(bits))()
    arr = (ctypes.c_int * len(bits))(*bits)
    rc = lib().or_coeff_modulus(n, arr, len(bits), out)
    if rc != 0:
        raise ValueError(f"or_coeff_modulus failed: {rc}")
    return [int(v) for v in out]


def minimal_root(q: int, order: int) -> int:
    return int(lib().or_minimal_root(q, order))


# --------------------------------------------------------------------------------
# context
# --------------------------------------------------------------------------------
class Ctx:
    """Oracle parameter context: n, primes (data primes then an optional special
    prime), plaintext modulus t."""

    def __init__(self, n: int, primes: list[int], data_k: int | None = None, t: int = ART002_T):
        self.n = n
        self.primes = [int(p) for p in primes]
        self.k = len(primes)
        self.data_k = self.k if data_k is None else data_k
        self.t = t
        arr = (U64 * self.k)(*self.primes)
        self._c = lib().or_ctx_new(n, self.k, arr, self.data_k, t)
        if not self._c:
            raise ValueError("or_ctx_new rejected the parameters")
        c = self._c.contents
        self.psi = [int(c.psi[i]) for i in range(self.k)]
        self.delta = [int(c.delta[i]) for i in range(self.data_k)]
        self.q_mod_t = int(c.q_mod_t)
        self.upper_half = int(c.upper_half)

    def __del__(self):
        if getattr(self, "_c", None) and _lib is not None:
            _lib.or_ctx_free(self._c)
            self._c = None

    @property
    def Q(self) -> int:
        q = 1
        for p in self.primes[: self.data_k]:
            q *= p
        return q

    @property
    def q_arr(self) -> np.ndarray:
        return u64(self.primes)

    def tables(self):
        """(fwd [k][n][2], inv [k][n][2], invn [k][2]) in the reference table layout."""
        c = self._c.contents
        size = self.k * self.n * 2
        fwd = np.ctypeslib.as_array(c.fwd, shape=(size,)).copy().reshape(self.k, self.n, 2)
        inv = np.ctypeslib.as_array(c.inv, shape=(size,)).copy().reshape(self.k, self.n, 2)
        invn = np.array([[c.invn[i][0], c.invn[i][1]] for i in range(self.k)], dtype=np.uint64)
        return fwd, inv, invn

    # ---- NTT --------------------------------------------------------------------
    def ntt(self, data: np.ndarray, prime_count: int | None = None, prime_offset: int = 0,
            inverse: bool = False, threads: int = 1) -> np.ndarray:
        """Batched transform of [..][n] with prime = offset + poly % prime_count."""
        a = u64(data).copy()
        polys = a.size // self.n
        pc = self.k if prime_count is None else prime_count
        lib().or_ntt_batch(self._c, _p(a), polys, pc, prime_offset, int(inverse), threads)
        return a

    def ntt_one(self, a, prime: int, inverse=False, canonical=False) -> np.ndarray:
        a = u64(a).copy()
        L = lib()
        if canonical:
            f = L.or_ntt_inverse_canonical if inverse else L.or_ntt_forward_canonical
        else:
            f = L.or_ntt_inverse if inverse else L.or_ntt_forward
        f(self._c, prime, _p(a))
        return a

    def ntt_naive(self, a, prime: int) -> np.ndarray:
        a = u64(a)
        out = np.zeros(self.n, dtype=np.uint64)
        lib().or_ntt_naive(self._c, prime, _p(a), _p(out))
        return out

    # ---- matrix -------------------------------------------------------------------
    def lift(self, ring: np.ndarray) -> np.ndarray:
        ring = u64(ring)
        blocks = ring.size // self.n
        out = np.zeros((blocks, self.data_k, self.n), dtype=np.uint64)
        lib().or_lift(self._c, _p(ring), blocks, _p(out))
        return out

    def matrix_open(self, cts: np.ndarray, threads: int = 1) -> np.ndarray:
        a = u64(cts).copy()
        inputs = a.size // (2 * self.data_k * self.n)
        lib().or_matrix_open(self._c, _p(a), inputs, threads)
        return a

    def matrix_evaluate(self, cts_ntt: np.ndarray, ring: np.ndarray, targets=None,
                        threads: int = 1) -> np.ndarray:
        cts_ntt = u64(cts_ntt)
        ring = u64(ring)
        inputs = cts_ntt.size // (2 * self.data_k * self.n)
        out = np.zeros((2, self.data_k, self.n), dtype=np.uint64)
        if targets is None:
            lib().or_matrix_evaluate(self._c, _p(cts_ntt), inputs, _p(ring), None, 0, _p(out), threads)
        else:
            tg = u64(targets)
            lib().or_matrix_evaluate(self._c, _p(cts_ntt), inputs, _p(ring), _p(tg), tg.size,
                                     _p(out), threads)
        return out

    # ---- masking / Enc0 -------------------------------------------------------------
    def scale_plain(self, m: int) -> list[int]:
        out = (U64 * self.data_k)()
        lib().or_scale_plain(self._c, m, out)
        return [int(v) for v in out]

    def sub_plain(self, c0: np.ndarray, mask: np.ndarray) -> np.ndarray:
        a = u64(c0).copy()
        lib().or_sub_plain(self._c, _p(a), _p(u64(mask)))
        return a

    def add_plain(self, c0: np.ndarray, plain: np.ndarray) -> np.ndarray:
        a = u64(c0).copy()
        p = u64(plain)
        lib().or_add_plain(self._c, _p(a), _p(p), p.size)
        return a

    def enc0(self, samples: np.ndarray, pk: np.ndarray) -> np.ndarray:
        out = np.zeros((2, self.data_k, self.n), dtype=np.uint64)
        lib().or_enc0(self._c, _p(u64(samples)), _p(u64(pk)), _p(out))
        return out

    def moddown(self, x: np.ndarray) -> np.ndarray:
        out = np.zeros((self.data_k, self.n), dtype=np.uint64)
        lib().or_moddown(self._c, _p(u64(x)), _p(out))
        return out

    def add(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = u64(a).copy()
        lib().or_add_inplace(self._c, _p(a), _p(u64(b)), a.size // self.n)
        return a

    # ---- Galois / keyswitch -------------------------------------------------------
    def galois(self, polys: np.ndarray, elt: int, prime_count: int | None = None) -> np.ndarray:
        a = u64(polys)
        out = np.zeros_like(a)
        pc = self.data_k if prime_count is None else prime_count
        lib().or_galois(self._c, _p(a), _p(out), a.size // self.n, pc, elt)
        return out

    def keyswitch(self, ct: np.ndarray, key: np.ndarray, elt: int) -> np.ndarray:
        out = np.zeros((2, self.data_k, self.n), dtype=np.uint64)
        lib().or_keyswitch_galois(self._c, _p(u64(ct)), _p(u64(key)), elt, _p(out))
        return out

    def keyswitch_many(self, cts: np.ndarray, keys: np.ndarray, elts, threads: int = 1) -> np.ndarray:
        cts = u64(cts)
        keys = u64(keys)
        el = (ctypes.c_uint32 * len(elts))(*[int(e) for e in elts])
        count = cts.size // (2 * self.data_k * self.n)
        out = np.zeros((len(elts), count, 2, self.data_k, self.n), dtype=np.uint64)
        lib().or_keyswitch_many(self._c, _p(cts), count, _p(keys), el, len(elts), _p(out), threads)
        return out

    def monomial_shift(self, ct: np.ndarray, exponent: int) -> np.ndarray:
        a = u64(ct).copy()
        lib().or_monomial_shift(self._c, _p(a), exponent)
        return a

    def packing_pair(self, left, right, key_one, key_level, level: int) -> np.ndarray:
        out = np.zeros((2, self.data_k, self.n), dtype=np.uint64)
        lib().or_packing_pair(self._c, _p(u64(left)), _p(u64(right)), _p(u64(key_one)),
                              _p(u64(key_level)), level, _p(out))
        return out

    def client_phase(self, c1: np.ndarray, sk_ntt: np.ndarray) -> np.ndarray:
        out = np.zeros((self.data_k, self.n), dtype=np.uint64)
        lib().or_client_phase(self._c, _p(u64(c1)), _p(u64(sk_ntt)), _p(out))
        return out

    def token_evaluate(self, inputs_ntt, slots, ring, scaled) -> np.ndarray:
        out = np.zeros((slots, 2, self.data_k, self.n), dtype=np.uint64)
        lib().or_token_evaluate(self._c, _p(u64(inputs_ntt)), slots, _p(u64(ring)), _p(u64(scaled)),
                                _p(out))
        return out

    def token_local_scaled(self, shares, slots, ring) -> np.ndarray:
        out = np.zeros((slots, self.data_k), dtype=np.uint64)
        lib().or_token_local_scaled(self._c, _p(u64(shares)), slots, _p(u64(ring)), _p(out))
        return out

    def uniform(self, seed: int, polys: int, prime_count: int | None = None) -> np.ndarray:
        pc = self.data_k if prime_count is None else prime_count
        out = np.zeros((polys, self.n), dtype=np.uint64)
        lib().or_fill_uniform(seed, _p(self.q_arr), pc, self.n, polys, _p(out))
        return out


def art002() -> Ctx:
    return Ctx(ART002_N, ART002_PRIMES, data_k=6, t=ART002_T)


# --------------------------------------------------------------------------------
# packing
# --------------------------------------------------------------------------------
@dataclass(frozen=True)
class Packing:
    reduction: int
    columns: int
    returns: int
    inputs: int


def matrix_packing(b: int, k: int, o: int) -> Packing:
    out = _OrPacking()
    if lib().or_matrix_packing(b, k, o, ctypes.byref(out)) != 0:
        raise ValueError("E_MATRIX_SHAPE")
    return Packing(int(out.reduction), int(out.columns), int(out.returns), int(out.inputs))


def packed_rows_per_ciphertext(d: int) -> int:
    return int(lib().or_packed_rows_per_ciphertext(d))


def pack_inputs(x: list[list[int]], d: int, blocks: int, n: int) -> np.ndarray:
    """x[b][blk*d+j] at coefficient b*(2d-1)+j of input block blk (bfv_matrix.inc:25-29)."""
    stride = 2 * d - 1
    out = np.zeros((blocks, n), dtype=np.uint64)
    for blk in range(blocks):
        for b, row in enumerate(x):
            for j in range(d):
                if blk * d + j < len(row):
                    out[blk, b * stride + j] = row[blk * d + j] & MASK59
    return out


def pack_weights(w_block_rows: list[list[list[int]]], d: int, batch: int, n: int) -> np.ndarray:
    """w[o][j] of block blk at coefficient o*B*(2d-1)+d-1-j (bfv_matrix.inc:156-160).
    w_block_rows[blk][o][j]."""
    stride = 2 * d - 1
    out = np.zeros((len(w_block_rows), n), dtype=np.uint64)
    for blk, rows in enumerate(w_block_rows):
        for o, row in enumerate(rows):
            for j, v in enumerate(row):
                out[blk, o * batch * stride + d - 1 - j] = v & MASK59
    return out


def targets(count: int, batch: int, d: int) -> list[int]:
    """(o*B+b)*(2d-1)+d-1 for o < count, b < B (bfv_matrix.inc:162-163)."""
    stride = 2 * d - 1
    return [(o * batch + b) * stride + d - 1 for o in range(count) for b in range(batch)]


# --------------------------------------------------------------------------------
# multi-precision pieces (GMP in the reference)
# --------------------------------------------------------------------------------
def crt(residues, primes) -> int:
    """rns_coefficient (bfv.cpp:138-147): sum_j a_j * (Q/q_j) * ((Q/q_j)^-1 mod q_j) mod Q."""
    Q = 1
    for p in primes:
        Q *= int(p)
    out = 0
    for a, p in zip(residues, primes):
        p = int(p)
        part = Q // p
        out += int(a) * part * pow(part, -1, p)
    return out % Q


def decode(phase: int, Q: int, t: int = ART002_T) -> int:
    """round(t*phase/Q) mod t, the value the locked decode circuit outputs
    (bfv.cpp:328-356: numerator = phase*2^59 + floor(q/2), quotient by q, low 59 bits)."""
    return ((phase * t + Q // 2) // Q) % t


# --------------------------------------------------------------------------------
# test-only BFV key material and encryption over the oracle's arithmetic
# --------------------------------------------------------------------------------
class TestBfv:
    """Seeded test keys (ternary s, uniform a, small e), public-key encryption and
    decryption.  pk = (-a*s + e, a) in NTT form at the key level, as the reference's
    PublicZero and matrix paths consume it (enc0/seal_adapter.cpp:179-181)."""

    def __init__(self, ctx: Ctx, seed: int = 1):
        self.ctx = ctx
        self.rng = np.random.default_rng(seed)
        n, k = ctx.n, ctx.k
        s = self.rng.integers(-1, 2, size=n)
        self.s_signed = s
        self.sk_coeff = self._signed_to_rns(s, k)  # [k][n]
        self.sk_ntt = ctx.ntt(self.sk_coeff, prime_count=k)  # [k][n]
        a = ctx.uniform(int(self.rng.integers(1 << 62)), k, prime_count=k)
        e = self._signed_to_rns(self.rng.integers(-3, 4, size=n), k)
        a_ntt = a  # uniform residues are a valid NTT-form polynomial
        e_ntt = ctx.ntt(e, prime_count=k)
        pk0 = np.zeros((k, n), dtype=np.uint64)
        for p, q in enumerate(ctx.primes):
            prod = (a_ntt[p].astype(object) * self.sk_ntt[p].astype(object)) % q
            pk0[p] = np.array([(int(e_ntt[p, z]) - int(prod[z])) % q for z in range(n)], dtype=np.uint64)
        self.pk = np.stack([pk0, a_ntt])  # [2][k][n]

    def _signed_to_rns(self, v, k) -> np.ndarray:
        out = np.zeros((k, self.ctx.n), dtype=np.uint64)
        for p in range(k):
            q = self.ctx.primes[p]
            out[p] = np.array([int(x) % q for x in v], dtype=np.uint64)
        return out

    def samples(self) -> np.ndarray:
        """[3][k][n]: ternary u, then e0, e1 (small centred values)."""
        k, n = self.ctx.k, self.ctx.n
        u = self._signed_to_rns(self.rng.integers(-1, 2, size=n), k)
        e0 = self._signed_to_rns(self.rng.integers(-5, 6, size=n), k)
        e1 = self._signed_to_rns(self.rng.integers(-5, 6, size=n), k)
        return np.stack([u, e0, e1])

    def encrypt(self, plain) -> np.ndarray:
        """Enc(0) then add the Delta-scaled plaintext to c0 (coefficient form,
        data level): [2][data_k][n]."""
        ct = self.ctx.enc0(self.samples(), self.pk)
        plain = u64(plain)
        ct[0] = self.ctx.add_plain(ct[0], plain)
        return ct

    def sk_data_ntt(self) -> np.ndarray:
        return np.ascontiguousarray(self.sk_ntt[: self.ctx.data_k])

    def phase_at(self, ct: np.ndarray, index: int) -> int:
        """c0 + c1*s at one coefficient, CRT'd to [0,Q)."""
        u = self.ctx.client_phase(ct[1], self.sk_data_ntt())
        dk = self.ctx.data_k
        res = [(int(ct[0][p][index]) + int(u[p][index])) % self.ctx.primes[p] for p in range(dk)]
        return crt(res, self.ctx.primes[:dk])

    def decrypt(self, ct: np.ndarray) -> list[int]:
        u = self.ctx.client_phase(ct[1], self.sk_data_ntt())
        dk = self.ctx.data_k
        Q = self.ctx.Q
        out = []
        for z in range(self.ctx.n):
            res = [(int(ct[0][p][z]) + int(u[p][z])) % self.ctx.primes[p] for p in range(dk)]
            out.append(decode(crt(res, self.ctx.primes[:dk]), Q, self.ctx.t))
        return out

    def galois_key(self, elt: int, target: "TestBfv | None" = None) -> np.ndarray:
        """Key [data_k][2][k][n] switching sigma_elt(s) -> target's s (self if None):
        key_j = (-a_j*s' + e_j + q_s*sigma(s)*[p == j], a_j) in NTT form, the acyclic
        key shape of bfv_acyclic_pack.hpp:23-36 (q_s = special prime)."""
        ctx = self.ctx
        tgt = target or self
        k, dk, n = ctx.k, ctx.data_k, ctx.n
        sig = ctx.galois(self.sk_coeff, elt, prime_count=k)
        sig_ntt = ctx.ntt(sig, prime_count=k)
        special = ctx.primes[-1]
        key = np.zeros((dk, 2, k, n), dtype=np.uint64)
        for j in range(dk):
            a = ctx.uniform(int(self.rng.integers(1 << 62)), k, prime_count=k)
            e = ctx.ntt(self._signed_to_rns(self.rng.integers(-3, 4, size=n), k), prime_count=k)
            for p, q in enumerate(ctx.primes):
                a_o = a[p].astype(object)
                prod = (a_o * tgt.sk_ntt[p].astype(object)) % q
                b = (e[p].astype(object) - prod) % q
                if p == j:
                    b = (b + (special % q) * sig_ntt[p].astype(object)) % q
                key[j, 0, p] = np.array(list(b), dtype=np.uint64)
                key[j, 1, p] = a[p]
        return key

"""Slot-packed (BFV batching) matrix-vector product: the plaintext side.

The benchmark's config 3 multiplies an int8 weight matrix W [O][K] by one token's vector
x in Z_t (t = 65537, n = 8192) with BFV slot packing and rotate-and-sum.  The reference's
own matrix protocol packs coefficients instead (bfv_layout.hpp:14-27), so this product has
no counterpart there; it is built from this library's hoisted rotations and multi-block
ct-pt product (`bfvgpu.SlotMatvec`, C ABI `bfvgpu_slots_*`).

Slots.  With t = 1 mod 2n the plaintext ring splits into n slots, the evaluations at the
odd powers of a primitive 2n-th root psi mod t.  They form two rows of n/2: row 0 slot i
is the evaluation at psi^(3^i), row 1 slot i at psi^(-3^i), so the automorphism X -> X^(3^r)
rotates both rows left by r and X -> X^(2n-1) swaps the rows (the standard batching layout
of SEAL's BatchEncoder).  A negacyclic forward NTT in bit-reversed order holds the
evaluation at psi^(2 brv(j) + 1) at position j, so encoding scatters slot values to their
positions and runs the inverse NTT mod t; decoding runs the forward NTT and gathers.

Product.  x is packed with period K in both rows, row 1 shifted by K/2.  With the
extended diagonals diag_k[i] = W[i][(i + k) mod K] (i < O, zero beyond), row 0 covers
k < K/2 and row 1 covers K/2 + k, and baby * giant = K/2:
    y = sum_g rot( sum_b pt[g][b] . rot(x, b), g*baby ),   pt[g][b] = rot(diag pair, -g*baby)
after which adding the row-swapped ciphertext leaves y[i] = sum_j W[i][j] x[j] in row 0.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def _brv(x: int, bits: int) -> int:
    r = 0
    for _ in range(bits):
        r = (r << 1) | (x & 1)
        x >>= 1
    return r


def slot_positions(n: int) -> np.ndarray:
    """NTT position (bit-reversed evaluation order) of every slot: [n] int64, a permutation."""
    logn = n.bit_length() - 1
    m, half = 2 * n, n // 2
    pos = np.empty(n, dtype=np.int64)
    e = 1
    for i in range(half):
        pos[i] = _brv((e - 1) >> 1, logn)
        pos[half + i] = _brv((m - e - 1) >> 1, logn)
        e = e * 3 % m
    return pos


def split_steps(half_k: int) -> tuple[int, int]:
    """(baby, giant) with baby * giant = half_k (a power of two), baby >= giant."""
    if half_k <= 0 or half_k & (half_k - 1):
        raise ValueError("E_SLOTS_SHAPE")
    lg = half_k.bit_length() - 1
    baby = 1 << ((lg + 1) // 2)
    return baby, half_k // baby


def rotation_elements(n: int, baby: int, giant: int) -> list[int]:
    """Galois elements of the keys SlotMatvec takes, in its order."""
    m = 2 * n
    return ([pow(3, b, m) for b in range(1, baby)] + [pow(3, g * baby, m) for g in range(1, giant)] + [m - 1])


@dataclass(frozen=True)
class SlotLayout:
    n: int
    inner: int    # K
    outputs: int  # O
    t: int = 65537

    def __post_init__(self):
        half = self.n // 2
        if self.inner % 2 or half % self.inner or not 0 < self.outputs <= half:
            raise ValueError("E_SLOTS_SHAPE")
        if (self.t - 1) % (2 * self.n):
            raise ValueError("E_SLOTS_PLAIN_MODULUS")

    @property
    def steps(self) -> tuple[int, int]:
        return split_steps(self.inner // 2)

    def pack_input(self, x) -> np.ndarray:
        """Slot vector [n] of x [K] (values in Z_t): row 0 x[i mod K], row 1 x[(i + K/2) mod K]."""
        x = np.asarray(x, dtype=np.int64) % self.t
        half, K = self.n // 2, self.inner
        i = np.arange(half)
        return np.concatenate([x[i % K], x[(i + K // 2) % K]])

    def diagonals_device(self, torch, w):
        """w [O][K] integer tensor (device) -> pre-rotated diagonal slot vectors
        [giant][baby][n] int64 (values mod t) on the same device."""
        baby, giant = self.steps
        half, K, O = self.n // 2, self.inner, self.outputs
        dev = w.device
        wt = torch.remainder(w.to(torch.int64), self.t)
        g = torch.arange(giant, device=dev).view(giant, 1, 1)
        b = torch.arange(baby, device=dev).view(1, baby, 1)
        i = torch.arange(half, device=dev).view(1, 1, half)
        j = torch.remainder(i - g * baby, half)  # diagonal index before the -g*baby rotation
        rows = []
        for r in range(2):
            k = r * (K // 2) + g * baby + b
            col = torch.remainder(j + k, K)
            inside = j < O
            v = wt[torch.clamp(j, max=O - 1), col]
            rows.append(torch.where(inside, v, torch.zeros_like(v)))
        return torch.cat(rows, dim=2).contiguous()

    def encode_device(self, torch, plain_ctx, slots):
        """Slot vectors [..][n] (int64 device tensor, values < t) -> plaintext polynomials
        [..][n] (coefficients < t): scatter to NTT positions, inverse NTT mod t on the
        device (plain_ctx: a one-prime context for t)."""
        pos = torch.from_numpy(slot_positions(self.n)).to(slots.device)
        flat = slots.reshape(-1, self.n)
        poly = torch.empty_like(flat)
        poly[:, pos] = flat
        plain_ctx.ntt_device(poly, flat.shape[0], 1, 0, inverse=True)
        return poly.view(slots.shape)

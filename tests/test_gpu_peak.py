"""The integer-pipe peak kernels (bfvgpu_int_peak_device) do the work they are credited with.

The bench divides each hot kernel's algorithmic operation count by these kernels' measured
rates, so a peak kernel whose loop the compiler shortened would inflate every integer
fraction.  Here one block runs a few iterations of each kind and every thread's checksum is
recomputed on the host from the same start values, twiddles and prime: the kernel must have
performed exactly blocks x 256 x 8 x iters operations of its kind (kinds 4 and 5 run on
the FP64 pipe and end with canonical residues, so only the residues are compared there).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

M64 = (1 << 64) - 1
THREADS, CHAINS = 256, 8


def _start(thread: int, chain: int, which: int, q: int) -> int:
    z = (thread * 0x9E3779B97F4A7C15 + (chain * 2 + which) * 0xD1B54A32D192ED03 + 1) & M64
    z ^= z >> 31
    z = (z * 0xBF58476D1CE4E5B9) & M64
    z ^= z >> 29
    return z % q


def _expected(kind: int, iters: int, q: int, tw) -> list[int]:
    out = []
    for thread in range(THREADS):
        a = [_start(thread, j, 0, q) for j in range(CHAINS)]
        b = [_start(thread, j, 1, q) for j in range(CHAINS)]
        if kind == 0:
            for _ in range(iters):
                for j in range(CHAINS):
                    w, wq = tw[j & 3]
                    x = a[j] - 2 * q if a[j] >= 2 * q else a[j]
                    t = (b[j] * w - ((b[j] * wq) >> 64) * q) & M64
                    a[j], b[j] = (x + t) & M64, (x + 2 * q - t) & M64
        elif kind == 1:
            acc = [0] * CHAINS
            for _ in range(iters):
                for j in range(CHAINS):
                    acc[j] = (acc[j] + a[j] * b[j]) & ((1 << 128) - 1)
                    a[j] = acc[j] & M64
            b = [v >> 64 for v in acc]
        elif kind == 2:
            for _ in range(iters):
                for j in range(CHAINS):
                    a[j] = a[j] * b[j] % q
        elif kind == 3:
            for _ in range(iters):
                for j in range(CHAINS):
                    a[j] = a[j] * tw[j & 3][0] % q
        elif kind == 4:  # residues only: the FP64 path's representatives are made canonical
            for _ in range(iters):
                for j in range(CHAINS):
                    w = tw[j & 3][0]
                    for _ in range(2):
                        t = b[j] * w % q
                        a[j], b[j] = (a[j] + t) % q, (a[j] - t) % q
        else:
            for _ in range(iters):
                for j in range(CHAINS):
                    a[j] = a[j] * tw[j & 3][0] % q
        h = 0
        for j in range(CHAINS):
            h ^= (a[j] * 0x9E3779B97F4A7C15 + b[j]) & M64
        out.append(h)
    return out


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4, 5])
def test_int_peak_checksums(bfv, oracle, kind):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    n, bits = 8192, [50, 50, 50, 50, 60]
    primes = oracle.coeff_modulus(n, bits)
    ctx = bfv.Context(n, primes, 4, 1, 65537, device=0)
    fwd, _, _ = ctx.tables(0)
    fwd = np.asarray(fwd, dtype=np.uint64).reshape(n, 2)
    tw = [(int(fwd[i, 0]), int(fwd[i, 1])) for i in range(1, 5)]
    iters = 3
    sink = torch.zeros(THREADS, dtype=torch.int64, device="cuda")
    ops = ctx.int_peak_device(kind, 1, iters, sink)
    torch.cuda.synchronize()
    assert ops == THREADS * CHAINS * iters * (2 if kind == 4 else 1)
    got = sink.cpu().numpy().view(np.uint64).tolist()
    assert got == _expected(kind, iters, primes[0], tw)

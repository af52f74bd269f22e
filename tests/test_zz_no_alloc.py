"""The allocation-free keyswitch entry point (bfvgpu_keyswitch_device_noalloc).

Callers such as a protocol worker whose device footprint is fixed and audited when the
session starts, or code that cannot afford cudaMalloc's implicit device synchronisation,
cannot allocate the scratch buffer that bfvgpu_keyswitch_device needs.  The variant
takes only inputs and outputs and works in a fixed 8 MiB array inside the library's
device image.  This test calls it through the C ABI twice in a row, with different
ciphertexts, keys and Galois elements, and requires its output to equal the allocating
entry point's bit for bit (the tolerance of every parity test here), then checks that a
batch beyond the array's limit is refused with a clear error before any device work.

The file name sorts last so that a run stopping at the first failure has already run
every other test; it passes alone in a fresh process and after the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N = 8192
BITS = [50, 50, 50, 50, 60]
LIMIT_BYTES = 8 << 20


def _uniform(rng, shape, primes):
    """Residues uniform in [0, q) with the prime chosen by the limb axis (-2)."""
    q = np.array(primes, dtype=np.uint64).reshape(*([1] * (len(shape) - 2)), len(primes), 1)
    raw = rng.integers(0, 1 << 62, size=shape, dtype=np.uint64)
    return np.ascontiguousarray(raw % q)


def test_noalloc_keyswitch_matches_allocating_entry_point(bfv):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    primes = bfv.find_primes(N, BITS)
    ctx = bfv.Context(N, primes, 4, 1, 65537, device=0)
    L = bfv.lib()
    count = LIMIT_BYTES // (2 * 5 * N * 8)  # 12: the most the fixed array holds here
    assert count == 12
    rng = np.random.default_rng(20261201)
    for call, elt in enumerate((3, pow(3, 9, 2 * N))):
        cts = _uniform(rng, (count, 2, 4, N), primes[:4])
        key = _uniform(rng, (4 * 2, 5, N), primes)
        d_cts = torch.from_numpy(cts.view(np.int64)).cuda()
        d_key = torch.from_numpy(key.view(np.int64)).cuda()
        scratch = torch.empty(ctx.keyswitch_scratch_words(count), dtype=torch.int64, device="cuda")
        out_ref = torch.empty_like(d_cts)
        out_na = torch.full_like(d_cts, -1)
        torch.cuda.synchronize()
        ctx.keyswitch_device(d_cts, count, d_key, elt, scratch, out_ref)
        rc = L.bfvgpu_keyswitch_device_noalloc(ctx.handle, d_cts.data_ptr(), count, d_key.data_ptr(), elt,
                                               out_na.data_ptr(), None)
        assert rc == 0, L.bfvgpu_last_error()
        torch.cuda.synchronize()
        assert torch.equal(out_na, out_ref), f"call {call}: differs from bfvgpu_keyswitch_device"
    # an empty batch is a no-op, as for the allocating entry point
    assert L.bfvgpu_keyswitch_device_noalloc(ctx.handle, d_cts.data_ptr(), 0, d_key.data_ptr(), 3,
                                             out_na.data_ptr(), None) == 0
    # one ciphertext beyond the fixed array: refused before any device work
    rc = L.bfvgpu_keyswitch_device_noalloc(ctx.handle, d_cts.data_ptr(), count + 1, d_key.data_ptr(), 3,
                                           out_na.data_ptr(), None)
    assert rc == 3  # BFVGPU_E_SHAPE
    assert b"E_BFVGPU_NOALLOC_SCRATCH_LIMIT" in L.bfvgpu_last_error()

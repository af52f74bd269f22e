"""The C ABI library loads and exports every entry point include/bfvgpu.h declares;
host-only behaviour (prime search, host contexts, validation that needs no device)."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "bfvgpu.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bfvgpu_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(bfv):
    L = bfv.lib()
    names = declared_functions()
    assert len(names) >= 40
    for name in names:
        assert hasattr(L, name), name
    # the Python binding covers every declared entry point
    assert set(names) <= set(bfv.EXPORTED)


def test_error_names(bfv):
    L = bfv.lib()
    assert L.bfvgpu_version() == 1
    assert L.bfvgpu_error_name(0) == b"BFVGPU_OK"
    assert L.bfvgpu_error_name(9) == b"BFVGPU_E_CUDA"
    assert L.bfvgpu_error_name(99) == b"BFVGPU_E_UNKNOWN"


def test_find_primes_matches_oracle(bfv, oracle):
    assert bfv.find_primes(16384, [60] * 7) == oracle.ART002_PRIMES
    assert bfv.find_primes(4096, [36, 36, 37]) == oracle.coeff_modulus(4096, [36, 36, 37])
    assert bfv.find_primes(8192, [50, 50, 50, 50, 60]) == oracle.coeff_modulus(8192, [50, 50, 50, 50, 60])
    with pytest.raises(bfv.BfvGpuInvalidArgument):
        bfv.find_primes(3000, [60])


def test_host_context_validation(bfv, oracle):
    bad = list(oracle.ART002_PRIMES)
    bad[2] += 2  # not prime / not 1 mod 2n
    with pytest.raises(bfv.BfvGpuInvalidArgument):
        bfv.Context(16384, bad, 6, 1, 1 << 59, device=-1)
    with pytest.raises(bfv.BfvGpuInvalidArgument):
        bfv.Context(1000, oracle.ART002_PRIMES, 6, 1, 1 << 59, device=-1)
    with pytest.raises(bfv.BfvGpuInvalidArgument):
        bfv.Context(16384, oracle.ART002_PRIMES[:6] + [oracle.ART002_PRIMES[0]], 6, 1, 1 << 59, device=-1)
    hc = bfv.Context.art002(device=-1)
    assert hc.k == 7 and hc.dk == 6
    fwd, inv, invn = hc.tables(0)
    assert fwd.shape == (16384, 2) and int(fwd[0, 0]) == 1
    hc.close()


def test_fp64_mode_switch_on_host(bfv, oracle):
    """bfvgpu_ctx_set_fp64: the prime records carry the FP64 flag and constants for primes
    below 2^50 only when the mode is on; the 60-bit special prime never; bad values rejected."""
    import ctypes
    import numpy as np
    primes = oracle.coeff_modulus(8192, [50, 50, 50, 50, 60])
    hc = bfv.Context(8192, primes, 4, 1, 65537, device=-1)
    m = np.asarray(hc.moduli())
    assert list(m[:, 10]) == [1, 1, 1, 1, 0]
    qinv = m[:4, 11].copy().view(np.float64)
    assert all(abs(float(v) * q - 1.0) < 1e-15 for v, q in zip(qinv, primes[:4]))
    hc.set_fp64(False)
    assert not np.asarray(hc.moduli())[:, 10].any()
    hc.set_fp64(True)
    assert list(np.asarray(hc.moduli())[:, 10]) == [1, 1, 1, 1, 0]
    from bfvgpu._lib import lib
    assert lib().bfvgpu_ctx_set_fp64(hc.handle, 2) != 0
    art = bfv.Context.art002(device=-1)
    assert not np.asarray(art.moduli())[:, 10].any()
    hc.close()
    art.close()


def test_host_only_context_refuses_device_work(bfv, gpu_available):
    hc = bfv.Context.art002(device=-1)
    with pytest.raises(bfv.BfvGpuError) as e:
        bfv.NttBatch(hc, key_level=False, batches=1)
    assert e.value.name == "BFVGPU_E_DEVICE"
    with pytest.raises(bfv.BfvGpuError):
        bfv.Matrix(hc, np.zeros((1, 2, 6, 16384), dtype=np.uint64))


@pytest.mark.parametrize("where", ["first", "last", "none"])
def test_canonical_check_of_a_large_batch(bfv, oracle, where):
    """A 64-ciphertext ART-002 batch (12.6 M words) is scanned by several host threads: a
    residue >= its prime in the first or the last polynomial is found; a clean batch passes
    validation and is refused only for the host-only context."""
    hc = bfv.Context.art002(device=-1)
    cts = np.zeros((64, 2, 6, 16384), dtype=np.uint64)
    if where == "first":
        cts[0, 0, 0, 7] = oracle.ART002_PRIMES[0]
    elif where == "last":
        cts[-1, -1, -1, -1] = oracle.ART002_PRIMES[5]
    with pytest.raises(bfv.BfvGpuError) as e:
        bfv.Matrix(hc, cts)
    assert e.value.name == ("BFVGPU_E_DEVICE" if where == "none" else "BFVGPU_E_CANONICAL")
    hc.close()


def test_device_context_without_gpu_fails_loudly(bfv, gpu_available):
    if gpu_available:
        pytest.skip("a GPU is present")
    with pytest.raises(bfv.BfvGpuError) as e:
        bfv.Context.art002(device=0)
    assert e.value.name == "BFVGPU_E_DEVICE"


def test_matrix_layout_helpers(bfv, oracle):
    x = np.arange(2 * 40, dtype=np.uint64).reshape(2, 40) + np.uint64(1 << 59)  # high bits masked
    ours = bfv.pack_inputs(x, 16, 3, 64)
    ref = oracle.pack_inputs([[int(v) for v in row] for row in x], 16, 3, 64)
    assert np.array_equal(ours, ref)
    blocks = [[[1, 2, 3], [4, 5, 6]], [[7, 8, 9], [(1 << 59) - 1, 0, 1]]]
    assert np.array_equal(bfv.pack_weights(blocks, 16, 2, 256), oracle.pack_weights(blocks, 16, 2, 256))
    assert bfv.targets(3, 2, 16) == oracle.targets(3, 2, 16)

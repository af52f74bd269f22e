"""The C++ drop-in boundary (include/bfvgpu_ref.hpp) compiled and run.

tests/cpp/adapter_check.cpp uses the reference-named adapter classes (matrix_gpu::Matrix,
Switch, PublicZero, NttBatch, TokenWeights) exactly as a C++ call site would, built with g++
against libbfvgpu.so.  On the CPU it checks every constructor's validation and error type on
a host-only context; on the GPU it runs Matrix::evaluate / evaluate_selective, Switch::apply,
NttBatch::transform and PublicZero::encrypt_from_samples, and this file compares their
outputs with the oracle word for word (plus close() records and use after close).
"""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "adapter_check.cpp")
OUT = os.path.join(ROOT, "tests", "cpp", "_build", "adapter_check")
LIBDIR = os.path.join(ROOT, "privacy-rag_b200", "lib")
CUDA_LIB = "/usr/local/cuda/lib64"


@pytest.fixture(scope="module")
def adapter_bin(built_lib):
    deps = [SRC, os.path.join(ROOT, "include", "bfvgpu_ref.hpp"), os.path.join(ROOT, "include", "bfvgpu.h"),
            built_lib]
    if not os.path.exists(OUT) or any(os.path.getmtime(d) > os.path.getmtime(OUT) for d in deps):
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        SRC, "-o", OUT, "-L", LIBDIR, "-lbfvgpu", "-L", CUDA_LIB, "-lcudart",
                        f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{CUDA_LIB}"], check=True)
    return OUT


def _run(binary, *args):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_adapter_validation_host_only(adapter_bin):
    assert _run(adapter_bin, "host").strip() == "host ok"


@pytest.mark.gpu
def test_adapter_calls_on_gpu(adapter_bin, oracle, tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    oc = oracle.art002()
    n, k, dk = oc.n, oc.k, oc.data_k
    rng = np.random.default_rng(4242)
    inputs = 3
    cts = oc.uniform(31, inputs * 2 * dk).reshape(inputs, 2, dk, n)
    ring = rng.integers(0, 1 << 59, size=(inputs, n), dtype=np.uint64)
    targets = np.array([0, 5, 63, 4000, n - 1], dtype=np.uint64)
    key = oc.uniform(32, dk * 2 * k, prime_count=k).reshape(dk, 2, k, n)
    elt = 2 * 5 + 1
    ct = oc.uniform(33, 2 * dk).reshape(2, dk, n)
    ntt_in = oc.uniform(34, 2 * dk)
    tb = oracle.TestBfv(oc, seed=35)
    samples = tb.samples()
    for name, a in (("cts", cts), ("ring", ring), ("targets", targets), ("key", key), ("ct", ct),
                    ("elt", np.array([elt], dtype=np.uint64)), ("ntt_in", ntt_in), ("pk", tb.pk),
                    ("samples", samples)):
        np.ascontiguousarray(a, dtype=np.uint64).tofile(tmp_path / f"{name}.bin")
    assert _run(adapter_bin, "gpu", str(tmp_path)).strip() == "gpu ok"
    got = lambda name: np.fromfile(tmp_path / f"{name}_out.bin", dtype=np.uint64)
    cn = oc.matrix_open(cts, threads=8)
    full = oc.matrix_evaluate(cn, ring, threads=8)
    assert np.array_equal(got("matrix").reshape(2, dk, n), full)
    sel = full.copy()
    keep = np.zeros(n, dtype=bool)
    keep[targets.astype(np.int64)] = True
    sel[0][:, ~keep] = 0
    assert np.array_equal(got("matrix_selective").reshape(2, dk, n), sel)
    assert np.array_equal(got("switch").reshape(2, dk, n), oc.keyswitch(ct, key, elt))
    assert np.array_equal(got("ntt").reshape(2 * dk, n), oc.ntt(ntt_in, prime_count=dk))
    assert np.array_equal(got("enc0").reshape(2, dk, n), oc.enc0(samples, tb.pk))

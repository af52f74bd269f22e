"""Shared fixtures.  `-m "not gpu"` runs everywhere (oracle, host logic, CPU emulation
of the kernel bodies, ABI exports); `-m gpu` needs an sm_100 device."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "privacy-rag_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; runs the CUDA path")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O  # noqa: E402  (tests/ may use the oracle as the checker)
    O.build()
    return O


@pytest.fixture(scope="session")
def built_lib():
    sys.path.insert(0, PKG)
    import build as B  # privacy-rag_b200/build.py
    return B.build()


@pytest.fixture(scope="session")
def bfv(built_lib):
    import bfvgpu
    bfvgpu.lib()
    return bfvgpu


@pytest.fixture(scope="session")
def emu(built_lib):
    """libemu.so: the kernel bodies compiled for the host (tests/emu/emu.cpp)."""
    import ctypes
    here = os.path.join(ROOT, "tests", "emu")
    out = os.path.join(here, "libemu.so")
    src = os.path.join(here, "emu.cpp")
    deps = [src] + [os.path.join(PKG, "csrc", f) for f in ("arith.cuh", "f64mod.cuh", "layout.cuh", "ntt_core.cuh", "block_ops.cuh")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["/usr/bin/g++", "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", "-x", "c++",
                        "-I", os.path.join(PKG, "csrc"), src, "-o", out], check=True)
    return ctypes.CDLL(out)


@pytest.fixture(scope="session")
def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False

"""Build libbfvgpu.so (sm_100a) in-tree with nvcc.

Usage: python privacy-rag_b200/build.py [--verbose]
The library lands in privacy-rag_b200/lib/libbfvgpu.so, next to the Python mirror,
so it travels with the repository snapshot to a GPU host.
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib", "libbfvgpu.so")
SOURCES = ["kernels.cu", "bfvgpu.cu", "noalloc.cu", "peak.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def dependencies() -> list[str]:
    """Every file the library is compiled from: the sources, every header beside them and
    the public headers (a new header is picked up without editing this list)."""
    deps = [os.path.join(CSRC, f) for f in SOURCES]
    deps += [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(ROOT, "include")  # the C ABI headers (the C++ adapters are header-only users)
    deps += [os.path.join(inc, f) for f in sorted(os.listdir(inc)) if f.endswith(".h")]
    deps.append(os.path.abspath(__file__))
    return deps


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in dependencies())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmds, objs = [], []
    for src in SOURCES:
        obj = os.path.join(PKG, "lib", src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
               "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        cmds.append(cmd)
        objs.append(obj)
    # the translation units compile independently: run them side by side
    with concurrent.futures.ThreadPoolExecutor(len(cmds)) as pool:
        for f in [pool.submit(subprocess.run, c, check=True) for c in cmds]:
            f.result()
    cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-lpthread"]
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose="--verbose" in sys.argv))

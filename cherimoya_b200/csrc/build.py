"""Build libcherimoya_b200.so (sm_100a) in-tree with nvcc.

    python -m cherimoya_b200.csrc.build [--verbose]

The library is plain CUDA C++ behind the C ABI of include/cherimoya_b200.h
(no torch headers), so it builds in seconds and loads with ctypes.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libcherimoya_b200.so")
SOURCES = [os.path.join(HERE, "chm_engine.cu")]
DEPS = SOURCES + [os.path.join(HERE, f) for f in ("chm_kernels.cuh", "chm_ptx.cuh")] + [
    os.path.join(ROOT, "include", "cherimoya_b200.h")]


def nvcc_path():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build(verbose=False, force=False):
    if not force and not needs_build():
        return LIB
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
           "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2", "-o", LIB + ".tmp"] + SOURCES
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libcherimoya_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    print(LIB)

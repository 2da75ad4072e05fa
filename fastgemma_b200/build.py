"""Compile the sm_100a CUDA library in-tree: fastgemma_b200/libfgm_cuda.so.

    python -m fastgemma_b200.build [-v]

nvcc cross-compiles for sm_100a without a GPU.  Objects go to
fastgemma_b200/_build/ and are rebuilt when a source or header is newer.
No fast-math: the kernels rely on IEEE f32 rounding for bit-exact parity.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfgm_cuda.so")
HOST = os.path.join(PKG, "host")
HOST_LIB = os.path.join(PKG, "libfgm_host.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
                     "-Xptxas", "-O3", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    hdr_time = _newest(headers)
    objs, procs = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_time):
            continue
        cmd = [nvcc()] + NVCC_FLAGS + (extra or []) + ["-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for s, p in procs:
        out = p.communicate()[0].decode()
        if verbose or p.returncode:
            sys.stdout.write(out)
        if p.returncode:
            failed.append(s)
    if failed:
        raise RuntimeError(f"nvcc failed on {failed}")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + \
            ["-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    build_host(verbose)
    return LIB


def build_host(verbose: bool = False) -> str:
    """The C++ host layer (host/fgm_host.cpp, host/fgm_model.cpp) over the C ABI: libfgm_host.so,
    linked against libfgm_cuda.so beside it."""
    srcs = [os.path.join(HOST, "fgm_host.cpp"), os.path.join(HOST, "fgm_model.cpp")]
    deps = srcs + [os.path.join(HOST, "fgm_host.hpp"), os.path.join(HOST, "fgm_model.hpp"),
                   os.path.join(INCLUDE, "fgm_cuda.h"), LIB]
    if os.path.exists(HOST_LIB) and os.path.getmtime(HOST_LIB) >= _newest(deps):
        return HOST_LIB
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-I", INCLUDE, "-I", HOST,
           "-o", HOST_LIB] + srcs + ["-L", PKG, "-lfgm_cuda", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return HOST_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))

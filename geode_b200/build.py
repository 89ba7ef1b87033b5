"""Builds the package's native libraries in-tree (so they travel with the repository snapshot):

- ``geode_b200/libgeode_cuda.so``: the CUDA backend and operators (geode_b200/csrc/*.cu, sm_100a), C ABI in
  include/geode_cuda.h;
- ``geode_b200/libgeode_host.so``: the C++ host side (geode_b200/host/*.cpp): the pack reader, the Model-shaped
  verify / keep interface and the speculation step over the backend, C ABI in include/geode_host.h.

``python -m geode_b200.build`` (or ``build()``) recompiles what is older than its sources.
"""
from __future__ import annotations

import glob
import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CUDA_SO = os.path.join(PKG, "libgeode_cuda.so")
HOST_SO = os.path.join(PKG, "libgeode_host.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC"]


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(force: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu")))
    deps = srcs + glob.glob(os.path.join(PKG, "csrc", "*.cuh")) + glob.glob(os.path.join(PKG, "csrc", "*.hpp")) + \
        [os.path.join(ROOT, "include", "geode_cuda.h")]
    if not force and not _stale(CUDA_SO, deps):
        return CUDA_SO
    bdir = os.path.join(PKG, "_build")
    os.makedirs(bdir, exist_ok=True)
    objs = []
    procs = []
    for s in srcs:
        o = os.path.join(bdir, os.path.basename(s) + ".o")
        objs.append(o)
        cmd = [NVCC, *ARCH, *CUDA_FLAGS, "-c", s, "-o", o]
        procs.append((cmd, subprocess.Popen(cmd)))
    for cmd, p in procs:
        if p.wait() != 0:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))
    subprocess.check_call([NVCC, *ARCH, "-shared", "-o", CUDA_SO, *objs, "-lcudart", "-lcuda", "-ldl"])
    return CUDA_SO


def build_host(force: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(PKG, "host", "*.cpp")))
    if not srcs:
        return ""
    deps = srcs + glob.glob(os.path.join(PKG, "host", "*.hpp")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    if not force and not _stale(HOST_SO, deps):
        return HOST_SO
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-I" + os.path.join(ROOT, "include"),
                           "-o", HOST_SO, *srcs, "-ldl", "-lpthread"])
    return HOST_SO


def build(force: bool = False):
    build_cuda(force)
    build_host(force)


if __name__ == "__main__":
    build(force=True)

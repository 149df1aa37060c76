"""Build recipe for the jules_b200 shared library (sm_100a).

``python -m jules_b200.build`` compiles jules_b200/csrc into
jules_b200/_lib/libjules_b200.so with nvcc (cross-compiles without a GPU).
The library is self-contained: static CUDA runtime, no libcuda link (the
tensor-map encoder is fetched through the runtime's driver entry point).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIB_DIR, "libjules_b200.so")

SOURCES = ["capi.cu", "host_api.cpp"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith(".cuh"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "-I" + os.path.join(ROOT, "include")]


def nccl_include() -> list:
    """-I for an NCCL include directory that has the device API headers
    (nccl_device.h, NCCL >= 2.28: symmetric windows, multicast pointers), if
    one is installed; without it the library builds with the multicast
    gather compiled out.  $JULES_NCCL_INCLUDE overrides the search."""
    cands = [os.environ.get("JULES_NCCL_INCLUDE")]
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia")
        for loc in (spec.submodule_search_locations or []) if spec else []:
            cands.append(os.path.join(loc, "nccl", "include"))
    except Exception:
        pass
    for d in cands:
        if d and os.path.exists(os.path.join(d, "nccl_device.h")):
            return ["-I" + d]
    return []


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files += [os.path.join(ROOT, "include", "jules_kernels.h")]
    inc = os.path.join(ROOT, "include", "jules", "Kernel")
    files += [os.path.join(inc, f) for f in sorted(os.listdir(inc))]
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc()] + NVCC_FLAGS + nccl_include() + ["-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

"""Build libhif4x.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

Each csrc/*.cu is compiled separately (codec.cu with -fmad=false as a
safety net: its arithmetic is written with explicit round-to-nearest
intrinsics and must never be contracted) and linked into
hif4x/libhif4x.so next to this file.  Rebuilds only when a source or header
is newer than the library.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # hif4-contest_b200/
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
OBJ = os.path.join(ROOT, "_build")
SO = os.path.join(PKG, "libhif4x.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I", INCLUDE, "-I", CSRC]
PER_FILE = {"codec.cu": ["-fmad=false"]}


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def stale() -> bool:
    if not os.path.exists(SO):
        return True
    t = os.path.getmtime(SO)
    return any(os.path.getmtime(d) > t for d in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    if not force and not stale():
        return SO
    os.makedirs(OBJ, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src in sources():
        name = os.path.basename(src)
        obj = os.path.join(OBJ, name + ".o")
        cmd = [nvcc, *ARCH, *COMMON, *PER_FILE.get(name, []), "-c", src, "-o", obj]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = SO + ".tmp"
    subprocess.check_call([nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"])
    os.replace(tmp, SO)
    return SO


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
    print(SO)

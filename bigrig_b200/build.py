"""Build libbigrig_b200.so (sm_100a) in-tree with nvcc.

    python -m bigrig_b200.build            # build if any source is newer than the library
    python -m bigrig_b200.build --force    # rebuild
    python -m bigrig_b200.build --ptxas-v  # also print register / spill / smem usage

The library is a plain C-ABI shared object (include/bigrig_b200.h); the Python
host loads it with ctypes.  Objects go to bigrig_b200/_build/, the library next to
this file so that it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libbigrig_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def sources() -> list:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target: str, deps: list) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, ptxas_v: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if ptxas_v or _stale(obj, [src] + headers()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if ptxas_v:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        if ptxas_v:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, ptxas_v: bool = False) -> str:
    """Compile every .cu under csrc/ and link libbigrig_b200.so; return its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, ptxas_v), srcs))
    if force or ptxas_v or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-ldl",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_v=a.ptxas_v))

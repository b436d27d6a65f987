"""Build the sm_100a C-ABI library ``dsv4attn/libdsv4attn.so`` in-tree.

    python tt-deepseek-v4_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (no PTX for other
architectures, no JIT) and links one shared library against the shared
CUDA runtime, so the process that loads it through ctypes shares one
runtime (and one primary context) with PyTorch.  Objects are rebuilt only
when a source or header is newer than the library.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "dsv4attn")
LIB = os.path.join(OUT_DIR, "libdsv4attn.so")
OBJ_DIR = os.path.join(HERE, "_build")

GENCODE = "-gencode=arch=compute_100a,code=sm_100a"
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", GENCODE, "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or add the CUDA toolkit to PATH)")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _sources() + _headers() + [__file__])


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    nvcc = find_nvcc()
    os.makedirs(OBJ_DIR, exist_ok=True)
    objs = []
    hdr_t = max(os.path.getmtime(p) for p in _headers())
    for src in _sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) > max(os.path.getmtime(src), hdr_t):
            continue
        cmd = [nvcc, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if ptxas_info:
            cmd[1:1] = ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc, GENCODE, "-shared", "-cudart", "shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    sys.exit(0)

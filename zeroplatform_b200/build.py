"""Builds libzero_tensor.so (the C-ABI library with every CUDA kernel) in-tree for sm_100a.

    python -m zeroplatform_b200.build          # incremental
    python -m zeroplatform_b200.build --clean  # from scratch

nvcc cross-compiles without a GPU.  Objects go to zeroplatform_b200/_build/, the library to
zeroplatform_b200/libzero_tensor.so (both git-ignored; the .so travels with the source tree).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libzero_tensor.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max(os.path.getmtime(p) for p in [src] + _headers())
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep and not verbose_ptxas:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(clean: bool = False, verbose_ptxas: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/shared-memory usage")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose_ptxas=a.ptxas_v))

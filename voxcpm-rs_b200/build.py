"""Build libvoxcpm_b200.so in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` is compiled to an object file (in parallel) under ``_build/`` and
linked into ``voxcpm-rs_b200/libvoxcpm_b200.so`` with the CUDA runtime linked statically.
Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
ROOT = os.path.dirname(PKG_DIR)
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libvoxcpm_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if "-Xptxas" in extra and r.stderr:
            sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with ThreadPoolExecutor(max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))

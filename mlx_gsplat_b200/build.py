"""Build ``libgsplat_b200.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m mlx_gsplat_b200.build`` (or ``build()`` from Python).
The library is a plain C ABI (``include/gsplat_b200.h``) loaded with ctypes;
no PyTorch headers are involved.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libgsplat_b200.so")
BUILD_DIR = os.path.join(PKG, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC")
    return cand


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale(objs, srcs) -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    srcs = sources()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = [os.path.join(BUILD_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if not force and not _stale(objs, srcs):
        return LIB
    nvcc = _nvcc()
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(pair):
        src, obj = pair
        cmd = [nvcc, *flags, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(compile_one, zip(srcs, objs)))
    if verbose:
        for s, log in zip(srcs, logs):
            if log.strip():
                print(f"--- {os.path.basename(s)}\n{log}", file=sys.stderr)
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    xs = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else []
    print(build(force="-f" in sys.argv or bool(xs), verbose=v or bool(xs), extra_flags=xs))

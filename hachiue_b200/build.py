"""Builds libhachiue_cuda.so in-tree with nvcc for sm_100a (B200).

    python -m hachiue_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` compiles to an object under ``hachiue_b200/_build/`` (in
parallel), then one shared library ``hachiue_b200/libhachiue_cuda.so`` is
linked with the static CUDA runtime.  Nothing needs a GPU.
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
LIB = os.path.join(PKG, "libhachiue_cuda.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max(os.path.getmtime(f) for f in files)


def _compile(src: str, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile every CUDA source and link the C-ABI library.  Returns its path."""
    extra = list(extra or [])
    if not force and not extra and os.path.exists(LIB) and os.path.getmtime(LIB) >= _deps_mtime():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage per kernel")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())

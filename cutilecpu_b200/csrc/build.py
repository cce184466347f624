"""Build libkernels.so (the C-ABI kernel library) for sm_100a, in-tree.

Every ``*.cu`` file in this directory is compiled by nvcc to an object under
``cutilecpu_b200/_build/`` and linked into ``cutilecpu_b200/libkernels.so``.
Only the CUDA runtime is linked; the driver API entry points the tensor-map
code needs are resolved at run time through ``cudaGetDriverEntryPoint``.
Rebuilds are incremental on source/header modification times.

Usage: ``python -m cutilecpu_b200.csrc.build [--force] [--debug-checks]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "libkernels.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(ROOT / "include"),
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: cannot build libkernels.so")
    return cand


def _deps() -> list[Path]:
    return sorted(HERE.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(out: Path, srcs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs)


def _compile(src: Path, extra: list[str], force: bool, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src] + _deps()):
        cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose_ptxas:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, debug_checks: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile every kernel source and link ``libkernels.so``; return its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(HERE.glob("*.cu"))
    extra = ["-DMK_DEBUG_CHECKS=1"] if debug_checks else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, force, verbose_ptxas), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of libkernels.so failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug-checks", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, debug_checks=a.debug_checks, verbose_ptxas=a.ptxas_v))

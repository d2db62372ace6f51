"""Build ``libtvk.so`` (all CUDA sources under ``csrc/``) in-tree for sm_100a.

Usage: ``python -m tinyvllm_b200.build [--force] [--verbose]``.  Objects go to
``tinyvllm_b200/_build/``; the shared library lands next to this file so it
travels with the source tree.  Rebuilds only when a source or header is newer
than the library.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libtvk.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    if not force and not needs_build():
        return LIB
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
        return obj

    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print register / smem usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    lib = build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose, extra_flags=extra)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())

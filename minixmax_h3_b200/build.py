"""Builds the in-tree C-ABI library ``libh3b.so`` for sm_100a.

Every ``csrc/*.cu`` file is compiled by nvcc (in parallel, skipped when the
object is newer than its sources) and linked into one shared library next to
this file, with the CUDA runtime linked statically.  Python loads the library
through ctypes (``_lib.py``); C/C++ callers link it directly against
``include/h3b.h``.

    python -m minixmax_h3_b200.build [--force] [--verbose]
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
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libh3b.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libh3b.so")
    return cand


def _deps(src: Path) -> list[Path]:
    return [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.hpp"), *INCLUDE.glob("*.h")]


def _compile(src: Path, force: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists():
        newest = max(p.stat().st_mtime for p in _deps(src))
        if obj.stat().st_mtime >= newest:
            return obj, ""
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles csrc/*.cu and links libh3b.so; returns the library path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError("no CUDA sources under csrc/")
    with cf.ThreadPoolExecutor(max_workers=min(len(sources), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), sources))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    relink = force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs)
    if relink:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()

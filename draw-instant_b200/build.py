"""Builds libdi.so (all CUDA sources under csrc/) in-tree for sm_100a with nvcc.

Usage: python draw-instant_b200/build.py [--force]
Objects go to draw-instant_b200/_build/, the shared library to draw-instant_b200/libdi.so.
Cross-compiles without a GPU.  Rebuilds a translation unit only when it or a header changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libdi.so"
INCLUDE = PKG.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]
HOST_CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else None


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime():
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, verbose_ptxas: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if HOST_CXX:
        cmd += ["-ccbin", HOST_CXX]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl", "-lrt",
               "-lpthread"]
        if HOST_CXX:
            cmd += ["-ccbin", HOST_CXX]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))

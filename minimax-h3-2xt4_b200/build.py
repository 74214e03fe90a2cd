"""Builds libh3b200.so (the sm_100a kernels behind include/h3b200.h) in-tree.

    python minimax-h3-2xt4_b200/build.py [--force] [--verbose]

Every .cu file under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with --fmad=false, so no floating-point
multiply-add is contracted behind the explicit __f*_rn intrinsics, and linked into
h3tp/_lib/libh3b200.so next to the Python package that loads it.  The static CUDA
runtime is linked in; the driver's cuTensorMapEncodeTiled is looked up at run time,
so the library needs no libcuda at link time and cross-compiles on a machine
without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT_DIR = HERE / "h3tp" / "_lib"
LIB = OUT_DIR / "libh3b200.so"
OBJ_DIR = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
         "-I" + str(INCLUDE), "-I" + str(CSRC)]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libh3b200.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links the library; returns its path.  Skips work when the sources
    are unchanged since the last build (a stamp file holds their digest)."""
    stamp = OUT_DIR / ".stamp"
    digest = _digest()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    cc = nvcc()

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, sources()))
    if verbose:
        for obj, log in results:
            print(f"== {obj.name}\n{log}")
    objs = [str(o) for o, _ in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    path = build(force=a.force, verbose=a.verbose)
    print(path)
    sys.exit(0)

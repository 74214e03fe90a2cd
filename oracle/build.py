"""Build recipe of the CPU oracle (test infrastructure only).

    python oracle/build.py

Compiles oracle/h3_oracle.c with gcc into oracle/_build/libh3oracle.so.  The flags
matter: -ffp-contract=off keeps every float operation a separate IEEE rounding (no
FMA contraction), and no -ffast-math.  OpenMP parallelises the per-row loops.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "h3_oracle.c"
OUT = HERE / "_build" / "libh3oracle.so"
FLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
         "-fopenmp", "-Wall"]


def build(force: bool = False) -> Path:
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc is required to build the CPU oracle")
    stamp = OUT.with_suffix(".stamp")
    digest = hashlib.sha256(SRC.read_bytes() + " ".join(FLAGS).encode()).hexdigest()
    if not force and OUT.exists() and stamp.exists() and stamp.read_text() == digest:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    r = subprocess.run([cc, *FLAGS, str(SRC), "-o", str(tmp), "-lm"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, OUT)
    stamp.write_text(digest)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))

"""Build the CPU oracle library (test infrastructure only).

    python oracle/build.py

Compiles oracle.c with gcc into oracle/lib/liboracle.so.  IEEE semantics are
required: no -ffast-math, and -ffp-contract=off so that a*b+c stays two
roundings (fmaf is written out where the formulation fuses).
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "oracle.c"
LIB = HERE / "lib" / "liboracle.so"
FLAGS = ["-O2", "-std=c11", "-Wall", "-Wextra", "-ffp-contract=off", "-fno-fast-math",
         "-fPIC", "-shared"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler found for the oracle")
    LIB.parent.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    proc = subprocess.run([cc, *FLAGS, "-o", str(tmp), str(SRC), "-lm"],
                          capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))

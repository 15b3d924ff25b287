"""Build the C-ABI shared library of the fused layer ops for sm_100a.

Compiles every ``csrc/*.cu`` with nvcc into ``lib/libanima_flat_b200.so``
inside the package (in-tree, so the built library travels with the source
tree).  The numerics contract needs IEEE fp32 division and square root and no
floating-point contraction, hence ``--fmad=false`` and no ``--use_fast_math``.

    python -m anima_flat_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

if __package__:
    from ._paths import LIB_DIR, LIB_PATH, PKG
else:  # run as a script
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from _paths import LIB_DIR, LIB_PATH, PKG

CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"

ARCH = "-gencode=arch=compute_100a,code=sm_100a"
NVCC_FLAGS = [
    ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--fmad=false",
    "-Xcompiler",
    "-fPIC,-O2",
    "-shared",
    "-cudart",
    "static",
]


def nvcc() -> str:
    """Path of nvcc (CUDA_HOME, /usr/local/cuda, or PATH)."""
    for root in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if root and (Path(root) / "bin" / "nvcc").exists():
            return str(Path(root) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if a source is newer than it (or ``force``)."""
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{CSRC}", f"-I{INCLUDE}", "-o", str(tmp)]
    cmd += [str(s) for s in sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr}")
    if verbose and proc.stderr:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()

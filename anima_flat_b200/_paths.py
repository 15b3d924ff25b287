"""Locations of the in-tree build products."""

from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_DIR = PKG / "lib"
LIB_PATH = LIB_DIR / "libanima_flat_b200.so"

"""ctypes binding of ``include/anima_flat_b200.h``.

The shared library is the only compute path: there is no CPU or Triton
fallback, and loading fails loudly when the library is missing.  Every entry
point returns a cudaError_t; a non-zero code is raised as ``RuntimeError``
carrying the library's message.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_void_p
from pathlib import Path

from ._paths import LIB_PATH

_P = c_void_p
_I = c_int64
_F = c_float

# name -> argument types, in header order.  Kept in sync with
# include/anima_flat_b200.h (a CPU test checks every declared symbol).
SIGNATURES: dict[str, tuple] = {
    "afb_residual_adaln": (_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P),
    "afb_adaln": (_P, _P, _P, _P, _I, _I, _I, _F, _P),
    "afb_residual_adaln_fp8": (_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P),
    "afb_adaln_fp8": (_P, _P, _P, _P, _P, _I, _I, _I, _F, _P),
    "afb_rowquant": (_P, _P, _P, _I, _I, c_int, _P),
    "afb_gelu_probe": (_P, _P, _P, _I, _P),
    "afb_silu_probe": (_P, _P),
    "afb_wait_probe": (ctypes.c_uint32, _P, _P),
    "afb_qkv_norm_rope": (_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P),
    "afb_head_norm": (_P, _P, _P, _I, _I, _I, _I, _F, _P),
    "afb_residual_adaln_bwd": (_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P,
                               ctypes.c_size_t, _P),
    "afb_adaln_bwd": (_P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P, ctypes.c_size_t, _P),
    "afb_residual_adaln_bwd_noalloc": (_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I,
                                       _F, _P),
    "afb_qkv_norm_rope_bwd": (_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P,
                              ctypes.c_size_t, _P),
    "afb_head_norm_bwd": (_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, ctypes.c_size_t, _P),
    "afb_ctx_scale": (_P, _P, _P, _P, _I, _I, _I, _I, _P),
    "afb_ctx_scale_rowquant": (_P, _P, _P, _P, _P, _I, _I, _I, _I, _P),
    "afb_ctx_scale_bwd": (_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P),
    "afb_rms_silu": (_P, _P, _P, _P, _P, _I, _I, _I, _I, c_int, _P),
    "afb_rms_silu_bwd": (_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, c_int, _P, ctypes.c_size_t, _P),
}

# Workspace-size queries: name -> argument types (return size_t).
WORKSPACE_QUERIES: dict[str, tuple] = {
    "afb_residual_adaln_bwd_workspace": (_I, _I, _I),
    "afb_adaln_bwd_workspace": (_I, _I, _I),
    "afb_qkv_norm_rope_bwd_workspace": (_I, _I, _I, _I),
    "afb_head_norm_bwd_workspace": (_I, _I, _I, _I),
    "afb_rms_silu_bwd_workspace": (_I, _I),
}

_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    """The in-tree shared library (override with AFB_LIBRARY)."""
    env = os.environ.get("AFB_LIBRARY")
    return Path(env) if env else LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"anima_flat_b200 CUDA library not found at {path}; "
            "build it with `python -m anima_flat_b200.build`"
        )
    lib = ctypes.CDLL(str(path))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = c_int
    for name, argtypes in WORKSPACE_QUERIES.items():
        fn = getattr(lib, name)
        fn.argtypes = list(argtypes)
        fn.restype = ctypes.c_size_t
    lib.afb_abi_version.restype = c_int
    lib.afb_abi_version.argtypes = []
    lib.afb_last_error.restype = ctypes.c_char_p
    lib.afb_last_error.argtypes = []
    lib.afb_device_status.argtypes = [ctypes.POINTER(c_int)]
    lib.afb_device_status.restype = c_int
    lib.afb_take_device_status.argtypes = [ctypes.POINTER(c_int)]
    lib.afb_take_device_status.restype = c_int
    lib.afb_set_pdl.argtypes = [c_int]
    lib.afb_set_pdl.restype = None
    lib.afb_get_pdl.argtypes = []
    lib.afb_get_pdl.restype = c_int
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call entry point `name`; raise RuntimeError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.afb_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with status {rc}: {msg}")


def workspace(name: str, device, *dims: int):
    """A float32 device buffer of the size the entry point `name` asks for
    (allocated through torch's caching allocator) and its size in bytes."""
    import torch

    nbytes = int(getattr(load(), f"{name}_workspace")(*dims))
    buf = torch.empty(max(1, (nbytes + 3) // 4), dtype=torch.float32, device=device)
    return buf, nbytes


def set_pdl(enabled: bool) -> None:
    """Turn programmatic dependent launch on or off for later launches."""
    load().afb_set_pdl(1 if enabled else 0)

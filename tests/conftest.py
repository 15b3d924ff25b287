"""Test configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on a CPU-only machine (oracle vs golden vectors, host
logic, C-ABI exports, gloo multi-process logic); ``-m gpu`` runs the CUDA
parity tests on a B200 through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def to_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns; e4m3 -> uint8; others -> numpy."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    """uint16 bit patterns -> bf16 tensor; float arrays -> float tensor."""
    if a.dtype == np.uint16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """One bf16 ulp at the magnitude of v (normal range floor)."""
    a = np.abs(v.astype(np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def ulp_diff_ok(ours_bits: np.ndarray, ref_f32: np.ndarray, ulps: float = 2.0,
                mag: np.ndarray | None = None) -> tuple[bool, float]:
    """|ours - ref| <= ulps * bf16_ulp(m) elementwise, m = ref or the given
    operand magnitude; returns (ok, worst ratio)."""
    ours = (ours_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    ref = ref_f32.astype(np.float64)
    scale = np.maximum(np.abs(ref), np.abs(mag)) if mag is not None else ref
    ratio = np.abs(ours - ref) / bf16_ulp(scale)
    worst = float(ratio.max()) if ratio.size else 0.0
    return worst <= ulps, worst


def bf16_ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 steps between two arrays of bf16 bit patterns (the
    patterns mapped to a monotone integer line, so -0 and +0 are 0 apart)."""
    def line(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(line(a_bits) - line(b_bits))


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")

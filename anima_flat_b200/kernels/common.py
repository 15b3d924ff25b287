"""Argument checks and launch plumbing shared by the op modules.

Mirrors src/kernels/common.py:6-9 (``_check``).  The reference's run-time
autotuner (``tuned_rows``, common.py:12-34) has no counterpart: every launch
shape here is fixed by the tensor shapes, so results never depend on timing.
"""

from __future__ import annotations

import torch

BF16 = torch.bfloat16


def _check(*ts: torch.Tensor) -> None:
    """Raise ValueError unless every tensor is on CUDA (common.py:6-9)."""
    for t in ts:
        if not t.is_cuda:
            raise ValueError("CUDA tensors required")


def _check_dtype(dtype: torch.dtype, what: str, *ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != dtype:
            raise ValueError(f"{what} must be {dtype}, got {t.dtype}")


def _check_vec(t: torch.Tensor, batch: int, dim: int, name: str) -> None:
    """Per-sample modulation vectors are [batch, dim] (adaln.py:34, :44-45)."""
    if t.numel() != batch * dim or t.shape[-1] != dim:
        raise ValueError(f"{name} must be [batch, dim] = [{batch}, {dim}], got {list(t.shape)}")


def _stream(t: torch.Tensor) -> int:
    """Handle of the current CUDA stream on the tensor's device."""
    return torch.cuda.current_stream(t.device).cuda_stream

"""FP8 activation quantisation: ``adaln_fp8``, ``residual_adaln_fp8``, ``rowquant``.

Drop-in for the activation-quantisation half of src/kernels/fp8.py
(fp8.py:56-232 and :260-328): same functions, signatures, output shapes
(``q`` [B, S, D] float8_e4m3fn, ``s`` [B*S, 1] float32) and ValueErrors.  The
outputs feed ``fp8_linear`` (``torch._scaled_mm`` with row scales,
fp8.py:234-257) unchanged; the weight-side helpers of that module are GEMM
plumbing and stay with the reference.

Per row: ``s = max(max|y|, 1e-12) / 448`` and ``q = e4m3(clamp(y / s, +-448))``
where ``y`` is the un-rounded fp32 AdaLN output (fp8.py:93-97) or the input,
optionally after the A&S 7.1.26 GELU (fp8.py:260-292).
"""

from __future__ import annotations

import torch

from .._lib import call
from .common import BF16, _check, _check_dtype, _check_vec, _stream

__all__ = ["FP8", "FP8_MAX", "adaln_fp8", "residual_adaln_fp8", "rowquant"]

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0


def _qs(B: int, S: int, D: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    return (
        torch.empty(B, S, D, dtype=FP8, device=device),
        torch.empty(B * S, 1, dtype=torch.float32, device=device),
    )


@torch.library.custom_op("anima_flat_b200::residual_adaln_fp8", mutates_args=())
def _residual_adaln_fp8(
    x: torch.Tensor,
    residual: torch.Tensor,
    gate: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    B, S, D = residual.shape
    q, s = _qs(B, S, D, residual.device)
    z = torch.empty_like(residual)
    call(
        "afb_residual_adaln_fp8",
        x.data_ptr(), residual.data_ptr(), gate.data_ptr(), shift.data_ptr(), scale.data_ptr(),
        q.data_ptr(), s.data_ptr(), z.data_ptr(), B, S, D, eps, _stream(residual),
    )
    return q, s, z


@_residual_adaln_fp8.register_fake
def _(x, residual, gate, shift, scale, eps):
    B, S, D = residual.shape
    q, s = _qs(B, S, D, residual.device)
    return q, s, torch.empty_like(residual)


@torch.library.custom_op("anima_flat_b200::adaln_fp8", mutates_args=())
def _adaln_fp8(
    z: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, D = z.shape
    q, s = _qs(B, S, D, z.device)
    call(
        "afb_adaln_fp8",
        z.data_ptr(), shift.data_ptr(), scale.data_ptr(), q.data_ptr(), s.data_ptr(),
        B, S, D, eps, _stream(z),
    )
    return q, s


@_adaln_fp8.register_fake
def _(z, shift, scale, eps):
    B, S, D = z.shape
    return _qs(B, S, D, z.device)


@torch.library.custom_op("anima_flat_b200::rowquant", mutates_args=())
def _rowquant(x: torch.Tensor, gelu: bool) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, K = x.shape
    q, s = _qs(B, S, K, x.device)
    call("afb_rowquant", x.data_ptr(), q.data_ptr(), s.data_ptr(), B * S, K, int(gelu), _stream(x))
    return q, s


@_rowquant.register_fake
def _(x, gelu):
    B, S, K = x.shape
    return _qs(B, S, K, x.device)


def _validate(x: torch.Tensor, *vecs: torch.Tensor) -> None:
    if x.ndim != 3:
        raise ValueError(f"expected [B, S, D] activations, got {list(x.shape)}")
    _check_dtype(BF16, "activations and modulation vectors", x, *vecs)
    B, _, D = x.shape
    for name, v in zip(("gate", "shift", "scale")[-len(vecs):], vecs):
        _check_vec(v, B, D, name)


def residual_adaln_fp8(
    x: torch.Tensor,
    residual: torch.Tensor,
    gate: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    eps: float = 1e-6,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``residual_adaln`` whose modulated output is returned as FP8 with a scale per token.

    Args:
        x: Sub-layer output, shape ``[B, S, D]`` bf16.
        residual: Residual stream, same shape and dtype as ``x``.
        gate: Gate, shape ``[B, D]``.
        shift: Shift, shape ``[B, D]``.
        scale: Scale (already including the +1), shape ``[B, D]``.
        eps: LayerNorm epsilon.

    Returns:
        ``(q, s, z)``: the FP8 output ``[B, S, D]``, its float32 token scales
        ``[B * S, 1]``, and the updated residual stream ``z`` ``[B, S, D]``.

    Raises:
        ValueError: If a tensor is not on CUDA, ``x`` and ``residual`` differ in
            shape or dtype, or a dtype/shape is unsupported.
    """
    _check(x, residual, gate, shift, scale)
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError("x and residual must match")
    _validate(residual, gate, shift, scale)
    return _residual_adaln_fp8(
        x.contiguous(),
        residual.contiguous(),
        gate.contiguous(),
        shift.contiguous(),
        scale.contiguous(),
        eps,
    )


def adaln_fp8(
    z: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6
) -> tuple[torch.Tensor, torch.Tensor]:
    """``adaln`` whose output is returned as FP8 with a scale per token.

    Args:
        z: Tokens, shape ``[B, S, D]`` bf16.
        shift: Shift, shape ``[B, D]``.
        scale: Scale (already including the +1), shape ``[B, D]``.
        eps: LayerNorm epsilon.

    Returns:
        ``(q, s)``: the FP8 output ``[B, S, D]`` and its float32 token scales ``[B * S, 1]``.

    Raises:
        ValueError: If a tensor is not on CUDA or a dtype/shape is unsupported.
    """
    _check(z, shift, scale)
    _validate(z, shift, scale)
    return _adaln_fp8(z.contiguous(), shift.contiguous(), scale.contiguous(), eps)


def rowquant(x: torch.Tensor, gelu: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize tokens to FP8 with a scale per token, optionally applying GELU first.

    Args:
        x: Tokens, shape ``[B, S, K]`` bf16, K a multiple of 16 up to 16384.
        gelu: Apply the A&S 7.1.26 GELU before quantizing.

    Returns:
        ``(q, s)``: the FP8 tokens ``[B, S, K]`` and their float32 scales ``[B * S, 1]``,
        as accepted by ``fp8_linear``.

    Raises:
        ValueError: If ``x`` is not on CUDA or a dtype/shape is unsupported.
    """
    _check(x)
    if x.ndim != 3:
        raise ValueError(f"expected [B, S, K] tokens, got {list(x.shape)}")
    _check_dtype(BF16, "x", x)
    return _rowquant(x.contiguous(), bool(gelu))

"""AdaLN modulate: ``adaln`` and ``residual_adaln`` (forward and backward).

Drop-in for src/kernels/adaln.py: same public functions, argument order,
defaults, output order and ValueErrors (adaln.py:298-314).  The custom ops are
registered under the ``anima_flat_b200`` namespace so they can be loaded next
to the reference's ``anima_flat`` ops.

Formulation (adaln.py:26-46), per row with b = row // S:
    z = bf16(residual + bf16(gate[b] * x))
    h = bf16(LN(z) * scale[b] + shift[b])      LN affine-free, eps 1e-6
``scale`` already includes the +1 (model.py:228).
"""

from __future__ import annotations

import torch

from .._lib import call, workspace
from .common import BF16, _check, _check_dtype, _check_vec, _stream

__all__ = ["adaln", "residual_adaln"]


@torch.library.custom_op("anima_flat_b200::residual_adaln", mutates_args=())
def _residual_adaln(
    x: torch.Tensor,
    residual: torch.Tensor,
    gate: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, D = residual.shape
    h = torch.empty_like(residual)
    z = torch.empty_like(residual)
    call(
        "afb_residual_adaln",
        x.data_ptr(), residual.data_ptr(), gate.data_ptr(), shift.data_ptr(),
        scale.data_ptr(), h.data_ptr(), z.data_ptr(), B, S, D, eps, _stream(residual),
    )
    return h, z


@_residual_adaln.register_fake
def _(x, residual, gate, shift, scale, eps):
    return torch.empty_like(residual), torch.empty_like(residual)


@torch.library.custom_op("anima_flat_b200::adaln", mutates_args=())
def _adaln(z: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float) -> torch.Tensor:
    B, S, D = z.shape
    h = torch.empty_like(z)
    call(
        "afb_adaln",
        z.data_ptr(), shift.data_ptr(), scale.data_ptr(), h.data_ptr(), B, S, D, eps, _stream(z),
    )
    return h


@_adaln.register_fake
def _(z, shift, scale, eps):
    return torch.empty_like(z)


# ------------------------------------------------------------------ backward --
# adaln.py:175-257.  Per-column gradients of gate/shift/scale are summed over
# the rows in a fixed order (see csrc/adaln_bwd.cu), so they are reproducible.
@torch.library.custom_op("anima_flat_b200::residual_adaln_bwd", mutates_args=())
def _residual_adaln_bwd_op(
    gh: torch.Tensor,
    gz: torch.Tensor | None,
    z: torch.Tensor,
    x: torch.Tensor,
    gate: torch.Tensor,
    scale: torch.Tensor,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    B, S, D = z.shape
    gh = gh.contiguous()
    gz = gz.contiguous() if gz is not None else None
    dx = torch.empty_like(x)
    dres = torch.empty_like(z)
    dgate = torch.empty_like(gate)
    dshift = torch.empty_like(scale)
    dscale = torch.empty_like(scale)
    ws, nbytes = workspace("afb_residual_adaln_bwd", z.device, B, S, D)
    call(
        "afb_residual_adaln_bwd",
        gh.data_ptr(), gz.data_ptr() if gz is not None else None, z.data_ptr(), x.data_ptr(),
        gate.data_ptr(), scale.data_ptr(), dx.data_ptr(), dres.data_ptr(), dgate.data_ptr(),
        dshift.data_ptr(), dscale.data_ptr(), B, S, D, eps, ws.data_ptr(), nbytes, _stream(z),
    )
    return dx, dres, dgate, dshift, dscale


@_residual_adaln_bwd_op.register_fake
def _(gh, gz, z, x, gate, scale, eps):
    return (torch.empty_like(x), torch.empty_like(z), torch.empty_like(gate),
            torch.empty_like(scale), torch.empty_like(scale))


@torch.library.custom_op("anima_flat_b200::adaln_bwd", mutates_args=())
def _adaln_bwd_op(
    gh: torch.Tensor, z: torch.Tensor, scale: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    B, S, D = z.shape
    gh = gh.contiguous()
    dz = torch.empty_like(z)
    dshift = torch.empty_like(scale)
    dscale = torch.empty_like(scale)
    ws, nbytes = workspace("afb_adaln_bwd", z.device, B, S, D)
    call(
        "afb_adaln_bwd",
        gh.data_ptr(), z.data_ptr(), scale.data_ptr(), dz.data_ptr(), dshift.data_ptr(),
        dscale.data_ptr(), B, S, D, eps, ws.data_ptr(), nbytes, _stream(z),
    )
    return dz, dshift, dscale


@_adaln_bwd_op.register_fake
def _(gh, z, scale, eps):
    return torch.empty_like(z), torch.empty_like(scale), torch.empty_like(scale)


def _residual_adaln_setup(ctx, inputs, output):
    x, _, gate, _, scale, eps = inputs
    ctx.save_for_backward(x, gate, scale, output[1])
    ctx.eps = eps


def _residual_adaln_backward(ctx, gh, gz):
    x, gate, scale, z = ctx.saved_tensors
    dx, dres, dgate, dshift, dscale = _residual_adaln_bwd_op(gh, gz, z, x, gate, scale, ctx.eps)
    return dx, dres, dgate, dshift, dscale, None


torch.library.register_autograd(
    "anima_flat_b200::residual_adaln", _residual_adaln_backward, setup_context=_residual_adaln_setup
)


def _adaln_setup(ctx, inputs, output):
    z, _, scale, eps = inputs
    ctx.save_for_backward(z, scale)
    ctx.eps = eps


def _adaln_backward(ctx, gh):
    z, scale = ctx.saved_tensors
    dz, dshift, dscale = _adaln_bwd_op(gh, z, scale, ctx.eps)
    return dz, dshift, dscale, None


torch.library.register_autograd("anima_flat_b200::adaln", _adaln_backward, setup_context=_adaln_setup)


def _validate(x: torch.Tensor, *vecs: torch.Tensor) -> None:
    if x.ndim != 3:
        raise ValueError(f"expected [B, S, D] activations, got {list(x.shape)}")
    _check_dtype(BF16, "activations and modulation vectors", x, *vecs)
    B, _, D = x.shape
    for name, v in zip(("gate", "shift", "scale")[-len(vecs):], vecs):
        _check_vec(v, B, D, name)


def residual_adaln(x, residual, gate, shift, scale, eps=1e-6):
    """Gated residual add, then affine-free LayerNorm and modulation.

    Args:
        x: Sub-layer output, shape ``[B, S, D]`` bf16.
        residual: Residual stream, same shape and dtype as ``x``.
        gate: Gate, shape ``[B, D]``.
        shift: Shift, shape ``[B, D]``.
        scale: Scale (already including the +1), shape ``[B, D]``.
        eps: LayerNorm epsilon.

    Returns:
        ``(h, z)``: the modulated output and the updated residual stream.

    Raises:
        ValueError: If a tensor is not on CUDA, ``x`` and ``residual`` differ in
            shape or dtype, or a dtype/shape is unsupported.
    """
    _check(x, residual, gate, shift, scale)
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError("x and residual must match")
    _validate(residual, gate, shift, scale)
    return _residual_adaln(
        x.contiguous(),
        residual.contiguous(),
        gate.contiguous(),
        shift.contiguous(),
        scale.contiguous(),
        eps,
    )


def adaln(z, shift, scale, eps=1e-6):
    """Affine-free LayerNorm and modulation (``residual_adaln`` without the residual).

    Args:
        z: Tokens, shape ``[B, S, D]`` bf16.
        shift: Shift, shape ``[B, D]``.
        scale: Scale (already including the +1), shape ``[B, D]``.
        eps: LayerNorm epsilon.

    Returns:
        The modulated output ``h``, shape ``[B, S, D]``.

    Raises:
        ValueError: If a tensor is not on CUDA or a dtype/shape is unsupported.
    """
    _check(z, shift, scale)
    _validate(z, shift, scale)
    return _adaln(z.contiguous(), shift.contiguous(), scale.contiguous(), eps)

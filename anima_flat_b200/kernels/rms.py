"""Channel RMS norm + SiLU of the VAE decoder (``rms_silu`` family).

Drop-in for src/kernels/rms.py: same public functions ``rms_silu``,
``add_rms_silu`` and ``shuffle_rms_silu`` (rms.py:283-335), the custom ops
with fake impls and autograd (:157-280), including ``rms_silu_bwd``.  Per
pixel of C channels (channels last): ``y = silu(normalize(s) * sqrt(C) *
gamma)`` in fp32, rounded once; ``s`` is ``x``, ``bf16(x + residual)``, or the
depth-to-space gather of ``u``.  The gamma gradient comes back in gamma's
dtype (rms.py:225).

Deliberate restrictions (ValueError): bf16 activations, C a multiple of 8 in
[8, 1024] (the VAE uses 96, 192 and 384).
"""

from __future__ import annotations

import torch

from .._lib import call, workspace
from .common import _check, _stream

__all__ = ["add_rms_silu", "rms_silu", "shuffle_rms_silu"]


def _validate(x: torch.Tensor, gamma: torch.Tensor, channels: int) -> None:
    if x.dtype != torch.bfloat16:
        raise ValueError(f"activations must be torch.bfloat16, got {x.dtype}")
    if channels % 8 or not 8 <= channels <= 1024:
        raise ValueError(f"channels must be a multiple of 8 in [8, 1024], got {channels}")
    if gamma.numel() != channels:
        raise ValueError(f"gamma must have {channels} elements, got {gamma.numel()}")


def _gamma32(gamma: torch.Tensor) -> torch.Tensor:
    """gamma as a contiguous fp32 array on a 16-byte boundary (the kernels
    read it in 16-byte vectors)."""
    g32 = gamma.float().contiguous()
    return g32 if g32.data_ptr() % 16 == 0 else g32.clone()


def _fwd(x, r, gamma, shuffled):
    C = gamma.numel()
    if shuffled:
        B, h, w, _ = x.shape
        shape, H, W = (B, 2 * h, 2 * w, C), 2 * h, 2 * w
    else:
        shape, H, W = tuple(x.shape), 0, 0
    rows = 1
    for d in shape[:-1]:
        rows *= d
    y = x.new_empty(shape)
    s = x.new_empty(shape) if (r is not None or shuffled) else None
    g32 = _gamma32(gamma)
    call("afb_rms_silu", x.data_ptr(), r.data_ptr() if r is not None else None, g32.data_ptr(),
         s.data_ptr() if s is not None else None, y.data_ptr(), rows, H, W, C, int(shuffled), _stream(x))
    return s, y


@torch.library.custom_op("anima_flat_b200::rms_silu", mutates_args=())
def _rms_silu(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    _check(x)
    return _fwd(x.contiguous(), None, gamma, False)[1]


@_rms_silu.register_fake
def _(x, gamma):
    return torch.empty_like(x)


@torch.library.custom_op("anima_flat_b200::add_rms_silu", mutates_args=())
def _add_rms_silu(
    x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    _check(x)
    return _fwd(x.contiguous(), residual.contiguous(), gamma, False)


@_add_rms_silu.register_fake
def _(x, residual, gamma):
    return torch.empty_like(x), torch.empty_like(x)


@torch.library.custom_op("anima_flat_b200::shuffle_rms_silu", mutates_args=())
def _shuffle_rms_silu(u: torch.Tensor, gamma: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _check(u)
    return _fwd(u.contiguous(), None, gamma, True)


@_shuffle_rms_silu.register_fake
def _(u, gamma):
    B, h, w, _ = u.shape
    shape = (B, 2 * h, 2 * w, gamma.numel())
    return u.new_empty(shape), u.new_empty(shape)


@torch.library.custom_op("anima_flat_b200::rms_silu_bwd", mutates_args=())
def _rms_silu_bwd(
    s: torch.Tensor,
    gamma: torch.Tensor,
    dy: torch.Tensor,
    gs: torch.Tensor | None,
    shuffled: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    C = gamma.numel()
    s, dy = s.contiguous(), dy.contiguous()
    gs = gs.contiguous() if gs is not None else None
    rows = s.numel() // C
    if shuffled:
        B, H, W, _ = s.shape
        ds_shape = (B, H // 2, W // 2, 4 * C)
    else:
        H = W = 0
        ds_shape = tuple(s.shape)
    ds = s.new_empty(ds_shape)
    dg = torch.empty(C, dtype=torch.float32, device=s.device)
    ws, nbytes = workspace("afb_rms_silu_bwd", s.device, rows, C)
    g32 = _gamma32(gamma)
    call("afb_rms_silu_bwd", s.data_ptr(), g32.data_ptr(), dy.data_ptr(),
         gs.data_ptr() if gs is not None else None, ds.data_ptr(), dg.data_ptr(), rows, H, W, C,
         int(shuffled), ws.data_ptr(), nbytes, _stream(s))
    return ds, dg.to(gamma.dtype)


@_rms_silu_bwd.register_fake
def _(s, gamma, dy, gs, shuffled):
    if shuffled:
        B, H, W, _ = s.shape
        return s.new_empty((B, H // 2, W // 2, 4 * gamma.numel())), torch.empty_like(gamma)
    return torch.empty_like(s), torch.empty_like(gamma)


def _setup_rms_silu(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _bwd_rms_silu(ctx, dy):
    x, gamma = ctx.saved_tensors
    return _rms_silu_bwd(x, gamma, dy, None, False)


_rms_silu.register_autograd(_bwd_rms_silu, setup_context=_setup_rms_silu)


def _setup_add(ctx, inputs, output):
    ctx.save_for_backward(output[0], inputs[2])


def _bwd_add(ctx, gs, dy):
    s, gamma = ctx.saved_tensors
    ds, dg = _rms_silu_bwd(s, gamma, dy, gs, False)
    return ds, ds, dg


_add_rms_silu.register_autograd(_bwd_add, setup_context=_setup_add)


def _setup_shuffle(ctx, inputs, output):
    ctx.save_for_backward(output[0], inputs[1])


def _bwd_shuffle(ctx, gs, dy):
    s, gamma = ctx.saved_tensors
    return _rms_silu_bwd(s, gamma, dy, gs, True)


_shuffle_rms_silu.register_autograd(_bwd_shuffle, setup_context=_setup_shuffle)


def rms_silu(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """Channel RMS norm followed by SiLU: ``silu(normalize(x, -1) * sqrt(C) * gamma)``.

    Args:
        x: Activations with channels last, shape ``[..., C]``, bf16, CUDA.
        gamma: Per-channel scale, shape ``[C]``.

    Returns:
        Tensor with the shape and dtype of ``x``.
    """
    _validate(x, gamma, x.shape[-1])
    return _rms_silu(x, gamma)


def add_rms_silu(
    x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """Residual add followed by ``rms_silu`` of the sum.

    Returns:
        ``(x + residual, rms_silu(x + residual, gamma))``.
    """
    _validate(x, gamma, x.shape[-1])
    if residual.shape != x.shape or residual.dtype != x.dtype:
        raise ValueError("residual must match x in shape and dtype")
    return _add_rms_silu(x, residual, gamma)


def shuffle_rms_silu(u: torch.Tensor, gamma: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Depth-to-space by 2 followed by ``rms_silu``.

    Args:
        u: Sub-pixel activations ``[B, H, W, 4 * C]``; channel ``(2a + b) * C + c``
            is channel ``c`` at output row ``2i + a``, column ``2j + b``.
        gamma: Per-channel scale, shape ``[C]``.

    Returns:
        ``(x, rms_silu(x, gamma))`` with ``x`` of shape ``[B, 2H, 2W, C]``.
    """
    if u.ndim != 4 or u.shape[-1] != 4 * gamma.numel():
        raise ValueError("u must be [B, H, W, 4 * C]")
    _validate(u, gamma, gamma.numel())
    return _shuffle_rms_silu(u, gamma)

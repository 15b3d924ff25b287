"""Trimmed-context gain of the cross attention (``ctx_scale``).

Drop-in for src/kernels/ctx_scale.py: same public function, arguments,
outputs and ValueError (ctx_scale.py:140-147), custom op with fake impl and
autograd (:40-137).  Per token s of batch entry b and head h:
``gain = 1 / (1 + exp(ln_pad[b] - lse[b, h, s]))`` and ``y = bf16(out * gain)``;
the backward returns ``dout = bf16(dy * gain)`` and
``dlse = sum(dy * out) * gain * (1 - gain)`` (fp32, [B, H, S]).
"""

from __future__ import annotations

import torch

from .._lib import call
from .common import _check, _stream

__all__ = ["ctx_scale", "ctx_scale_rowquant"]


@torch.library.custom_op("anima_flat_b200::ctx_scale", mutates_args=())
def _ctx_scale(out: torch.Tensor, lse: torch.Tensor, ln_pad: torch.Tensor) -> torch.Tensor:
    B, S, H, hd = out.shape
    y = torch.empty_like(out)
    call("afb_ctx_scale", out.data_ptr(), lse.data_ptr(), ln_pad.data_ptr(), y.data_ptr(),
         B, S, H, hd, _stream(out))
    return y


@_ctx_scale.register_fake
def _(out, lse, ln_pad):
    return torch.empty_like(out)


@torch.library.custom_op("anima_flat_b200::ctx_scale_bwd", mutates_args=())
def _ctx_scale_bwd_op(
    out: torch.Tensor, lse: torch.Tensor, ln_pad: torch.Tensor, dy: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, H, hd = out.shape
    dy = dy.contiguous()
    dout = torch.empty_like(out)
    dlse = torch.empty_like(lse)
    call("afb_ctx_scale_bwd", out.data_ptr(), lse.data_ptr(), ln_pad.data_ptr(), dy.data_ptr(),
         dout.data_ptr(), dlse.data_ptr(), B, S, H, hd, _stream(out))
    return dout, dlse


@_ctx_scale_bwd_op.register_fake
def _(out, lse, ln_pad, dy):
    return torch.empty_like(out), torch.empty_like(lse)


def _ctx_scale_setup(ctx, inputs, output):
    out, lse, ln_pad = inputs
    ctx.save_for_backward(out, lse, ln_pad)


def _ctx_scale_backward(ctx, dy):
    out, lse, ln_pad = ctx.saved_tensors
    dout, dlse = _ctx_scale_bwd_op(out, lse, ln_pad, dy)
    return dout, dlse, None


torch.library.register_autograd(
    "anima_flat_b200::ctx_scale", _ctx_scale_backward, setup_context=_ctx_scale_setup
)


def ctx_scale(out: torch.Tensor, lse: torch.Tensor, ln_pad: torch.Tensor) -> torch.Tensor:
    """Rescale a trimmed cross-attention output to the full padded context.

    Args:
        out: Attention output over the kept keys, [B, S, H, hd] bf16.
        lse: Its log-sum-exp, [B, H, S] (cast to fp32).
        ln_pad: log of the number of removed padding keys, [B] (cast to fp32).

    Returns:
        ``out * gain``, [B, S, H, hd], dtype of ``out``.
    """
    _check(out, lse, ln_pad)
    if out.ndim != 4 or lse.shape != (out.shape[0], out.shape[2], out.shape[1]):
        raise ValueError("out must be [B, S, H, hd] and lse [B, H, S]")
    if out.dtype != torch.bfloat16:
        raise ValueError(f"out must be torch.bfloat16, got {out.dtype}")
    return _ctx_scale(out.contiguous(), lse.float().contiguous(), ln_pad.float().contiguous())


@torch.library.custom_op("anima_flat_b200::ctx_scale_rowquant", mutates_args=())
def _ctx_scale_rowquant(
    out: torch.Tensor, lse: torch.Tensor, ln_pad: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, H, hd = out.shape
    q = torch.empty(B, S, H * hd, dtype=torch.float8_e4m3fn, device=out.device)
    s = torch.empty(B * S, 1, dtype=torch.float32, device=out.device)
    call("afb_ctx_scale_rowquant", out.data_ptr(), lse.data_ptr(), ln_pad.data_ptr(), q.data_ptr(),
         s.data_ptr(), B, S, H, hd, _stream(out))
    return q, s


@_ctx_scale_rowquant.register_fake
def _(out, lse, ln_pad):
    B, S, H, hd = out.shape
    return (out.new_empty((B, S, H * hd), dtype=torch.float8_e4m3fn),
            out.new_empty((B * S, 1), dtype=torch.float32))


def ctx_scale_rowquant(
    out: torch.Tensor, lse: torch.Tensor, ln_pad: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """``rowquant(ctx_scale(out, lse, ln_pad).flatten(2))`` in one pass.

    The FP8 forward quantises the trimmed cross-attention's output right after
    its gain (src/model.py:457 with src/attention.py:180).  This returns the
    same codes and scales, bit for bit, without writing the bf16 scaled output.
    Inference only (FP8 has no backward), like rowquant.

    Args:
        out: Attention output over the kept keys, [B, S, H, hd] bf16.
        lse: Its log-sum-exp, [B, H, S] (cast to fp32).
        ln_pad: log of the number of removed padding keys, [B] (cast to fp32).

    Returns:
        ``(q, s)``: q [B, S, H*hd] float8_e4m3fn, s [B*S, 1] fp32.
    """
    _check(out, lse, ln_pad)
    if out.ndim != 4 or lse.shape != (out.shape[0], out.shape[2], out.shape[1]):
        raise ValueError("out must be [B, S, H, hd] and lse [B, H, S]")
    if out.dtype != torch.bfloat16:
        raise ValueError(f"out must be torch.bfloat16, got {out.dtype}")
    return _ctx_scale_rowquant(out.contiguous(), lse.float().contiguous(), ln_pad.float().contiguous())

"""q/k RMSNorm fused with 3D RoPE (``qkv_norm_rope``) and ``head_norm``.

Drop-in for src/kernels/rope.py: same public functions, signatures, defaults
(q/k eps 1e-5), outputs and ValueErrors (rope.py:616-652).  In no-grad mode v
is returned as a strided view of ``qkv`` (rope.py:641-645); in grad mode
(``qkv`` or ``q_weight`` requires grad) the ``qkv_norm_rope_v`` op copies it
(rope.py:639-640).

Per token and head (rope.py:39-58): ``rstd = rsqrt(mean(x^2) + eps)``,
``a, b = bf16(x * rstd * w)`` for the two halves, then for q and k
``a' = a*cos - b*sin``, ``b' = b*cos + a*sin`` with fp32 tables
``cos, sin [S, head_dim // 2]`` at ``position = token % S``.
"""

from __future__ import annotations

import torch

from .._lib import call, workspace
from .common import BF16, _check, _check_dtype, _stream

__all__ = ["head_norm", "qkv_norm_rope"]

F32 = torch.float32


def _launch_qkv(qkv, q_weight, k_weight, cos, sin, heads, eps, with_v):
    B, S, _ = qkv.shape
    half = cos.shape[1]
    q = qkv.new_empty((B, S, heads, 2 * half))
    k = torch.empty_like(q)
    v = torch.empty_like(q) if with_v else None
    call(
        "afb_qkv_norm_rope",
        qkv.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(), cos.data_ptr(), sin.data_ptr(),
        q.data_ptr(), k.data_ptr(), v.data_ptr() if v is not None else None,
        B, S, heads, 2 * half, eps, _stream(qkv),
    )
    return q, k, v


@torch.library.custom_op("anima_flat_b200::qkv_norm_rope", mutates_args=())
def _qkv_norm_rope(
    qkv: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    heads: int,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    q, k, _ = _launch_qkv(qkv, q_weight, k_weight, cos, sin, heads, eps, False)
    return q, k


@_qkv_norm_rope.register_fake
def _(qkv, q_weight, k_weight, cos, sin, heads, eps):
    B, S, _ = qkv.shape
    q = qkv.new_empty((B, S, heads, 2 * cos.shape[1]))
    return q, torch.empty_like(q)


@torch.library.custom_op("anima_flat_b200::qkv_norm_rope_v", mutates_args=())
def _qkv_norm_rope_v(
    qkv: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    heads: int,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    q, k, v = _launch_qkv(qkv, q_weight, k_weight, cos, sin, heads, eps, True)
    return q, k, v


@_qkv_norm_rope_v.register_fake
def _(qkv, q_weight, k_weight, cos, sin, heads, eps):
    B, S, _ = qkv.shape
    q = qkv.new_empty((B, S, heads, 2 * cos.shape[1]))
    return q, torch.empty_like(q), torch.empty_like(q)


@torch.library.custom_op("anima_flat_b200::head_norm", mutates_args=())
def _head_norm(x: torch.Tensor, weight: torch.Tensor, heads: int, eps: float) -> torch.Tensor:
    B, S, _ = x.shape
    hd = weight.numel()
    y = x.new_empty((B, S, heads, hd))
    call(
        "afb_head_norm",
        x.data_ptr(), weight.data_ptr(), y.data_ptr(), B, S, heads, hd, eps, _stream(x),
    )
    return y


@_head_norm.register_fake
def _(x, weight, heads, eps):
    return x.new_empty((x.shape[0], x.shape[1], heads, weight.numel()))


# ------------------------------------------------------------------ backward --
# rope.py:443-613.  Weight gradients are reduced over all tokens and heads in a
# fixed order (see csrc/headnorm_bwd.cu).
@torch.library.custom_op("anima_flat_b200::head_norm_bwd", mutates_args=())
def _head_norm_bwd_op(
    x: torch.Tensor, dy: torch.Tensor, weight: torch.Tensor, heads: int, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    B, S, _ = x.shape
    hd = weight.numel()
    dy = dy.contiguous()
    dx = torch.empty_like(x)
    dw = torch.empty(hd, dtype=F32, device=x.device)
    ws, nbytes = workspace("afb_head_norm_bwd", x.device, B, S, heads, hd)
    call(
        "afb_head_norm_bwd",
        x.data_ptr(), dy.data_ptr(), weight.data_ptr(), dx.data_ptr(), dw.data_ptr(),
        B, S, heads, hd, eps, ws.data_ptr(), nbytes, _stream(x),
    )
    return dx, dw.to(weight.dtype)


@_head_norm_bwd_op.register_fake
def _(x, dy, weight, heads, eps):
    return torch.empty_like(x), torch.empty_like(weight)


def _head_norm_setup(ctx, inputs, output):
    x, weight, heads, eps = inputs
    ctx.save_for_backward(x, weight)
    ctx.heads = heads
    ctx.eps = eps


def _head_norm_backward(ctx, dy):
    x, weight = ctx.saved_tensors
    dx, dw = _head_norm_bwd_op(x, dy, weight, ctx.heads, ctx.eps)
    return dx, dw, None, None


torch.library.register_autograd(
    "anima_flat_b200::head_norm", _head_norm_backward, setup_context=_head_norm_setup
)


@torch.library.custom_op("anima_flat_b200::qkv_norm_rope_bwd", mutates_args=())
def _qkv_norm_rope_bwd_op(
    qkv: torch.Tensor,
    dq: torch.Tensor,
    dk: torch.Tensor,
    dv: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    heads: int,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    B, S, _ = qkv.shape
    hd = 2 * cos.shape[1]
    dq, dk, dv = dq.contiguous(), dk.contiguous(), dv.contiguous()
    dqkv = torch.empty_like(qkv)
    dqw = torch.empty(hd, dtype=F32, device=qkv.device)
    dkw = torch.empty(hd, dtype=F32, device=qkv.device)
    ws, nbytes = workspace("afb_qkv_norm_rope_bwd", qkv.device, B, S, heads, hd)
    call(
        "afb_qkv_norm_rope_bwd",
        qkv.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), q_weight.data_ptr(),
        k_weight.data_ptr(), cos.data_ptr(), sin.data_ptr(), dqkv.data_ptr(), dqw.data_ptr(),
        dkw.data_ptr(), B, S, heads, hd, eps, ws.data_ptr(), nbytes, _stream(qkv),
    )
    return dqkv, dqw.to(q_weight.dtype), dkw.to(k_weight.dtype)


@_qkv_norm_rope_bwd_op.register_fake
def _(qkv, dq, dk, dv, q_weight, k_weight, cos, sin, heads, eps):
    return torch.empty_like(qkv), torch.empty_like(q_weight), torch.empty_like(k_weight)


def _qkv_norm_rope_setup(ctx, inputs, output):
    qkv, q_weight, k_weight, cos, sin, heads, eps = inputs
    ctx.save_for_backward(qkv, q_weight, k_weight, cos, sin)
    ctx.heads = heads
    ctx.eps = eps


def _qkv_norm_rope_backward(ctx, dq, dk, dv):
    qkv, q_weight, k_weight, cos, sin = ctx.saved_tensors
    dqkv, dqw, dkw = _qkv_norm_rope_bwd_op(
        qkv, dq, dk, dv, q_weight, k_weight, cos, sin, ctx.heads, ctx.eps
    )
    return dqkv, dqw, dkw, None, None, None, None


torch.library.register_autograd(
    "anima_flat_b200::qkv_norm_rope_v", _qkv_norm_rope_backward, setup_context=_qkv_norm_rope_setup
)


def _f32(w: torch.Tensor) -> torch.Tensor:
    """fp32 contiguous copy of a norm weight or table (the kernels read fp32)."""
    return w.to(F32).contiguous()


def qkv_norm_rope(qkv, q_weight, k_weight, cos, sin, heads, eps=1e-5):
    """RMS-normalise q and k per head and apply rotary embeddings; split off v.

    Args:
        qkv: Fused projection output, contiguous ``[B, S, 3 * heads * head_dim]`` bf16.
        q_weight: q RMSNorm weight ``[head_dim]``.
        k_weight: k RMSNorm weight ``[head_dim]``.
        cos: Rotary cosines ``[S, head_dim // 2]`` (power-of-two width).
        sin: Rotary sines, same shape.
        heads: Number of heads.
        eps: RMSNorm epsilon.

    Returns:
        ``(q, k, v)``, each ``[B, S, heads, head_dim]``; v is a view of ``qkv``
        unless autograd needs it.

    Raises:
        ValueError: On non-CUDA tensors or inconsistent shapes (rope.py:618-629).
    """
    _check(qkv, q_weight, k_weight, cos, sin)
    if (
        not qkv.is_contiguous()
        or qkv.ndim != 3
        or qkv.shape[-1] != 3 * heads * 2 * cos.shape[1]
    ):
        raise ValueError("qkv must be contiguous [B, S, 3 * heads * head_dim]")
    if (
        cos.shape != sin.shape
        or cos.shape[0] != qkv.shape[1]
        or (cos.shape[1] & (cos.shape[1] - 1))
    ):
        raise ValueError("cos/sin must be [S, head_dim // 2] with a power-of-two width")
    _check_dtype(BF16, "qkv", qkv)
    args = (qkv, _f32(q_weight), _f32(k_weight), _f32(cos), _f32(sin), heads, eps)
    if torch.is_grad_enabled() and (qkv.requires_grad or q_weight.requires_grad):
        return _qkv_norm_rope_v(*args)
    q, k = _qkv_norm_rope(*args)
    B, S, _ = qkv.shape
    v = qkv.view(B, S, 3, heads, 2 * cos.shape[1])[:, :, 2]
    return q, k, v


def head_norm(x, weight, heads, eps=1e-5):
    """RMS-normalise each head of ``x`` (the cross-attention queries).

    Args:
        x: Contiguous ``[B, S, heads * head_dim]`` bf16.
        weight: RMSNorm weight ``[head_dim]``.
        heads: Number of heads.
        eps: RMSNorm epsilon.

    Returns:
        ``[B, S, heads, head_dim]``.

    Raises:
        ValueError: On non-CUDA tensors or a shape mismatch (rope.py:649-651).
    """
    _check(x, weight)
    if not x.is_contiguous() or x.shape[-1] != heads * weight.numel():
        raise ValueError("x must be contiguous [B, S, heads * head_dim]")
    _check_dtype(BF16, "x", x)
    return _head_norm(x, _f32(weight), heads, eps)

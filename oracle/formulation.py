"""The reference's unfused PyTorch-eager fp32 composition — TEST/BASELINE ONLY.

This is the CPU baseline the task names (F.layer_norm, elementwise
mul/add, per-head RMSNorm, rotate-half RoPE, amax/divide/clamp/cast), written
with torch ops in fp32 and rounded to bf16 at the reference's rounding points
(src/kernels/adaln.py:33-46, fp8.py:80-97 and :260-292, rope.py:39-58).  It
runs on any device; tests use it as the tolerance reference for the kernels
(bf16 outputs within 2 bf16 ulp), bench.py times it on the host cores.
Reduction order is torch's own, so it is not a bit-exact target.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16
FP8 = torch.float8_e4m3fn


def _rows(v: torch.Tensor, B: int, D: int) -> torch.Tensor:
    return v.float().reshape(B, 1, D)


def residual_z(x, res, gate):
    """z = bf16(res + bf16(gate * x))  (adaln.py:33-36)."""
    B, _, D = res.shape
    p = (_rows(gate, B, D) * x.float()).to(BF16).float()
    return (res.float() + p).to(BF16)


def adaln_y(z, shift, scale, eps):
    """fp32 y = LN(z) * scale + shift  (adaln.py:40-46, fp8.py:87-93)."""
    B, _, D = z.shape
    return F.layer_norm(z.float(), (D,), eps=eps) * _rows(scale, B, D) + _rows(shift, B, D)


def residual_adaln(x, res, gate, shift, scale, eps=1e-6):
    z = residual_z(x, res, gate)
    return adaln_y(z, shift, scale, eps).to(BF16), z


def adaln(z, shift, scale, eps=1e-6):
    return adaln_y(z, shift, scale, eps).to(BF16)


def quantize_rows(y: torch.Tensor):
    """s = max(amax, 1e-12) / 448; q = e4m3(clamp(y / s))  (fp8.py:94-97)."""
    lead = y.shape[:-1]
    y2 = y.float().reshape(-1, y.shape[-1])
    s = y2.abs().amax(dim=1, keepdim=True).clamp_min(1e-12) / 448.0
    q = (y2 / s).clamp(-448.0, 448.0).to(FP8)
    return q.reshape(*lead, y.shape[-1]), s


def residual_adaln_fp8(x, res, gate, shift, scale, eps=1e-6):
    z = residual_z(x, res, gate)
    q, s = quantize_rows(adaln_y(z, shift, scale, eps))
    return q, s, z


def adaln_fp8(z, shift, scale, eps=1e-6):
    return quantize_rows(adaln_y(z, shift, scale, eps))


def gelu_as(x: torch.Tensor) -> torch.Tensor:
    """A&S 7.1.26 GELU in fp32 (fp8.py:260-270)."""
    x = x.float()
    z = x * 0.7071067811865476
    az = z.abs()
    t = 1.0 / (1.0 + 0.3275911 * az)
    poly = ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t
            + 0.254829592) * t
    y = 1.0 - poly * torch.exp(-az * az)
    return 0.5 * x * (1.0 + torch.where(z < 0, -y, y))


def rowquant(x, gelu=False):
    y = gelu_as(x) if gelu else x.float()
    return quantize_rows(y)


def _rms_heads(t: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16(x * rsqrt(mean(x^2) + eps) * w) per head  (rope.py:41-48)."""
    tf = t.float()
    rstd = torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps)
    return (tf * rstd * w.float()).to(BF16)


def rotate(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on bf16 heads [B,S,H,hd] with fp32 [S, hd/2] tables (rope.py:49-56)."""
    half = t.shape[-1] // 2
    a, b = t.float()[..., :half], t.float()[..., half:]
    c = cos.float()[None, :, None, :]
    s = sin.float()[None, :, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).to(BF16)


def qkv_norm_rope(qkv, q_weight, k_weight, cos, sin, heads, eps=1e-5):
    B, S, W = qkv.shape
    hd = W // (3 * heads)
    q, k, v = qkv.view(B, S, 3, heads, hd).unbind(2)
    q = rotate(_rms_heads(q, q_weight, eps), cos, sin)
    k = rotate(_rms_heads(k, k_weight, eps), cos, sin)
    return q, k, v.contiguous()


def head_norm(x, weight, heads, eps=1e-5):
    B, S, W = x.shape
    return _rms_heads(x.view(B, S, heads, W // heads), weight, eps)

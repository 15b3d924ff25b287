"""Rotary tables for the DiT token grid (the input producer of ``qkv_norm_rope``).

Restates src/model.py:51-84 (``rope_tables``): the head's half-dims are split
time:height:width = (hd - 2*dh)/2 : dh/2 : dh/2 with ``dh = hd // 6 * 2``
(22:21:21 for hd = 128); time angles are zero for a single image; the height
and width frequencies are ``1 / (10000 * rope_scale**(dh / (dh - 2)))**(2i / dh)``.
Cosmos-Predict2-2B uses rope_scale (4, 4) (src/config.py:30).
"""

from __future__ import annotations

import torch


def rope_tables(
    h: int,
    w: int,
    head_dim: int,
    device: str | torch.device = "cpu",
    rope_scale: tuple = (1.0, 1.0),
) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``(cos, sin)`` of shape ``[h * w, head_dim // 2]`` for an ``h x w`` grid."""
    dh = head_dim // 6 * 2
    dt = head_dim - 2 * dh
    exponent = dh / (dh - 2)
    steps = torch.arange(0, dh, 2, device=device, dtype=torch.float32) / dh
    freq_h = 1.0 / ((10000.0 * rope_scale[0] ** exponent) ** steps)
    freq_w = 1.0 / ((10000.0 * rope_scale[1] ** exponent) ** steps)
    rows = torch.arange(h, device=device, dtype=torch.float32)
    cols = torch.arange(w, device=device, dtype=torch.float32)
    ang_h = (rows[:, None] * freq_h[None, :])[:, None, :].expand(h, w, dh // 2)
    ang_w = (cols[:, None] * freq_w[None, :])[None, :, :].expand(h, w, dh // 2)
    ang_t = torch.zeros(h, w, dt // 2, device=device)
    ang = torch.cat([ang_t, ang_h, ang_w], dim=-1).reshape(h * w, head_dim // 2)
    return ang.cos(), ang.sin()

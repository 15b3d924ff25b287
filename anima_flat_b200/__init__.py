"""anima_flat_b200 — the fused DiT layer ops of anima-flat, hand-written for B200 (sm_100a).

Public functions mirror src/kernels/{adaln,fp8,rope,ctx_scale,rms}.py of the reference:

    adaln, residual_adaln                         (AdaLN modulate, gated residual)
    adaln_fp8, residual_adaln_fp8, rowquant       (per-row FP8 e4m3 quantisation)
    qkv_norm_rope, head_norm                      (q/k RMSNorm + 3D RoPE)
    ctx_scale                                     (trimmed cross-attention gain)
    ctx_scale_rowquant                            (the gain and FP8 quantisation in one pass)
    rms_silu, add_rms_silu, shuffle_rms_silu      (VAE channel RMS norm + SiLU)

All run through the C-ABI library ``lib/libanima_flat_b200.so`` (see
``include/anima_flat_b200.h``); there is no CPU fallback.
"""

from .kernels.adaln import adaln, residual_adaln
from .kernels.ctx_scale import ctx_scale, ctx_scale_rowquant
from .kernels.fp8 import FP8, FP8_MAX, adaln_fp8, residual_adaln_fp8, rowquant
from .kernels.rms import add_rms_silu, rms_silu, shuffle_rms_silu
from .kernels.rope import head_norm, qkv_norm_rope
from .tables import rope_tables

__all__ = [
    "FP8",
    "FP8_MAX",
    "adaln",
    "add_rms_silu",
    "adaln_fp8",
    "ctx_scale",
    "ctx_scale_rowquant",
    "head_norm",
    "qkv_norm_rope",
    "residual_adaln",
    "residual_adaln_fp8",
    "rms_silu",
    "rope_tables",
    "rowquant",
    "shuffle_rms_silu",
]

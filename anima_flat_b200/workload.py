"""The fused-op call sequence of one denoiser forward, and its byte model.

Mirrors the order in which the reference's ``AnimaFlat.forward_fused``
(src/model.py:339-376, per block ``_fused_block`` :297-337) and
``forward_fp8`` (:403-473) call the hot-path ops, so that a benchmark step
launches exactly the ops, shapes and counts of one forward pass.  GEMMs and
attention between the ops are not part of the path; their outputs are
stand-in input buffers.

Algorithmic bytes count every activation read and written once per call plus
the per-call parameter vectors and tables (the §(d) byte model): they are the
numerator of the reported HBM GB/s.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shape:
    batch: int = 1
    seq: int = 4096
    dim: int = 2048
    heads: int = 16
    head_dim: int = 128
    layers: int = 28
    mlp: int = 8192

    @property
    def rows(self) -> int:
        return self.batch * self.seq


def bytes_residual_adaln(s: Shape) -> int:
    return s.rows * s.dim * 2 * 4 + 3 * s.batch * s.dim * 2


def bytes_adaln(s: Shape) -> int:
    return s.rows * s.dim * 2 * 2 + 2 * s.batch * s.dim * 2


def bytes_qkv_norm_rope(s: Shape, with_v: bool = False) -> int:
    w = s.heads * s.head_dim
    per_row = (2 * w + 2 * w) * 2 + (2 * w * 2 if with_v else 0)
    tables = 2 * s.seq * (s.head_dim // 2) * 4
    return s.rows * per_row + tables + 2 * s.head_dim * 4


def bytes_head_norm(s: Shape) -> int:
    return s.rows * s.heads * s.head_dim * 2 * 2 + s.head_dim * 4


def bytes_residual_adaln_fp8(s: Shape) -> int:
    return s.rows * (s.dim * 2 * 3 + s.dim + 4) + 3 * s.batch * s.dim * 2


def bytes_adaln_fp8(s: Shape) -> int:
    return s.rows * (s.dim * 2 + s.dim + 4) + 2 * s.batch * s.dim * 2


def bytes_rowquant(s: Shape, K: int) -> int:
    return s.rows * (K * 2 + K + 4)


def bytes_residual_adaln_bwd(s: Shape) -> int:
    # read gh, gz, z, x; write dres, dx; gate/scale in, dgate/dshift/dscale out
    return s.rows * s.dim * 2 * 6 + 5 * s.batch * s.dim * 2


def bytes_adaln_bwd(s: Shape) -> int:
    # read gh, z; write dz; scale in, dshift/dscale out
    return s.rows * s.dim * 2 * 3 + 3 * s.batch * s.dim * 2


def bytes_qkv_norm_rope_bwd(s: Shape) -> int:
    w = s.heads * s.head_dim
    # read the q/k sections of qkv and dq, dk, dv; write dqkv (all three sections)
    tables = 2 * s.seq * (s.head_dim // 2) * 4
    return s.rows * (2 * w + 3 * w + 3 * w) * 2 + tables + 4 * s.head_dim * 4


def bytes_head_norm_bwd(s: Shape) -> int:
    w = s.heads * s.head_dim
    return s.rows * 3 * w * 2 + 2 * s.head_dim * 4


def bytes_ctx_scale(s: Shape) -> int:
    # out read, y written; lse [B, H, S] fp32 read; ln_pad [B]
    return s.rows * s.heads * s.head_dim * 2 * 2 + s.rows * s.heads * 4 + s.batch * 4


def bytes_ctx_scale_rowquant(s: Shape) -> int:
    # out read; q (1 B per element) and s [rows] fp32 written; lse, ln_pad read
    return s.rows * s.heads * s.head_dim * (2 + 1) + s.rows * 4 + s.rows * s.heads * 4 + s.batch * 4


def bytes_ctx_scale_bwd(s: Shape) -> int:
    # out, dy read, dout written; lse read, dlse written; ln_pad
    return s.rows * s.heads * s.head_dim * 2 * 3 + s.rows * s.heads * 4 * 2 + s.batch * 4


# The VAE decoder's last stage at 1024x1024: 1M pixels of 96 channels.
VAE_ROWS = 1024 * 1024
VAE_C = 96


def bytes_rms(name: str, rows: int = VAE_ROWS, C: int = VAE_C) -> int:
    """Algorithmic bytes of the rms_silu family: bf16 activations read and
    written once, plus gamma (and gamma's gradient)."""
    t = rows * C * 2
    return {
        "rms_silu": 2 * t + C * 4,                 # x in, y out
        "add_rms_silu": 4 * t + C * 4,             # x, r in; s, y out
        "shuffle_rms_silu": 3 * t + C * 4,         # u in; s, y out
        "rms_silu_bwd": 4 * t + 2 * C * 4,         # s, dy, gs in; ds out; gamma in, dgamma out
    }[name]


def bf16_forward_calls(s: Shape) -> list[str]:
    """Op names in call order for forward_fused (model.py:366-375)."""
    calls = ["adaln"]
    for layer in range(s.layers):
        calls += ["qkv_norm_rope", "residual_adaln", "head_norm", "residual_adaln"]
        if layer + 1 < s.layers:
            calls.append("residual_adaln")
    calls.append("residual_adaln")  # final layer (model.py:375)
    return calls


def fp8_forward_calls(s: Shape) -> list[str]:
    """Op names in call order for forward_fp8 (model.py:434-472)."""
    calls = ["adaln_fp8"]
    for layer in range(s.layers):
        calls += ["qkv_norm_rope", "rowquant", "residual_adaln_fp8", "head_norm", "rowquant",
                  "residual_adaln_fp8", "rowquant_gelu"]
        if layer + 1 < s.layers:
            calls.append("residual_adaln_fp8")
    calls.append("residual_adaln")
    return calls


def call_bytes(name: str, s: Shape) -> int:
    return {
        "adaln": bytes_adaln,
        "residual_adaln": bytes_residual_adaln,
        "qkv_norm_rope": bytes_qkv_norm_rope,
        "head_norm": bytes_head_norm,
        "adaln_fp8": bytes_adaln_fp8,
        "residual_adaln_fp8": bytes_residual_adaln_fp8,
        "rowquant": lambda sh: bytes_rowquant(sh, sh.dim),
        "rowquant_gelu": lambda sh: bytes_rowquant(sh, sh.mlp),
        "residual_adaln_bwd": bytes_residual_adaln_bwd,
        "adaln_bwd": bytes_adaln_bwd,
        "qkv_norm_rope_bwd": bytes_qkv_norm_rope_bwd,
        "head_norm_bwd": bytes_head_norm_bwd,
        "ctx_scale": bytes_ctx_scale,
        "ctx_scale_bwd": bytes_ctx_scale_bwd,
        "ctx_scale_rowquant": bytes_ctx_scale_rowquant,
        "rms_silu": lambda sh: bytes_rms("rms_silu"),
        "add_rms_silu": lambda sh: bytes_rms("add_rms_silu"),
        "shuffle_rms_silu": lambda sh: bytes_rms("shuffle_rms_silu"),
        "rms_silu_bwd": lambda sh: bytes_rms("rms_silu_bwd"),
    }[name](s)


def step_bytes(calls: list[str], s: Shape) -> int:
    return sum(call_bytes(c, s) for c in calls)

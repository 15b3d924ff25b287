"""Generate golden vectors by running the reference's own Triton kernels.

    python tests/golden/gen_golden.py --reference PATH

Imports tan0210/anima-flat's src/kernels from the checkout at PATH (read
only) with TRITON_INTERPRET=1, launches each hot-path kernel through its
JITFunction (``kernel.fn[grid](...)``, bypassing the GPU-only autotuner) on
small seeded CPU inputs, and writes the inputs and outputs to
tests/golden/<case>.npz.  bf16 tensors are stored as uint16 bit patterns,
e4m3 as uint8.  The interpreter truncates fp32->bf16 casts and evaluates
tl.sum with numpy; the oracle's INTERP mode reproduces both, and the tests
compare it with these files.  Only this script reads the reference; the
fixtures are what the tests use.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def bits(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy().copy()
    return t.contiguous().numpy().copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of tan0210/anima-flat (read only)")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)
    import torch
    import triton
    from src.kernels import adaln as A
    from src.kernels import ctx_scale as CS
    from src.kernels import rms as RM
    from src.kernels import fp8 as F8
    from src.kernels import rope as R
    from src.model import rope_tables

    bf = torch.bfloat16
    gen = torch.Generator().manual_seed(20261201)

    def randn(*shape, std=1.0, outliers=0.0):
        t = torch.randn(*shape, generator=gen) * std
        if outliers:
            m = torch.rand(*shape, generator=gen) < outliers
            t = torch.where(m, t * 20.0, t)
        return t

    def mods(B, D):
        shift = randn(B, D, std=0.1).to(bf)
        scale = (1.0 + randn(B, D, std=0.1)).to(bf)
        gate = randn(B, D, std=0.1).to(bf)
        return shift, scale, gate

    def save(name, **arrays):
        np.savez_compressed(OUT / f"{name}.npz", **{k: bits(v) if isinstance(v, torch.Tensor) else v
                                                     for k, v in arrays.items()})
        print("wrote", name, {k: getattr(v, "shape", v) for k, v in arrays.items()})

    # --- AdaLN / residual AdaLN (adaln.py:10-46) -------------------------------------
    for name, (B, S, D, has_x, outl) in {
        "residual_adaln_d2048": (2, 3, 2048, True, 0.0),
        "adaln_d2048": (2, 3, 2048, False, 0.0),
        "residual_adaln_d256": (1, 5, 256, True, 0.01),
    }.items():
        x = randn(B, S, D, outliers=outl).to(bf)
        res = randn(B, S, D, outliers=outl).to(bf)
        shift, scale, gate = mods(B, D)
        h = torch.empty_like(res)
        z = torch.empty_like(res)
        if has_x:
            A._residual_adaln_kernel.fn[(B * S,)](x, res, gate, shift, scale, h, z, S, 1e-6,
                                                  D=D, BLOCK=triton.next_power_of_2(D), HAS_X=True)
            save(name, x=x, res=res, gate=gate, shift=shift, scale=scale, h=h, z=z,
                 eps=np.float32(1e-6))
        else:
            A._residual_adaln_kernel.fn[(B * S,)](res, res, shift, shift, scale, h, h, S, 1e-6,
                                                  D=D, BLOCK=triton.next_power_of_2(D), HAS_X=False)
            save(name, res=res, shift=shift, scale=scale, h=h, eps=np.float32(1e-6))

    # --- FP8 AdaLN (fp8.py:56-97) -----------------------------------------------------
    for name, has_x in {"residual_adaln_fp8_d2048": True, "adaln_fp8_d2048": False}.items():
        B, S, D = 2, 3, 2048
        x = randn(B, S, D, outliers=0.01).to(bf)
        res = randn(B, S, D, outliers=0.01).to(bf)
        shift, scale, gate = mods(B, D)
        q = torch.empty(B, S, D, dtype=torch.float8_e4m3fn)
        s = torch.empty(B * S, 1, dtype=torch.float32)
        z = torch.empty_like(res)
        if has_x:
            F8._residual_adaln_fp8_kernel.fn[(B * S,)](x, res, gate, shift, scale, q, s, z, S, 1e-6,
                                                       D=D, BLOCK=D, HAS_X=True)
            save(name, x=x, res=res, gate=gate, shift=shift, scale=scale, q=q, s=s, z=z,
                 eps=np.float32(1e-6))
        else:
            F8._residual_adaln_fp8_kernel.fn[(B * S,)](res, res, shift, shift, scale, q, s, res, S,
                                                       1e-6, D=D, BLOCK=D, HAS_X=False)
            save(name, res=res, shift=shift, scale=scale, q=q, s=s, eps=np.float32(1e-6))

    # --- rowquant (fp8.py:273-292) ----------------------------------------------------
    for name, (rows, K, gelu) in {
        "rowquant_k2048": (6, 2048, False),
        "rowquant_k8192": (4, 8192, False),
        "rowquant_gelu_k8192": (4, 8192, True),
        "rowquant_gelu_k2048": (6, 2048, True),
    }.items():
        x = randn(1, rows, K, outliers=0.01).to(bf)
        q = torch.empty(1, rows, K, dtype=torch.float8_e4m3fn)
        s = torch.empty(rows, 1, dtype=torch.float32)
        F8._rowquant_kernel.fn[(rows,)](x, q, s, K=K, BLOCK=K, GELU=gelu)
        save(name, x=x, q=q, s=s, gelu=np.bool_(gelu))

    # --- q/k RMSNorm + RoPE and head norm (rope.py:12-172) ----------------------------
    for name, (B, hh, ww, H, hd, eps) in {
        "qkv_norm_rope_h4": (2, 4, 4, 4, 128, 1e-5),
        "qkv_norm_rope_eps1e6": (1, 2, 3, 2, 128, 1e-6),
    }.items():
        S = hh * ww
        cos, sin = rope_tables(hh, ww, hd, "cpu", (4.0, 4.0))
        qkv = randn(B, S, 3 * H * hd).to(bf)
        qw = 1.0 + randn(hd, std=0.02)
        kw = 1.0 + randn(hd, std=0.02)
        q = torch.empty(B, S, H, hd, dtype=bf)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        hpp = 2
        R._qkv_norm_rope_kernel.fn[(B * S, 3 * triton.cdiv(H, hpp))](
            qkv, q, k, v, qw, kw, cos, sin, S, eps, HEADS=H, HALF=hd // 2, HPP=hpp)
        save(name, qkv=qkv, qw=qw, kw=kw, cos=cos, sin=sin, q=q, k=k, v=v, heads=np.int64(H),
             eps=np.float32(eps))

    # --- backward (adaln.py:111-217, rope.py:277-577), partials summed as the
    # reference's wrappers do ------------------------------------------------------
    for name, (B, S, D, has_x, has_gz) in {
        "residual_adaln_bwd_d2048": (2, 11, 2048, True, True),
        "residual_adaln_bwd_nogz_d256": (1, 20, 256, True, False),
        "adaln_bwd_d2048": (2, 9, 2048, False, False),
    }.items():
        rows = 8
        nchunks = triton.cdiv(S, rows)
        z = randn(B, S, D).to(bf)
        x = randn(B, S, D).to(bf)
        gh = randn(B, S, D, std=1e-2).to(bf)
        gz = randn(B, S, D, std=1e-2).to(bf)
        shift, scale, gate = mods(B, D)
        dz = torch.empty_like(z)
        dx = torch.empty_like(z)
        part = lambda: torch.empty(B, nchunks, D, dtype=torch.float32)
        psh, psc, pg = part(), part(), part()
        A._residual_adaln_bwd_kernel.fn[(B, nchunks)](
            gh, gz if has_gz else gh, z, x if has_x else z, gate if has_x else scale, scale, dz,
            dx if has_x else dz, psh, psc, pg if has_x else psh, S, 1e-6, D=D,
            BLOCK=triton.next_power_of_2(D), ROWS=rows, HAS_X=has_x, HAS_GZ=has_gz)
        out = dict(gh=gh, z=z, scale=scale, dz=dz, dshift=psh.sum(1).to(bf), dscale=psc.sum(1).to(bf),
                   eps=np.float32(1e-6))
        if has_x:
            out.update(x=x, gate=gate, dx=dx, dgate=pg.sum(1).to(bf))
        if has_gz:
            out.update(gz=gz)
        save(name, **out)

    B, hh, ww, H, hd, rows = 2, 3, 4, 5, 128, 8
    S = hh * ww
    cos, sin = rope_tables(hh, ww, hd, "cpu", (4.0, 4.0))
    qkv = randn(B, S, 3 * H * hd).to(bf)
    dq, dk, dv = (randn(B, S, H, hd, std=1e-2).to(bf) for _ in range(3))
    qw = 1.0 + randn(hd, std=0.02)
    kw = 1.0 + randn(hd, std=0.02)
    hpp = min(4, triton.next_power_of_2(H))
    gq = triton.cdiv(H, hpp)
    chunks = B * triton.cdiv(S, rows)
    dqkv = torch.empty_like(qkv)
    pw = torch.empty(chunks, 3 * gq, hd, dtype=torch.float32)
    R._qkv_norm_rope_bwd_kernel.fn[(chunks, 3 * gq)](
        qkv, dq, dk, dv, dqkv, qw, kw, cos, sin, pw, S, 1e-5, HEADS=H, HALF=hd // 2, HPP=hpp,
        ROWS=rows)
    save("qkv_norm_rope_bwd_h5", qkv=qkv, dq=dq, dk=dk, dv=dv, qw=qw, kw=kw, cos=cos, sin=sin,
         dqkv=dqkv, dqw=pw[:, :gq].sum((0, 1)), dkw=pw[:, gq:2 * gq].sum((0, 1)),
         heads=np.int64(H), eps=np.float32(1e-5))

    x = randn(B, S, H * hd).to(bf)
    dy = randn(B, S, H, hd, std=1e-2).to(bf)
    w = 1.0 + randn(hd, std=0.02)
    groups = triton.cdiv(H, hpp)
    dx = torch.empty_like(x)
    pw = torch.empty(chunks, groups, hd, dtype=torch.float32)
    R._head_norm_bwd_kernel.fn[(chunks, groups)](x, dy, dx, w, pw, S, 1e-5, HEADS=H,
                                                 HALF=hd // 2, HPP=hpp, ROWS=rows)
    save("head_norm_bwd_h5", x=x, dy=dy, w=w, dx=dx, dw=pw.sum((0, 1)), heads=np.int64(H),
         eps=np.float32(1e-5))

    B, S, H, hd = 2, 5, 4, 128
    x = randn(B, S, H * hd).to(bf)
    w = 1.0 + randn(hd, std=0.02)
    y = torch.empty(B, S, H, hd, dtype=bf)
    R._head_norm_kernel.fn[(B * S, triton.cdiv(H, 2))](x, y, w, 1e-5, HEADS=H, HALF=hd // 2, HPP=2)
    save("head_norm_h4", x=x, w=w, y=y, heads=np.int64(H), eps=np.float32(1e-5))

    # ctx_scale forward and backward (src/kernels/ctx_scale.py:8-37, :61-100).
    # lse spreads over saturated gains on both sides.
    for (B, S, H, hd) in ((2, 5, 4, 128), (1, 3, 5, 64)):
        out = randn(B, S, H, hd).to(bf)
        lse = randn(B, H, S, std=4.0) + 2.0
        ln_pad = torch.tensor([0.5, 4.0][:B], dtype=torch.float32)
        dy = randn(B, S, H, hd, std=1e-2).to(bf)
        block = triton.next_power_of_2(H)
        y = torch.empty_like(out)
        CS._ctx_scale_kernel[(B * S,)](out, lse, ln_pad, y, S, HEADS=H, HD=hd, BLOCK_H=block)
        dout = torch.empty_like(out)
        dlse = torch.empty_like(lse)
        CS._ctx_scale_bwd_kernel[(B * S,)](out, lse, ln_pad, dy, dout, dlse, S, HEADS=H, HD=hd,
                                              BLOCK_H=block)
        save(f"ctx_scale_h{H}_d{hd}", out=out, lse=lse, ln_pad=ln_pad, dy=dy, y=y, dout=dout, dlse=dlse)

    # VAE rms_silu family (src/kernels/rms.py:35-125), launched through the
    # autotuner's JITFunction with a fixed tile: R = 1 row per step, ROWS = 8
    # rows per backward chunk.
    for name, (shape, C, add, shuf) in {
        "rms_silu_c96": ((1, 4, 6, 96), 96, False, False),
        "add_rms_silu_c192": ((2, 3, 5, 192), 192, True, False),
        "shuffle_rms_silu_c96": ((1, 2, 3, 384), 96, False, True),
    }.items():
        x = randn(*shape).to(bf)
        r = randn(*shape).to(bf) if add else None
        g = 1.0 + randn(C, std=0.1)
        if shuf:
            B, h, w, _ = shape
            oshape, H, W = (B, 2 * h, 2 * w, C), 2 * h, 2 * w
        else:
            oshape, H, W = shape, 0, 0
        N = int(np.prod(oshape[:-1]))
        y = torch.empty(oshape, dtype=bf)
        s = torch.empty(oshape, dtype=bf) if (add or shuf) else x
        RM._fwd_kernel.fn[(N,)](x, r if r is not None else x, g, s, y, N, H, W, C=C,
                                BLOCK=triton.next_power_of_2(C), HAS_R=add, SHUF=shuf, R=1)
        dy = randn(*oshape, std=1e-2).to(bf)
        gs = randn(*oshape, std=1e-2).to(bf) if (add or shuf) else None
        rows = 8
        chunks = triton.cdiv(N, rows)
        ds = torch.empty(x.shape, dtype=bf)
        pg = torch.empty(chunks, C, dtype=torch.float32)
        RM._bwd_kernel.fn[(chunks,)](s, g, dy, gs if gs is not None else dy, ds, pg, N, H, W, C=C,
                                     BLOCK=triton.next_power_of_2(C), ROWS=rows, HAS_GS=gs is not None,
                                     SHUF=shuf, R=1)
        arrays = dict(x=x, g=g, y=y, dy=dy, ds=ds, dg=pg.sum(0))
        if r is not None:
            arrays["r"] = r
        if add or shuf:
            arrays["s"] = s
            arrays["gs"] = gs
        save(name, **arrays)

    # Config-scale rows: 64 rows at the model's D = 2048 (and 64 tokens of the
    # model's 16 x 128 heads), so the pin covers more than a handful of rows.
    # A generator of its own keeps every fixture above unchanged.
    gen.manual_seed(20261202)
    B, S, D = 1, 64, 2048
    x = randn(B, S, D, outliers=0.01).to(bf)
    res = randn(B, S, D, outliers=0.01).to(bf)
    shift, scale, gate = mods(B, D)
    h = torch.empty_like(res)
    z = torch.empty_like(res)
    A._residual_adaln_kernel.fn[(B * S,)](x, res, gate, shift, scale, h, z, S, 1e-6,
                                          D=D, BLOCK=triton.next_power_of_2(D), HAS_X=True)
    save("residual_adaln_d2048_r64", x=x, res=res, gate=gate, shift=shift, scale=scale, h=h, z=z,
         eps=np.float32(1e-6))
    q = torch.empty(B, S, D, dtype=torch.float8_e4m3fn)
    s8 = torch.empty(B * S, 1, dtype=torch.float32)
    z8 = torch.empty_like(res)
    F8._residual_adaln_fp8_kernel.fn[(B * S,)](x, res, gate, shift, scale, q, s8, z8, S, 1e-6,
                                               D=D, BLOCK=D, HAS_X=True)
    save("residual_adaln_fp8_d2048_r64", x=x, res=res, gate=gate, shift=shift, scale=scale, q=q,
         s=s8, z=z8, eps=np.float32(1e-6))
    hh, ww, H, hd = 8, 8, 16, 128
    cos, sin = rope_tables(hh, ww, hd, "cpu", (4.0, 4.0))
    qkv = randn(1, hh * ww, 3 * H * hd).to(bf)
    qw = 1.0 + randn(hd, std=0.02)
    kw = 1.0 + randn(hd, std=0.02)
    qo = torch.empty(1, hh * ww, H, hd, dtype=bf)
    ko = torch.empty_like(qo)
    vo = torch.empty_like(qo)
    R._qkv_norm_rope_kernel.fn[(hh * ww, 3 * triton.cdiv(H, 2))](
        qkv, qo, ko, vo, qw, kw, cos, sin, hh * ww, 1e-5, HEADS=H, HALF=hd // 2, HPP=2)
    save("qkv_norm_rope_s64_h16", qkv=qkv, qw=qw, kw=kw, cos=cos, sin=sin, q=qo, k=ko, v=vo,
         heads=np.int64(H), eps=np.float32(1e-5))


if __name__ == "__main__":
    main()

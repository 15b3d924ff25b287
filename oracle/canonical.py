"""numpy front end of oracle.c (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Arrays: bf16 tensors are passed as uint16 bit patterns, e4m3 as uint8.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p

import numpy as np

from .build import build

RNE = 0
INTERP = 1

_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(build()))
        P, I, F, N = c_void_p, c_int64, c_float, c_int
        sigs = {
            "orc_adaln_fwd": ([P] * 9 + [I, I, I, F, N, N, N], None),
            "orc_rowquant": ([P, P, P, P, I, I, N, N], None),
            "orc_qkv_norm_rope": ([P] * 8 + [I, I, I, I, F, N], None),
            "orc_head_norm": ([P, P, P, I, I, I, I, F, N], None),
            "orc_gelu_many": ([P, P, I], None),
            "orc_canonical_sum": ([P, I, N], c_float),
            "orc_numpy_sum": ([P, I], c_float),
            "orc_f32_to_e4m3": ([c_float, N], ctypes.c_uint8),
            "orc_adaln_bwd": ([P] * 11 + [I, I, I, F, N, N, N], None),
            "orc_headnorm_bwd": ([P, I, I, I, I] + [P] * 10 + [I, I, I, I, F, N, N, N, N, N], None),
            "orc_e4m3_to_f32": ([ctypes.c_uint8], c_float),
            "orc_exp": ([c_float], c_float),
            "orc_ctx_scale": ([P] * 7 + [I, I, I, I, N], None),
            "orc_rms_lpr": ([I], N),
            "orc_rms_silu_fwd": ([P] * 5 + [I, I, I, I, N, N], None),
            "orc_rms_silu_bwd": ([P] * 6 + [I, I, I, I, N, N], None),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data_as(c_void_p)


def u16(a) -> np.ndarray:
    """Contiguous uint16 view/copy of a bf16 bit-pattern array."""
    return np.ascontiguousarray(a, dtype=np.uint16)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def e4m3_to_f32(a: np.ndarray) -> np.ndarray:
    table = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return table[a]


def canonical_sum(x: np.ndarray, P: int = 32) -> float:
    x = f32(x)
    return lib().orc_canonical_sum(_p(x), x.size, P)


def numpy_sum(x: np.ndarray) -> float:
    x = f32(x)
    return lib().orc_numpy_sum(_p(x), x.size)


def adaln_fwd(res, shift, scale, x=None, gate=None, eps=1e-6, fp8=False, mode=RNE):
    """Row AdaLN (optionally gated residual, optionally FP8).  res/x: [B, S, D] uint16."""
    res = u16(res)
    B, S, D = res.shape
    shift, scale = u16(shift), u16(scale)
    has_x = x is not None
    x = u16(x) if has_x else None
    gate = u16(gate) if has_x else None
    h = None if fp8 else np.empty((B, S, D), np.uint16)
    z = np.empty((B, S, D), np.uint16) if has_x else None
    q = np.empty((B, S, D), np.uint8) if fp8 else None
    s = np.empty((B * S, 1), np.float32) if fp8 else None
    lib().orc_adaln_fwd(_p(x), _p(res), _p(gate), _p(shift), _p(scale), _p(h), _p(z), _p(q),
                        _p(s), B, S, D, eps, int(has_x), int(fp8), mode)
    return {"h": h, "z": z, "q": q, "s": s}


def rowquant(x, gelu=False, mode=RNE, want_y=False):
    """Per-row e4m3 quantisation.  x: [..., K] uint16 -> (q uint8, s [rows,1] f32[, y])."""
    x = u16(x)
    K = x.shape[-1]
    rows = x.size // K
    q = np.empty(x.shape, np.uint8)
    s = np.empty((rows, 1), np.float32)
    y = np.empty(x.shape, np.float32) if want_y else None
    lib().orc_rowquant(_p(x), _p(q), _p(s), _p(y), rows, K, int(gelu), mode)
    return (q, s, y) if want_y else (q, s)


def qkv_norm_rope(qkv, qw, kw, cos, sin, heads, eps=1e-5, with_v=False, mode=RNE):
    qkv = u16(qkv)
    B, S, W = qkv.shape
    hd = W // (3 * heads)
    q = np.empty((B, S, heads, hd), np.uint16)
    k = np.empty_like(q)
    v = np.empty_like(q) if with_v else None
    lib().orc_qkv_norm_rope(_p(qkv), _p(f32(qw)), _p(f32(kw)), _p(f32(cos)), _p(f32(sin)), _p(q),
                            _p(k), _p(v), B, S, heads, hd, eps, mode)
    return q, k, v


def head_norm(x, w, heads, eps=1e-5, mode=RNE):
    x = u16(x)
    B, S, W = x.shape
    hd = W // heads
    y = np.empty((B, S, heads, hd), np.uint16)
    lib().orc_head_norm(_p(x), _p(f32(w)), _p(y), B, S, heads, hd, eps, mode)
    return y


def gelu(x_bits: np.ndarray) -> np.ndarray:
    """Canonical GELU of bf16 inputs (fp32 outputs)."""
    x = u16(x_bits)
    y = np.empty(x.shape, np.float32)
    lib().orc_gelu_many(_p(x), _p(y), x.size)
    return y


# Chunk geometry of the CUDA backward kernels (csrc/adaln_bwd.cu, headnorm_bwd.cu):
# it fixes the order of the parameter-gradient sums.  AdaLN: chunks of 28 rows,
# each column summed over the chunk's rows in increasing order from zero (one
# stream of 28 rows).
BWD_WARPS = 1
BWD_ROWS_PER_WARP = 28
HN_WARPS = 8
HN_TOK_PER_WARP = 1


def adaln_bwd(gh, z, scale, x=None, gate=None, gz=None, eps=1e-6, mode=RNE):
    """Backward of (residual_)adaln.  Returns dict dz, dx, dgate, dshift, dscale."""
    gh, z, scale = u16(gh), u16(z), u16(scale)
    B, S, D = z.shape
    has_x = x is not None
    x = u16(x) if has_x else None
    gate = u16(gate) if has_x else None
    gz = u16(gz) if gz is not None else None
    dz = np.empty((B, S, D), np.uint16)
    dx = np.empty((B, S, D), np.uint16) if has_x else None
    dgate = np.empty((B, D), np.uint16) if has_x else None
    dshift = np.empty((B, D), np.uint16)
    dscale = np.empty((B, D), np.uint16)
    lib().orc_adaln_bwd(_p(gh), _p(gz), _p(z), _p(x), _p(gate), _p(scale), _p(dz), _p(dx),
                        _p(dgate), _p(dshift), _p(dscale), B, S, D, eps, BWD_WARPS,
                        BWD_ROWS_PER_WARP, mode)
    return {"dz": dz, "dx": dx, "dgate": dgate, "dshift": dshift, "dscale": dscale}


def qkv_norm_rope_bwd(qkv, dq, dk, dv, qw, kw, cos, sin, heads, eps=1e-5, mode=RNE):
    qkv = u16(qkv)
    B, S, W = qkv.shape
    hd = W // (3 * heads)
    width = heads * hd
    dqkv = np.empty_like(qkv)
    dqw = np.empty(hd, np.float32)
    dkw = np.empty(hd, np.float32)
    lib().orc_headnorm_bwd(_p(qkv), 3 * width, 0, width, 2 * width, _p(u16(dq)), _p(u16(dk)),
                           _p(u16(dv)), _p(f32(qw)), _p(f32(kw)), _p(f32(cos)), _p(f32(sin)),
                           _p(dqkv), _p(dqw), _p(dkw), B * S, S, heads, hd, eps, 1, 2, HN_WARPS,
                           HN_TOK_PER_WARP, mode)
    return dqkv, dqw, dkw


def head_norm_bwd(x, dy, w, heads, eps=1e-5, mode=RNE):
    x = u16(x)
    B, S, W = x.shape
    hd = W // heads
    dx = np.empty_like(x)
    dw = np.empty(hd, np.float32)
    lib().orc_headnorm_bwd(_p(x), W, 0, 0, 0, _p(u16(dy)), None, None, _p(f32(w)), None, None,
                           None, _p(dx), _p(dw), None, B * S, S, heads, hd, eps, 0, 1, HN_WARPS,
                           HN_TOK_PER_WARP, mode)
    return dx, dw


def exp(a: float) -> float:
    """The canonical fp32 exp (Cody-Waite reduction, degree-7 Taylor)."""
    return float(lib().orc_exp(float(a)))


def ctx_scale(out, lse, ln_pad, dy=None, mode=RNE):
    """ctx_scale forward (dy None: returns y) or backward (returns dout, dlse).
    out/dy: [B,S,H,hd] bf16 bits; lse: [B,H,S] fp32; ln_pad: [B] fp32."""
    out = u16(out)
    B, S, H, hd = out.shape
    lse, ln_pad = f32(lse), f32(ln_pad)
    if dy is None:
        y = np.empty_like(out)
        lib().orc_ctx_scale(_p(out), _p(lse), _p(ln_pad), None, _p(y), None, None, B, S, H, hd, mode)
        return y
    dout = np.empty_like(out)
    dlse = np.empty_like(lse)
    lib().orc_ctx_scale(_p(out), _p(lse), _p(ln_pad), _p(u16(dy)), None, _p(dout), _p(dlse), B, S, H,
                        hd, mode)
    return dout, dlse


def ctx_scale_rowquant(out, lse, ln_pad, mode=RNE):
    """rowquant(ctx_scale(out, lse, ln_pad).flatten(2)): the two restatements
    one after the other.  Returns (q [B, S, H*hd] uint8, s [B*S, 1] f32)."""
    y = ctx_scale(out, lse, ln_pad, mode=mode)
    B, S, H, hd = y.shape
    return rowquant(y.reshape(B, S, H * hd), mode=mode)


def rms_lpr(C: int) -> int:
    """Lanes per row of the canonical rms order (P of its row sums)."""
    return int(lib().orc_rms_lpr(C))


def rms_silu_fwd(x, g, r=None, shuffled=False, mode=RNE):
    """rms_silu (r None, not shuffled): returns y; add_rms_silu (r given) and
    shuffle_rms_silu (shuffled, x = u [B, h, w, 4C]): return (s, y).
    Activations are bf16 bits, channels last; g is [C] fp32."""
    x = u16(x)
    g = f32(g)
    C = g.size
    if shuffled:
        B, h, w, _ = x.shape
        shape, H, W = (B, 2 * h, 2 * w, C), 2 * h, 2 * w
    else:
        shape, H, W = x.shape, 0, 0
    N = int(np.prod(shape[:-1]))
    y = np.empty(shape, np.uint16)
    s = np.empty(shape, np.uint16) if (r is not None or shuffled) else None
    lib().orc_rms_silu_fwd(_p(x), _p(u16(r)) if r is not None else None, _p(g), _p(s), _p(y), N, H, W,
                           C, int(shuffled), mode)
    return y if s is None else (s, y)


def rms_silu_bwd(s, g, dy, gs=None, shuffled=False, mode=RNE):
    """Returns (ds, dg): ds in the input layout (u's with shuffled), dg [C] fp32."""
    s = u16(s)
    g = f32(g)
    C = g.size
    if shuffled:
        B, H, W, _ = s.shape
        ds_shape = (B, H // 2, W // 2, 4 * C)
    else:
        H = W = 0
        ds_shape = s.shape
    N = int(np.prod(s.shape[:-1]))
    ds = np.empty(ds_shape, np.uint16)
    dg = np.empty(C, np.float32)
    lib().orc_rms_silu_bwd(_p(s), _p(g), _p(u16(dy)), _p(u16(gs)) if gs is not None else None, _p(ds),
                           _p(dg), N, H, W, C, int(shuffled), mode)
    return ds, dg

"""Forward kernels on the GPU against the CPU oracle (bit-exact) and the torch
fp32 formulation (2 bf16 ulp).  Inputs are seeded on the CPU so both sides
see identical bits; every call goes through the public API and the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import anima_flat_b200 as afb
from anima_flat_b200 import _lib
from oracle import canonical as C
from oracle import formulation as Fm
from tests.conftest import from_bits, to_bits, ulp_diff_ok

pytestmark = pytest.mark.gpu


def rng(seed):
    return np.random.default_rng(seed)


def bf_bits(a: np.ndarray) -> np.ndarray:
    return to_bits(torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16))


def act(r, shape, outliers=0.0, std=1.0):
    a = r.standard_normal(shape, dtype=np.float32) * std
    if outliers:
        a = np.where(r.random(shape) < outliers, a * 20.0, a)
    return bf_bits(a)


def mods(r, B, D):
    return (bf_bits(r.standard_normal((B, D), dtype=np.float32) * 0.1),        # shift
            bf_bits(1.0 + r.standard_normal((B, D), dtype=np.float32) * 0.1),  # scale (+1)
            bf_bits(r.standard_normal((B, D), dtype=np.float32) * 0.1))        # gate


def dev(a, cuda_dev):
    return from_bits(a, cuda_dev)


# (64, 1, 2048) and (40, 3, 1024): CTAs whose rows span more than two batch
# entries read the modulation from global memory instead of shared memory.
# (3, 8192, 512) and (5, 4096, 2048): long launches (>= 128 rows per CTA),
# which take the deep ring; at D = 2048 the residual one gives up the
# shared-memory modulation slots for it.  The FP8 kernels at D = 2048 run 12
# warp pairs per CTA in short launches ((2, 4096, 2048), (64, 1, 2048)) and 8
# in long ones ((5, 4096, 2048)).
ADALN_SHAPES = [(1, 1, 2048), (2, 3, 2048), (1, 4096, 2048), (2, 37, 1024), (3, 5, 256),
                (1, 7, 4096), (1, 9, 8), (2, 11, 2040), (1, 3, 520), (64, 1, 2048), (40, 3, 1024),
                (3, 8192, 512), (5, 4096, 2048)]


@pytest.mark.parametrize("B,S,D", ADALN_SHAPES)
def test_residual_adaln_bit_exact(B, S, D, cuda_dev):
    r = rng(B * 1000 + S + D)
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    h, z = afb.residual_adaln(*(dev(a, cuda_dev) for a in (x, res, gate, shift, scale)))
    o = C.adaln_fwd(res, shift, scale, x=x, gate=gate)
    np.testing.assert_array_equal(to_bits(z), o["z"])
    np.testing.assert_array_equal(to_bits(h), o["h"])


@pytest.mark.parametrize("B,S,D", ADALN_SHAPES)
def test_adaln_bit_exact(B, S, D, cuda_dev):
    r = rng(B * 2000 + S + D)
    z = act(r, (B, S, D), outliers=0.01)
    shift, scale, _ = mods(r, B, D)
    h = afb.adaln(*(dev(a, cuda_dev) for a in (z, shift, scale)))
    o = C.adaln_fwd(z, shift, scale)
    np.testing.assert_array_equal(to_bits(h), o["h"])


@pytest.mark.parametrize("B,S,D", [(1, 1, 2048), (2, 4096, 2048), (2, 37, 1024), (3, 5, 256),
                                   (1, 7, 4096), (2, 11, 2040), (64, 1, 2048), (40, 3, 1024),
                                   (3, 8192, 512), (5, 4096, 2048)])
@pytest.mark.parametrize("has_x", [True, False])
def test_adaln_fp8_bit_exact(B, S, D, has_x, cuda_dev):
    r = rng(B * 3000 + S + D + has_x)
    x, res = act(r, (B, S, D), 0.01), act(r, (B, S, D), 0.01)
    shift, scale, gate = mods(r, B, D)
    if has_x:
        q, s, z = afb.residual_adaln_fp8(*(dev(a, cuda_dev) for a in (x, res, gate, shift, scale)))
        o = C.adaln_fwd(res, shift, scale, x=x, gate=gate, fp8=True)
        np.testing.assert_array_equal(to_bits(z), o["z"])
    else:
        q, s = afb.adaln_fp8(*(dev(a, cuda_dev) for a in (res, shift, scale)))
        o = C.adaln_fwd(res, shift, scale, fp8=True)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (B * S, 1) and s.dtype == torch.float32
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), o["s"].view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), o["q"])


@pytest.mark.parametrize("D", [2048, 1024])
@pytest.mark.parametrize("has_x", [True, False])
def test_adaln_fp8_nonfinite_rows(D, has_x, cuda_dev):
    """Rows holding a NaN or an infinity (in the residual stream, or through an
    infinite shift) take the NaN-ignoring row max and the NaN clamp to -448,
    bit-exact against the oracle; finite rows of the same launch are
    unaffected."""
    B, S = 2, 7
    r = rng(D + 7 * has_x)
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    resf = from_bits(res, "cpu").float().numpy()
    resf[0, 1, 5] = np.nan
    resf[0, 3, 9] = np.inf
    resf[1, 2, 17] = -np.inf
    res = bf_bits(resf)
    shf = from_bits(shift, "cpu").float().numpy()
    shf[1, 33] = -np.inf
    shift = bf_bits(shf)
    if has_x:
        q, s, z = afb.residual_adaln_fp8(*(dev(a, cuda_dev) for a in (x, res, gate, shift, scale)))
        o = C.adaln_fwd(res, shift, scale, x=x, gate=gate, fp8=True)
        # z: NaN where the oracle has NaN (the GPU writes the canonical NaN
        # 0x7FFF, the host's arithmetic may set the sign bit), equal bits elsewhere
        zb = to_bits(z)
        nan = (zb & 0x7FFF) > 0x7F80
        np.testing.assert_array_equal(nan, (o["z"] & 0x7FFF) > 0x7F80)
        assert nan.any()
        np.testing.assert_array_equal(zb[~nan], o["z"][~nan])
    else:
        q, s = afb.adaln_fp8(*(dev(a, cuda_dev) for a in (res, shift, scale)))
        o = C.adaln_fwd(res, shift, scale, fp8=True)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), o["s"].view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), o["q"])
    assert not np.isfinite(o["s"]).all() or (o["q"] == 0xFE).any()


@pytest.mark.parametrize("rows,K", [(1, 16), (7, 2048), (8192, 2048), (5, 2064), (3, 4096),
                                    (9, 8192), (2, 16384), (4, 6144)])
def test_rowquant_bit_exact(rows, K, cuda_dev):
    r = rng(rows + K)
    x = act(r, (1, rows, K), 0.01)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=False)
    oq, os_ = C.rowquant(x)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), oq)


def _midpoint_rows(K: int) -> np.ndarray:
    """Rows whose quotients y / s sit on and next to e4m3 rounding midpoints.

    Row amax A in {1344, 2240, 3136, 448, 1000} gives s = A/448 in {3, 5, 7,
    1, RN(1000/448)}; for the integer s, x = s*M is exact in bf16 for every
    e4m3 midpoint M (4 significant bits), so x / s is exactly a tie, where
    x * RN(1/s) can round to the wrong side.  Each row also holds the bf16
    neighbours of those x, tiny values below the e4m3 normal range, and
    signed zeros."""
    mids = []
    for e in range(-6, 9):
        for m in range(8):
            v = (1.0 + (2 * m + 1) / 16.0) * 2.0 ** e
            if v < 448.0:
                mids.append(v)
    mids = np.array(mids, dtype=np.float32)
    rows = []
    for amax in (1344.0, 2240.0, 3136.0, 448.0, 1000.0):
        s = np.float32(amax) / np.float32(448.0)
        x = (mids * s).astype(np.float32)
        xb = torch.from_numpy(x).to(torch.bfloat16)
        up = torch.nextafter(xb, torch.full_like(xb, float("inf")))
        dn = torch.nextafter(xb, torch.full_like(xb, float("-inf")))
        vals = torch.cat([xb, up, dn, -xb, -up]).float().numpy()
        tiny = np.array([1e-6, -1e-6, 3e-5 * amax, -2e-5 * amax, 0.0, -0.0], dtype=np.float32)
        row = np.concatenate([vals, tiny, np.array([amax], dtype=np.float32)])
        row = np.resize(row, K)
        row[-1] = amax
        rows.append(row)
    return bf_bits(np.stack(rows)[None])


@pytest.mark.parametrize("K", [2048, 8192])
def test_rowquant_codes_at_e4m3_midpoints(K, cuda_dev):
    """The exact rowquant path settles codes from y * RN(1/s) only away from
    e4m3 ties; on and next to ties its codes must still equal the IEEE
    quotient's (bit-exact against the oracle, signed zeros included)."""
    x = _midpoint_rows(K)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=False)
    oq, os_ = C.rowquant(x)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), oq)


def _nonfinite_rows(K: int) -> np.ndarray:
    r = rng(K + 99)
    x = r.standard_normal((5, K)).astype(np.float32)
    x[0, 5], x[0, 100] = np.nan, -0.0
    x[1, 7] = np.inf
    x[2, :] = 0.0
    x[2, 3] = -0.0
    x[3, 9], x[3, 10] = -np.inf, np.nan
    x[4, 11] = np.nan
    return bf_bits(x[None])


@pytest.mark.parametrize("K", [2048, 8192])
def test_rowquant_nonfinite_and_signed_zero(K, cuda_dev):
    """NaN takes the code of -448 (the reference clamps with max(NaN, -448)),
    an infinite row max gives an infinite scale, an all-zero row the 1e-12
    floor, and zeros keep their sign: bit-exact against the oracle."""
    x = _nonfinite_rows(K)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=False)
    oq, os_ = C.rowquant(x)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), oq)


def test_rowquant_gelu_nan_codes(cuda_dev):
    """GELU path: NaN inputs leave the exact scale alone and take code -448."""
    K = 8192
    x = _nonfinite_rows(K)[:, [0, 2, 4]]
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=True)
    oq, os_ = C.rowquant(x, gelu=True)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    xf = from_bits(x, "cpu").float().numpy().reshape(3, K)
    qb = to_bits(q).reshape(3, K)
    nan = np.isnan(xf)
    assert nan.sum() == 2 and np.all(qb[nan] == 0xFE) and np.all(oq.reshape(3, K)[nan] == 0xFE)


def _codes_at_ties_only(q_bits, y, s):
    """Codes equal e4m3(y/s) except where y/s is within 4 fp32 ulp of an e4m3 tie."""
    rows = s.shape[0]
    v = np.clip((y.reshape(rows, -1) / s.reshape(rows, 1)).astype(np.float32), -448, 448)
    exact = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    bad = q_bits.reshape(rows, -1) != exact
    if bad.any():
        lo, hi = v[bad], v[bad]
        for _ in range(4):
            lo = np.nextafter(lo, -np.inf, dtype=np.float32)
            hi = np.nextafter(hi, np.inf, dtype=np.float32)
        c = lambda a: torch.from_numpy(a).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.all(c(lo) != c(hi)), "an FP8 code differs away from a rounding tie"
    return int(bad.sum())


@pytest.mark.parametrize("rows,K,outliers", [(7, 2048, 0.01), (8192, 8192, 0.01), (256, 8192, 0.0),
                                             (64, 2048, 0.0), (3, 16384, 0.0), (5, 16, 0.0)])
def test_rowquant_gelu_scale_exact_codes_at_ties(rows, K, outliers, cuda_dev):
    r = rng(rows * 7 + K)
    x = act(r, (1, rows, K), outliers)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=True)
    oq, os_, oy = C.rowquant(x, gelu=True, want_y=True)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    _codes_at_ties_only(to_bits(q), oy, os_)


@pytest.mark.parametrize("K", [8192, 2048, 16384, 1024, 16])
def test_rowquant_gelu_exhaustive(K, cuda_dev):
    """Every finite bf16 input, in rows of K inputs of neighbouring magnitude
    (both signs, shuffled within the row, zero padding), so that each row's
    codes span the e4m3 range, and (K >= 128) the non-finite rows of
    _nonfinite_rows, +inf and -inf included: GELU scales bit-exact against
    the oracle, codes equal to the oracle's except where y/s lies within 4
    fp32 ulp of an e4m3 rounding tie."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = (bits.astype(np.uint32) << 16).view(np.float32)
    fin = bits[np.isfinite(vals)]
    fin = fin[np.argsort(fin & 0x7FFF, kind="stable")]
    pad = (-fin.size) % K
    x = np.concatenate([fin, np.zeros(pad, np.uint16)]).reshape(-1, K)
    r = rng(K)
    for row in x:
        r.shuffle(row)
    x = x[None]
    if K >= 128:
        x = np.concatenate([x, _nonfinite_rows(K)], axis=1)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=True)
    oq, os_, oy = C.rowquant(x, gelu=True, want_y=True)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    qb = to_bits(q).reshape(oq.shape)
    bad = qb != oq
    if bad.any():
        rows = os_.shape[0]
        with np.errstate(invalid="ignore"):  # rows of +inf: inf / inf where the codes agree
            v = (oy.reshape(rows, -1) / os_.reshape(rows, 1)).astype(np.float32).reshape(oq.shape)[bad]
        assert np.all(np.isfinite(v)), "a code differs where the quotient is not finite"
        lo, hi = v.copy(), v.copy()
        for _ in range(4):
            lo = np.nextafter(lo, -np.inf, dtype=np.float32)
            hi = np.nextafter(hi, np.inf, dtype=np.float32)
        c = lambda a: torch.from_numpy(np.clip(a, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.all(c(lo) != c(hi)), "an FP8 code differs away from a rounding tie"


@pytest.mark.parametrize("K", [8192, 2048, 16])
def test_rowquant_exhaustive_bit_exact(K, cuda_dev):
    """Without GELU: every finite bf16 input, in rows of neighbouring
    magnitude as above, and (K >= 128) the non-finite rows: codes and scales
    bit-exact against the oracle."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = (bits.astype(np.uint32) << 16).view(np.float32)
    fin = bits[np.isfinite(vals)]
    fin = fin[np.argsort(fin & 0x7FFF, kind="stable")]
    pad = (-fin.size) % K
    x = np.concatenate([fin, np.zeros(pad, np.uint16)]).reshape(-1, K)
    r = rng(K + 1)
    for row in x:
        r.shuffle(row)
    x = x[None]
    if K >= 128:
        x = np.concatenate([x, _nonfinite_rows(K)], axis=1)
    q, s = afb.rowquant(dev(x, cuda_dev), gelu=False)
    oq, os_ = C.rowquant(x)
    np.testing.assert_array_equal(to_bits(s).view(np.uint32), os_.view(np.uint32))
    np.testing.assert_array_equal(to_bits(q), oq)


def test_gelu_probe_exhaustive(cuda_dev):
    """Over all finite bf16 inputs: the device canonical GELU equals the
    oracle's bit for bit, and the fast GELU stays within the bound the row
    kernel relies on (|fast - canon| <= 2^-20 + 2^-12 |canon|)."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = (bits.astype(np.uint32) << 16).view(np.float32)
    bits = bits[np.isfinite(vals)]
    x = torch.from_numpy(bits.view(np.int16)).to(cuda_dev)
    fast = torch.empty(x.numel(), dtype=torch.float32, device=cuda_dev)
    canon = torch.empty_like(fast)
    _lib.call("afb_gelu_probe", x.data_ptr(), fast.data_ptr(), canon.data_ptr(), x.numel(),
              torch.cuda.current_stream().cuda_stream)
    canon_h = canon.cpu().numpy()
    np.testing.assert_array_equal(canon_h.view(np.uint32), C.gelu(bits).view(np.uint32))
    f = fast.cpu().numpy().astype(np.float64)
    c = canon_h.astype(np.float64)
    bound = 2.0 ** -20 + 2.0 ** -12 * np.abs(c)
    assert np.all(np.abs(f - c) <= bound)


# (1, 19000, 4, 128): a long launch (>= 256 units per CTA, deep ring).
QKV_CASES = [(1, 4096, 16, 128, 1e-5), (2, 16, 4, 128, 1e-5), (1, 6, 3, 64, 1e-6),
             (1, 5, 2, 256, 1e-5), (2, 7, 5, 128, 1e-6), (3, 1, 16, 128, 1e-5),
             (1, 19000, 4, 128, 1e-5)]


def qkv_inputs(r, B, S, H, hd):
    qkv = act(r, (B, S, 3 * H * hd))
    qw = (1.0 + r.standard_normal(hd) * 0.02).astype(np.float32)
    kw = (1.0 + r.standard_normal(hd) * 0.02).astype(np.float32)
    ang = r.random((S, hd // 2)).astype(np.float32) * 6.0
    return qkv, qw, kw, np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


@pytest.mark.parametrize("B,S,H,hd,eps", QKV_CASES)
def test_qkv_norm_rope_bit_exact(B, S, H, hd, eps, cuda_dev):
    r = rng(B + S + H + hd)
    qkv, qw, kw, cos, sin = qkv_inputs(r, B, S, H, hd)
    args = [from_bits(a, cuda_dev) for a in (qkv, qw, kw, cos, sin)]
    with torch.no_grad():
        q, k, v = afb.qkv_norm_rope(*args, H, eps)
    oq, ok, _ = C.qkv_norm_rope(qkv, qw, kw, cos, sin, H, eps)
    np.testing.assert_array_equal(to_bits(q), oq)
    np.testing.assert_array_equal(to_bits(k), ok)
    assert v.data_ptr() == args[0].data_ptr() + 2 * H * hd * 2  # strided view of qkv
    # grad mode copies v through the kernel
    qkv_g = args[0].clone().requires_grad_(True)
    q2, k2, v2 = afb.qkv_norm_rope(qkv_g, *args[1:], H, eps)
    np.testing.assert_array_equal(to_bits(q2), oq)
    np.testing.assert_array_equal(to_bits(v2), qkv.reshape(B, S, 3, H, hd)[:, :, 2])


@pytest.mark.parametrize("B,S,H,hd", [(1, 4096, 16, 128), (2, 5, 4, 128), (1, 3, 7, 64), (2, 2, 3, 256),
                                      (1, 38000, 2, 64)])
def test_head_norm_bit_exact(B, S, H, hd, cuda_dev):
    r = rng(B * 11 + S + H + hd)
    x = act(r, (B, S, H * hd))
    w = (1.0 + r.standard_normal(hd) * 0.02).astype(np.float32)
    y = afb.head_norm(from_bits(x, cuda_dev), from_bits(w, cuda_dev), H, 1e-5)
    np.testing.assert_array_equal(to_bits(y), C.head_norm(x, w, H, 1e-5))


def test_config2_within_2_ulp_of_torch_fp32(cuda_dev):
    """The config-2 shapes against the reference's unfused torch fp32 composition."""
    r = rng(2)
    B, S, D, H, hd = 1, 4096, 2048, 16, 128
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    t = [dev(a, cuda_dev) for a in (x, res, gate, shift, scale)]
    h, z = afb.residual_adaln(*t)
    h_ref, z_ref = Fm.residual_adaln(*t)
    assert torch.equal(z, z_ref)
    # 2 bf16 ulp at the magnitude of the last addition's operands (LN(z)*scale
    # and shift): where they cancel, the result itself is no measure of error.
    t_ref = torch.nn.functional.layer_norm(z_ref.float(), (D,), eps=1e-6) * t[4].float()[:, None]
    y_ref = t_ref + t[3].float()[:, None]
    mag = torch.maximum(y_ref.abs(), torch.maximum(t_ref.abs(), t[3].float()[:, None].abs()))
    ok, worst = ulp_diff_ok(to_bits(h), y_ref.cpu().numpy(), 2.0, mag=mag.cpu().numpy())
    assert ok, worst
    # and in ulp of the output itself, except where the last addition cancels
    # by more than 2x (there any fp32 evaluation, torch's included, is off by
    # several ulp of y: torch on the GPU and on the CPU disagree by tens)
    keep = (y_ref.abs() * 2.0 >= mag).cpu().numpy()
    hb = to_bits(h)
    ok, strict = ulp_diff_ok(hb[keep], y_ref.cpu().numpy()[keep], 2.0)
    assert ok, strict
    print(f"residual_adaln vs torch fp32: worst {worst:.3f} ulp (operand scale), {strict:.2f} ulp of y "
          f"outside 2x cancellation ({100.0 * (1 - keep.mean()):.1f}% excluded)")
    qkv, qw, kw, cos, sin = qkv_inputs(r, B, S, H, hd)
    a = [from_bits(v, cuda_dev) for v in (qkv, qw, kw, cos, sin)]
    with torch.no_grad():
        q, k, _ = afb.qkv_norm_rope(*a, H, 1e-5)
    # fp32 rotation of the torch-normed heads; tolerance at the rotation operands' scale
    qkv_t = a[0].view(B, S, 3, H, hd)
    for ours, part, w in ((q, qkv_t[:, :, 0], a[1]), (k, qkv_t[:, :, 1], a[2])):
        n = Fm._rms_heads(part, w, 1e-5).float()
        half = hd // 2
        na, nb = n[..., :half], n[..., half:]
        c, s_ = a[3][None, :, None, :], a[4][None, :, None, :]
        y = torch.cat([na * c - nb * s_, nb * c + na * s_], dim=-1)
        mag = torch.cat([torch.maximum((na * c).abs(), (nb * s_).abs()),
                         torch.maximum((nb * c).abs(), (na * s_).abs())], dim=-1)
        ok, worst = ulp_diff_ok(to_bits(ours), y.cpu().numpy(), 2.0, mag=mag.cpu().numpy())
        assert ok, worst


def test_pdl_off_gives_identical_results(cuda_dev):
    r = rng(5)
    B, S, D = 2, 300, 2048
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    t = [dev(a, cuda_dev) for a in (x, res, gate, shift, scale)]
    h1, z1 = afb.residual_adaln(*t)
    _lib.set_pdl(False)
    try:
        h2, z2 = afb.residual_adaln(*t)
    finally:
        _lib.set_pdl(True)
    assert torch.equal(h1, h2) and torch.equal(z1, z2)


def test_side_stream_and_noncontiguous_modulation(cuda_dev):
    """Launches follow the current stream; strided [B, D] views are accepted
    (the final layer passes fin.chunk(2, -1) halves, model.py:374-375)."""
    r = rng(6)
    B, S, D = 2, 64, 2048
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    t = [dev(a, cuda_dev) for a in (x, res, gate, shift, scale)]
    fin = torch.cat([t[3], t[4]], dim=-1)
    sh_view, sc_view = fin.chunk(2, dim=-1)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        h, z = afb.residual_adaln(t[0], t[1], t[2], sh_view, sc_view)
    side.synchronize()
    o = C.adaln_fwd(res, shift, scale, x=x, gate=gate)
    np.testing.assert_array_equal(to_bits(h), o["h"])

"""ctx_scale forward and backward on the GPU against the CPU oracle, bit-exact
(y and dout bf16 bits, dlse fp32 bits), through the public API and the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import anima_flat_b200 as afb
from oracle import canonical as C
from tests.conftest import from_bits, to_bits

pytestmark = pytest.mark.gpu


def _inputs(B, S, H, hd, seed, spread=4.0):
    r = np.random.default_rng(seed)
    bf = lambda a: to_bits(torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16))
    out = bf(r.standard_normal((B, S, H, hd)))
    dy = bf(r.standard_normal((B, S, H, hd)) * 1e-2)
    lse = (r.standard_normal((B, H, S)) * spread + 2.0).astype(np.float32)
    ln_pad = np.log(r.integers(1, 400, B)).astype(np.float32)
    return out, lse, ln_pad, dy


CASES = [(1, 4096, 16, 128), (2, 37, 5, 64), (1, 7, 8, 256), (3, 1, 16, 128), (2, 300, 3, 128)]


@pytest.mark.parametrize("B,S,H,hd", CASES)
def test_ctx_scale_bit_exact(B, S, H, hd, cuda_dev):
    out, lse, ln_pad, dy = _inputs(B, S, H, hd, B * 100 + S + H + hd)
    y = afb.ctx_scale(from_bits(out, cuda_dev), torch.from_numpy(lse).to(cuda_dev),
                      torch.from_numpy(ln_pad).to(cuda_dev))
    np.testing.assert_array_equal(to_bits(y), C.ctx_scale(out, lse, ln_pad))


@pytest.mark.parametrize("B,S,H,hd", CASES)
def test_ctx_scale_bwd_bit_exact(B, S, H, hd, cuda_dev):
    out, lse, ln_pad, dy = _inputs(B, S, H, hd, B * 200 + S + H + hd)
    dout, dlse = torch.ops.anima_flat_b200.ctx_scale_bwd(
        from_bits(out, cuda_dev), torch.from_numpy(lse).to(cuda_dev),
        torch.from_numpy(ln_pad).to(cuda_dev), from_bits(dy, cuda_dev))
    od, ol = C.ctx_scale(out, lse, ln_pad, dy=dy)
    np.testing.assert_array_equal(to_bits(dout), od)
    np.testing.assert_array_equal(to_bits(dlse).view(np.uint32), ol.view(np.uint32))


def test_ctx_scale_saturated_gains(cuda_dev):
    """lse far below / above ln_pad: exp overflows to inf (gain 0) or
    underflows to 0 (gain 1); both bit-exact, dlse 0 at saturation."""
    B, S, H, hd = 2, 64, 4, 128
    out, lse, ln_pad, dy = _inputs(B, S, H, hd, 7)
    lse[:, :, ::3] = -150.0
    lse[:, :, 1::3] = 300.0
    y = afb.ctx_scale(from_bits(out, cuda_dev), torch.from_numpy(lse).to(cuda_dev),
                      torch.from_numpy(ln_pad).to(cuda_dev))
    np.testing.assert_array_equal(to_bits(y), C.ctx_scale(out, lse, ln_pad))
    dout, dlse = torch.ops.anima_flat_b200.ctx_scale_bwd(
        from_bits(out, cuda_dev), torch.from_numpy(lse).to(cuda_dev),
        torch.from_numpy(ln_pad).to(cuda_dev), from_bits(dy, cuda_dev))
    od, ol = C.ctx_scale(out, lse, ln_pad, dy=dy)
    np.testing.assert_array_equal(to_bits(dout), od)
    np.testing.assert_array_equal(to_bits(dlse).view(np.uint32), ol.view(np.uint32))


def test_ctx_scale_autograd_uses_the_backward_op(cuda_dev):
    B, S, H, hd = 1, 33, 16, 128
    out, lse, ln_pad, dy = _inputs(B, S, H, hd, 9)
    o = from_bits(out, cuda_dev).requires_grad_(True)
    lt = torch.from_numpy(lse).to(cuda_dev).requires_grad_(True)
    y = afb.ctx_scale(o, lt, torch.from_numpy(ln_pad).to(cuda_dev))
    y.backward(from_bits(dy, cuda_dev))
    od, ol = C.ctx_scale(out, lse, ln_pad, dy=dy)
    np.testing.assert_array_equal(to_bits(o.grad), od)
    np.testing.assert_array_equal(to_bits(lt.grad).view(np.uint32), ol.view(np.uint32))


def test_ctx_scale_rejects_bad_shapes(cuda_dev):
    out = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(ValueError):
        afb.ctx_scale(out, torch.zeros(1, 4, 2, device=cuda_dev), torch.zeros(1, device=cuda_dev))
    with pytest.raises(ValueError):
        afb.ctx_scale(out.cpu(), torch.zeros(1, 2, 4), torch.zeros(1))


# The trimmed cross-attention output path of the FP8 forward in one pass.
FUSED_CASES = [(2, 4096, 16, 128), (1, 37, 5, 64), (3, 9, 8, 256), (2, 300, 3, 128), (1, 5, 64, 256)]


@pytest.mark.parametrize("B,S,H,hd", FUSED_CASES)
def test_ctx_scale_rowquant_equals_the_two_ops(B, S, H, hd, cuda_dev):
    """Codes and scales equal rowquant(ctx_scale(...)) on the device and the
    oracle's composition of the two, bit for bit; saturated gains included.
    (The fused op takes rows up to 16384 wide; ctx_scale alone up to 2048, so
    wider cases compare with the oracle only.)"""
    out, lse, ln_pad, _ = _inputs(B, S, H, hd, B * 300 + S + H + hd)
    lse[:, :, ::7] = -150.0
    lse[:, :, 3::7] = 300.0
    o, l_, lp = from_bits(out, cuda_dev), torch.from_numpy(lse).to(cuda_dev), torch.from_numpy(ln_pad).to(cuda_dev)
    q, s = afb.ctx_scale_rowquant(o, l_, lp)
    assert q.shape == (B, S, H * hd) and q.dtype == torch.float8_e4m3fn and s.shape == (B * S, 1)
    if H * hd <= 2048:
        rq, rs = afb.rowquant(afb.ctx_scale(o, l_, lp).flatten(2))
        assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8))
        assert torch.equal(s.view(torch.int32), rs.view(torch.int32))
    oq, os_ = C.ctx_scale_rowquant(out, lse, ln_pad)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), oq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), os_.view(np.uint32))


def test_ctx_scale_rowquant_rejects_bad_shapes(cuda_dev):
    out = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(ValueError):
        afb.ctx_scale_rowquant(out, torch.zeros(1, 4, 2, device=cuda_dev), torch.zeros(1, device=cuda_dev))
    with pytest.raises(ValueError):
        afb.ctx_scale_rowquant(out.float(), torch.zeros(1, 2, 4, device=cuda_dev), torch.zeros(1, device=cuda_dev))

"""VAE rms_silu family on the GPU against the CPU oracle, bit-exact (s, y, ds
bf16 bits; the gamma gradient fp32 bits), through the public API, the custom
ops' autograd and the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import anima_flat_b200 as afb
from oracle import canonical as C
from tests.conftest import from_bits, to_bits

pytestmark = pytest.mark.gpu


def _bf(a):
    return to_bits(torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16))


def _gamma(Cn, seed):
    return (1.0 + 0.1 * np.random.default_rng(seed).standard_normal(Cn)).astype(np.float32)


# (1, 300, 300): many units per warp and a ragged last unit; C = 128 and
# 1024 fill all four vector slots of a lane.
SHAPES = [((1, 16, 24), 96), ((2, 9, 7), 192), ((1, 5, 11), 384), ((3, 4, 4), 8), ((1, 6, 6), 40),
          ((1, 33, 31), 1024), ((1, 64, 64), 96), ((1, 300, 300), 96), ((2, 45, 37), 128)]


@pytest.mark.parametrize("lead,Cn", SHAPES)
def test_rms_silu_bit_exact(lead, Cn, cuda_dev):
    r = np.random.default_rng(Cn + lead[1])
    x = _bf(r.standard_normal((*lead, Cn)))
    g = _gamma(Cn, 1)
    y = afb.rms_silu(from_bits(x, cuda_dev), torch.from_numpy(g).to(cuda_dev))
    np.testing.assert_array_equal(to_bits(y), C.rms_silu_fwd(x, g))


@pytest.mark.parametrize("lead,Cn", SHAPES[:4])
def test_add_rms_silu_bit_exact(lead, Cn, cuda_dev):
    r = np.random.default_rng(2 * Cn + lead[1])
    x, res = _bf(r.standard_normal((*lead, Cn))), _bf(r.standard_normal((*lead, Cn)))
    g = _gamma(Cn, 2)
    s, y = afb.add_rms_silu(from_bits(x, cuda_dev), from_bits(res, cuda_dev), torch.from_numpy(g).to(cuda_dev))
    os_, oy = C.rms_silu_fwd(x, g, r=res)
    np.testing.assert_array_equal(to_bits(s), os_)
    np.testing.assert_array_equal(to_bits(y), oy)


@pytest.mark.parametrize("B,h,w,Cn", [(1, 8, 12, 96), (2, 3, 5, 192), (1, 16, 16, 96), (1, 128, 160, 96),
                                       (3, 7, 1, 1024), (1, 9, 2, 8)])
def test_shuffle_rms_silu_bit_exact(B, h, w, Cn, cuda_dev):
    r = np.random.default_rng(h * w + Cn)
    u = _bf(r.standard_normal((B, h, w, 4 * Cn)))
    g = _gamma(Cn, 3)
    s, y = afb.shuffle_rms_silu(from_bits(u, cuda_dev), torch.from_numpy(g).to(cuda_dev))
    os_, oy = C.rms_silu_fwd(u, g, shuffled=True)
    np.testing.assert_array_equal(to_bits(s), os_)
    np.testing.assert_array_equal(to_bits(y), oy)


@pytest.mark.parametrize("lead,Cn,with_gs,shuffled", [((1, 16, 24), 96, False, False),
                                                      ((2, 9, 7), 192, True, False),
                                                      ((1, 8, 12), 96, True, True),
                                                      ((1, 5, 11), 384, False, False),
                                                      ((1, 40, 40), 96, True, False),
                                                      ((3, 4, 4), 8, False, False),
                                                      ((1, 300, 300), 96, True, False),
                                                      ((1, 64, 80), 96, True, True),
                                                      ((2, 45, 37), 128, False, False),
                                                      ((1, 8, 6), 1024, True, True)])
def test_rms_silu_bwd_bit_exact(lead, Cn, with_gs, shuffled, cuda_dev):
    r = np.random.default_rng(Cn * 3 + lead[1])
    s = _bf(r.standard_normal((*lead, Cn)))
    dy = _bf(r.standard_normal((*lead, Cn)) * 1e-2)
    gs = _bf(r.standard_normal((*lead, Cn)) * 1e-2) if with_gs else None
    g = _gamma(Cn, 4)
    ds, dg = torch.ops.anima_flat_b200.rms_silu_bwd(
        from_bits(s, cuda_dev), torch.from_numpy(g).to(cuda_dev), from_bits(dy, cuda_dev),
        from_bits(gs, cuda_dev) if gs is not None else None, shuffled)
    ods, odg = C.rms_silu_bwd(s, g, dy, gs=gs, shuffled=shuffled)
    np.testing.assert_array_equal(to_bits(ds), ods)
    np.testing.assert_array_equal(to_bits(dg).view(np.uint32), odg.view(np.uint32))


def test_rms_silu_autograd(cuda_dev):
    r = np.random.default_rng(5)
    x = _bf(r.standard_normal((1, 6, 10, 96)))
    dy = _bf(r.standard_normal((1, 6, 10, 96)) * 1e-2)
    g = _gamma(96, 6)
    xt = from_bits(x, cuda_dev).requires_grad_(True)
    gt = torch.from_numpy(g).to(cuda_dev).requires_grad_(True)
    afb.rms_silu(xt, gt).backward(from_bits(dy, cuda_dev))
    ods, odg = C.rms_silu_bwd(x, g, dy)
    np.testing.assert_array_equal(to_bits(xt.grad), ods)
    np.testing.assert_array_equal(to_bits(gt.grad).view(np.uint32), odg.view(np.uint32))


def test_rms_silu_rejects_bad_inputs(cuda_dev):
    g = torch.ones(100, device=cuda_dev)
    with pytest.raises(ValueError):
        afb.rms_silu(torch.zeros(2, 100, dtype=torch.bfloat16, device=cuda_dev), g)
    with pytest.raises(ValueError):
        afb.rms_silu(torch.zeros(2, 96, dtype=torch.float32, device=cuda_dev), torch.ones(96, device=cuda_dev))


def test_rms_silu_bwd_doubled_chunks(cuda_dev):
    """More than 32768 chunks of 8 tiles (C = 8: 256 rows a chunk): the chunk
    doubles to 16 tiles, in the oracle and on the device alike."""
    lead, Cn = (1, 2900, 2900), 8
    r = np.random.default_rng(77)
    s = _bf(r.standard_normal((*lead, Cn)))
    dy = _bf(r.standard_normal((*lead, Cn)) * 1e-2)
    g = _gamma(Cn, 8)
    ds, dg = torch.ops.anima_flat_b200.rms_silu_bwd(
        from_bits(s, cuda_dev), torch.from_numpy(g).to(cuda_dev), from_bits(dy, cuda_dev), None, False)
    ods, odg = C.rms_silu_bwd(s, g, dy)
    np.testing.assert_array_equal(to_bits(ds), ods)
    np.testing.assert_array_equal(to_bits(dg).view(np.uint32), odg.view(np.uint32))


def test_silu_fast_path_exhaustive(cuda_dev):
    """Every fp32 input: where the forward keeps the SFU value (settled), its
    bf16 rounding equals the canonical SiLU's, and the recomputed share stays
    small; the backward's branch-free sigmoid equals the canonical one bit for
    bit on every |a| <= 87."""
    from anima_flat_b200 import _lib

    stats = torch.zeros(515, dtype=torch.int64, device=cuda_dev)
    _lib.call("afb_silu_probe", stats.data_ptr(), torch.cuda.current_stream().cuda_stream)
    st = stats.cpu().numpy().astype(np.uint64)
    assert st[0] == 0, f"{st[0]} settled inputs round differently"
    assert st[514] == 0, f"{st[514]} inputs where the fast sigmoid differs"
    n_small = 2 * (0x41000000 + 1)  # fp32 values with |a| <= 8
    assert st[1] / n_small < 0.002, f"unsettled share {st[1] / n_small:.4%}"

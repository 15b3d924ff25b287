"""Backward kernels (LoRA training path) on the GPU against the CPU oracle.

Per-row gradients and the parameter gradients are bit-exact: both sides sum
the parameter gradients in the same fixed chunk order.  Autograd through the
public functions is checked against the same oracle, and against torch
autograd of the fp32 composition within tolerance."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import anima_flat_b200 as afb
from oracle import canonical as C
from tests.conftest import from_bits, to_bits
from tests.test_gpu_forward import act, mods, qkv_inputs, rng

pytestmark = pytest.mark.gpu


# (2, 33000, 256): more than 1024 chunks of 28 rows per batch entry, so the
# parameter gradients take the two-launch finalize, with two batch entries.
@pytest.mark.parametrize("B,S,D", [(1, 4096, 2048), (2, 37, 2048), (1, 5, 256), (3, 17, 1024),
                                   (1, 1, 2048), (2, 33, 2040), (2, 33000, 256)])
@pytest.mark.parametrize("has_gz", [True, False])
def test_residual_adaln_bwd_bit_exact(B, S, D, has_gz, cuda_dev):
    r = rng(B * 100 + S + D + has_gz)
    z, x = act(r, (B, S, D)), act(r, (B, S, D))
    gh, gz = act(r, (B, S, D), std=1e-2), act(r, (B, S, D), std=1e-2)
    shift, scale, gate = mods(r, B, D)
    t = lambda a: from_bits(a, cuda_dev)
    dx, dres, dgate, dshift, dscale = torch.ops.anima_flat_b200.residual_adaln_bwd(
        t(gh), t(gz) if has_gz else None, t(z), t(x), t(gate), t(scale), 1e-6)
    o = C.adaln_bwd(gh, z, scale, x=x, gate=gate, gz=gz if has_gz else None)
    np.testing.assert_array_equal(to_bits(dres), o["dz"])
    np.testing.assert_array_equal(to_bits(dx), o["dx"])
    np.testing.assert_array_equal(to_bits(dgate), o["dgate"])
    np.testing.assert_array_equal(to_bits(dshift), o["dshift"])
    np.testing.assert_array_equal(to_bits(dscale), o["dscale"])


@pytest.mark.parametrize("S", [28, 30])
def test_residual_adaln_bwd_many_batch_entries(S, cuda_dev):
    """Short sequences, so that nearly every 28-row chunk starts a new batch
    entry and needs its own scale and gate rows in the modulation slot; five
    calls in a row, bit-exact every time.  Each row-pair group must wait for
    the chunk's modulation rows before reading them, whichever stage carries
    them."""
    B, D = 256, 2048
    r = rng(S + 4242)
    z, x = act(r, (B, S, D)), act(r, (B, S, D))
    gh, gz = act(r, (B, S, D), std=1e-2), act(r, (B, S, D), std=1e-2)
    _, scale, gate = mods(r, B, D)
    t = lambda a: from_bits(a, cuda_dev)
    o = C.adaln_bwd(gh, z, scale, x=x, gate=gate, gz=gz)
    args = [t(gh), t(gz), t(z), t(x), t(gate), t(scale)]
    for _ in range(5):
        dx, dres, dgate, dshift, dscale = torch.ops.anima_flat_b200.residual_adaln_bwd(*args, 1e-6)
        np.testing.assert_array_equal(to_bits(dres), o["dz"])
        np.testing.assert_array_equal(to_bits(dx), o["dx"])
        np.testing.assert_array_equal(to_bits(dgate), o["dgate"])
        np.testing.assert_array_equal(to_bits(dscale), o["dscale"])


@pytest.mark.parametrize("B,S,D", [(1, 4096, 2048), (2, 19, 512)])
def test_adaln_bwd_bit_exact(B, S, D, cuda_dev):
    r = rng(B * 200 + S + D)
    z, gh = act(r, (B, S, D)), act(r, (B, S, D), std=1e-2)
    shift, scale, _ = mods(r, B, D)
    t = lambda a: from_bits(a, cuda_dev)
    dz, dshift, dscale = torch.ops.anima_flat_b200.adaln_bwd(t(gh), t(z), t(scale), 1e-6)
    o = C.adaln_bwd(gh, z, scale)
    np.testing.assert_array_equal(to_bits(dz), o["dz"])
    np.testing.assert_array_equal(to_bits(dshift), o["dshift"])
    np.testing.assert_array_equal(to_bits(dscale), o["dscale"])


@pytest.mark.parametrize("B,S,H,hd", [(1, 4096, 16, 128), (2, 7, 5, 128), (1, 9, 3, 64), (1, 3, 2, 256),
                                      (1, 9000, 2, 64)])
def test_qkv_norm_rope_bwd_bit_exact(B, S, H, hd, cuda_dev):
    r = rng(B + S * 3 + H + hd)
    qkv, qw, kw, cos, sin = qkv_inputs(r, B, S, H, hd)
    dq, dk, dv = (act(r, (B, S, H, hd), std=1e-2) for _ in range(3))
    t = lambda a: from_bits(a, cuda_dev)
    dqkv, dqw, dkw = torch.ops.anima_flat_b200.qkv_norm_rope_bwd(
        t(qkv), t(dq), t(dk), t(dv), t(qw), t(kw), t(cos), t(sin), H, 1e-5)
    o_dqkv, o_dqw, o_dkw = C.qkv_norm_rope_bwd(qkv, dq, dk, dv, qw, kw, cos, sin, H, 1e-5)
    np.testing.assert_array_equal(to_bits(dqkv), o_dqkv)
    np.testing.assert_array_equal(to_bits(dqw).view(np.uint32), o_dqw.view(np.uint32))
    np.testing.assert_array_equal(to_bits(dkw).view(np.uint32), o_dkw.view(np.uint32))


@pytest.mark.parametrize("B,S,H,hd", [(1, 4096, 16, 128), (2, 5, 7, 128), (1, 6, 2, 64), (2, 9000, 2, 64)])
def test_head_norm_bwd_bit_exact(B, S, H, hd, cuda_dev):
    r = rng(B * 5 + S + H + hd)
    x, dy = act(r, (B, S, H * hd)), act(r, (B, S, H, hd), std=1e-2)
    w = (1.0 + r.standard_normal(hd) * 0.02).astype(np.float32)
    t = lambda a: from_bits(a, cuda_dev)
    dx, dw = torch.ops.anima_flat_b200.head_norm_bwd(t(x), t(dy), t(w), H, 1e-5)
    o_dx, o_dw = C.head_norm_bwd(x, dy, w, H, 1e-5)
    np.testing.assert_array_equal(to_bits(dx), o_dx)
    np.testing.assert_array_equal(to_bits(dw).view(np.uint32), o_dw.view(np.uint32))


def test_autograd_through_the_public_functions(cuda_dev):
    """loss.backward() through residual_adaln, qkv_norm_rope (grad mode) and
    head_norm routes to the backward kernels and matches the oracle."""
    r = rng(11)
    B, S, D, H, hd = 1, 64, 2048, 16, 128
    x, res = act(r, (B, S, D)), act(r, (B, S, D))
    shift, scale, gate = mods(r, B, D)
    gh, gz = act(r, (B, S, D), std=1e-2), act(r, (B, S, D), std=1e-2)
    leaf = lambda a: from_bits(a, cuda_dev).requires_grad_(True)
    tx, tres, tgate, tshift, tscale = (leaf(a) for a in (x, res, gate, shift, scale))
    h, z = afb.residual_adaln(tx, tres, tgate, tshift, tscale)
    torch.autograd.backward([h, z], [from_bits(gh, cuda_dev), from_bits(gz, cuda_dev)])
    o = C.adaln_bwd(gh, to_bits(z), scale, x=x, gate=gate, gz=gz)
    np.testing.assert_array_equal(to_bits(tx.grad), o["dx"])
    np.testing.assert_array_equal(to_bits(tres.grad), o["dz"])
    np.testing.assert_array_equal(to_bits(tgate.grad), o["dgate"])
    np.testing.assert_array_equal(to_bits(tshift.grad), o["dshift"])
    np.testing.assert_array_equal(to_bits(tscale.grad), o["dscale"])

    qkv, qw, kw, cos, sin = qkv_inputs(r, B, S, H, hd)
    tq = leaf(qkv)
    tqw, tkw = leaf(qw), leaf(kw)
    q, k, v = afb.qkv_norm_rope(tq, tqw, tkw, from_bits(cos, cuda_dev), from_bits(sin, cuda_dev), H)
    dq, dk, dv = (act(r, (B, S, H, hd), std=1e-2) for _ in range(3))
    torch.autograd.backward([q, k, v], [from_bits(a, cuda_dev) for a in (dq, dk, dv)])
    o_dqkv, o_dqw, o_dkw = C.qkv_norm_rope_bwd(qkv, dq, dk, dv, qw, kw, cos, sin, H, 1e-5)
    np.testing.assert_array_equal(to_bits(tq.grad), o_dqkv)
    np.testing.assert_array_equal(to_bits(tqw.grad).view(np.uint32), o_dqw.view(np.uint32))
    np.testing.assert_array_equal(to_bits(tkw.grad).view(np.uint32), o_dkw.view(np.uint32))


def test_backward_against_torch_autograd_fp32(cuda_dev):
    """Config-4 shapes: kernel gradients vs torch autograd of the fp32
    LayerNorm+modulate composition (fp32 reference, bf16 results): dz within
    2 bf16 ulp at the gradient's scale, parameter gradients within 2 bf16 ulp
    of their magnitude."""
    r = rng(12)
    B, S, D = 1, 4096, 2048
    z, gh = act(r, (B, S, D)), act(r, (B, S, D), std=1e-2)
    shift, scale, _ = mods(r, B, D)
    dz, dshift, dscale = torch.ops.anima_flat_b200.adaln_bwd(
        from_bits(gh, cuda_dev), from_bits(z, cuda_dev), from_bits(scale, cuda_dev), 1e-6)
    zf = from_bits(z, cuda_dev).float().requires_grad_(True)
    scf = from_bits(scale, cuda_dev).float().requires_grad_(True)
    shf = from_bits(shift, cuda_dev).float().requires_grad_(True)
    y = torch.nn.functional.layer_norm(zf, (D,), eps=1e-6) * scf[:, None] + shf[:, None]
    y.backward(from_bits(gh, cuda_dev).float())
    row_scale = zf.grad.abs().amax(-1, keepdim=True)
    assert ((dz.float() - zf.grad).abs() <= 2 * 2.0 ** -8 * row_scale).all()
    for ours, ref in ((dshift, shf.grad), (dscale, scf.grad)):
        assert ((ours.float() - ref).abs() <= 2 * 2.0 ** -8 * ref.abs() + 1e-6 * ref.abs().max()).all()

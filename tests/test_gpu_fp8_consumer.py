"""End-to-end check of the FP8 wire format: our (q, s) fed to torch._scaled_mm
exactly as the reference's fp8_linear does (src/kernels/fp8.py:234-257:
q viewed [B*S, K], the weight's codes transposed, scale_a = s [B*S, 1],
scale_b = the weight's per-row scales [1, N], bf16 out).

For the exact paths (rowquant without GELU, residual_adaln_fp8) our codes and
scales equal the oracle's bit for bit, so the GEMM outputs must be identical.
For GELU the scales are exact and the codes may differ only at e4m3 ties, so
the outputs agree to within a few code steps; both stay within FP8
quantisation error of a bf16 GEMM of gelu(x)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import anima_flat_b200 as afb
from oracle import canonical as C
from tests.conftest import from_bits, to_bits

pytestmark = pytest.mark.gpu


def _weight(N: int, K: int, dev):
    """Per-output-row FP8 weight as the reference's quantize_weight makes it:
    s = amax(|w_row|) / 448, codes = e4m3(w / s)."""
    g = torch.Generator().manual_seed(N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).to(dev)
    s = w.abs().amax(dim=1).clamp_min(1e-12) / 448.0
    q = (w / s[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, s.float(), w


def _scaled_mm(q, s, wq, ws):
    B, S, K = q.shape
    return torch._scaled_mm(q.view(B * S, K), wq.t(), scale_a=s, scale_b=ws.view(1, -1),
                            out_dtype=torch.bfloat16)


def _from_oracle(oq: np.ndarray, os_: np.ndarray, shape, dev):
    q = torch.from_numpy(oq.reshape(shape)).view(torch.float8_e4m3fn).to(dev)
    s = torch.from_numpy(os_.reshape(-1, 1).astype(np.float32)).to(dev)
    return q, s


def _bits(B, S, K, seed, outliers=0.01):
    r = np.random.default_rng(seed)
    a = r.standard_normal((B, S, K), dtype=np.float32)
    a = np.where(r.random((B, S, K)) < outliers, a * 20.0, a)
    return to_bits(torch.from_numpy(a).to(torch.bfloat16))


def _supported(dev) -> bool:
    try:
        q = torch.zeros(16, 16, device=dev).to(torch.float8_e4m3fn)
        one = torch.ones(16, 1, device=dev)
        torch._scaled_mm(q, q.t(), scale_a=one, scale_b=one.view(1, -1), out_dtype=torch.bfloat16)
        return True
    except (RuntimeError, TypeError):
        return False


@pytest.mark.parametrize("K,N", [(2048, 2048), (2048, 6144)])
def test_rowquant_codes_drive_scaled_mm_identically(K, N, cuda_dev):
    if not _supported(cuda_dev):
        pytest.skip("torch._scaled_mm with row-wise scales is not available on this device")
    B, S = 2, 256
    x = _bits(B, S, K, K + N)
    q, s = afb.rowquant(from_bits(x, cuda_dev), gelu=False)
    oq, os_ = C.rowquant(x)
    rq, rs = _from_oracle(oq, os_, (B, S, K), cuda_dev)
    wq, ws, _ = _weight(N, K, cuda_dev)
    ours, ref = _scaled_mm(q, s, wq, ws), _scaled_mm(rq, rs, wq, ws)
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))


def test_residual_adaln_fp8_codes_drive_scaled_mm_identically(cuda_dev):
    if not _supported(cuda_dev):
        pytest.skip("torch._scaled_mm with row-wise scales is not available on this device")
    B, S, D, N = 2, 256, 2048, 2048
    r = np.random.default_rng(11)
    bf = lambda a: to_bits(torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16))
    x, res = _bits(B, S, D, 12), _bits(B, S, D, 13)
    shift = bf(r.standard_normal((B, D)) * 0.1)
    scale = bf(1.0 + r.standard_normal((B, D)) * 0.1)
    gate = bf(r.standard_normal((B, D)) * 0.1)
    q, s, _ = afb.residual_adaln_fp8(*(from_bits(a, cuda_dev) for a in (x, res, gate, shift, scale)))
    o = C.adaln_fwd(res, shift, scale, x=x, gate=gate, fp8=True)
    rq, rs = _from_oracle(o["q"], o["s"], (B, S, D), cuda_dev)
    wq, ws, _ = _weight(N, D, cuda_dev)
    assert torch.equal(_scaled_mm(q, s, wq, ws).view(torch.int16), _scaled_mm(rq, rs, wq, ws).view(torch.int16))


def test_rowquant_gelu_codes_drive_scaled_mm(cuda_dev):
    if not _supported(cuda_dev):
        pytest.skip("torch._scaled_mm with row-wise scales is not available on this device")
    B, S, K, N = 2, 128, 8192, 2048
    x = _bits(B, S, K, 21)
    q, s = afb.rowquant(from_bits(x, cuda_dev), gelu=True)
    oq, os_ = C.rowquant(x, gelu=True)
    rq, rs = _from_oracle(oq, os_, (B, S, K), cuda_dev)
    assert torch.equal(s.view(torch.int32), rs.view(torch.int32))  # exact scales
    wq, ws, w = _weight(N, K, cuda_dev)
    ours = _scaled_mm(q, s, wq, ws).float()
    ref = _scaled_mm(rq, rs, wq, ws).float()
    # Codes may differ at ties only: one e4m3 step on a small fraction of the
    # K terms of each dot product, so the products stay close overall ...
    assert ((ours - ref).norm() / ref.norm()).item() < 5e-3
    # ... and ours tracks the dense product of the canonical GELU exactly as
    # well as the oracle's codes do (FP8 quantisation error of both).
    g = torch.from_numpy(C.gelu(x.reshape(-1)).reshape(B * S, K)).to(cuda_dev)
    dense = g @ (wq.float() * ws[:, None]).t()
    rel_ours = ((ours - dense).norm() / dense.norm()).item()
    rel_ref = ((ref - dense).norm() / dense.norm()).item()
    assert rel_ours < 0.05 and rel_ours <= 1.05 * rel_ref + 1e-4

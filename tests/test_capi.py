"""The C-ABI library and the Python boundary, without launching anything (CPU only)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import anima_flat_b200 as afb
from anima_flat_b200 import _lib
from tests.conftest import ROOT

HEADER_FUNCS = sorted(
    set(re.findall(r"\b(afb_\w+)\s*\(", "\n".join(p.read_text() for p in (ROOT / "include").glob("*.h"))))
)


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.afb_abi_version() == 1
    assert Path(_lib.library_path()).exists()


@pytest.mark.parametrize("name", HEADER_FUNCS)
def test_every_declared_symbol_is_exported(name):
    lib = _lib.load()
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_signature_table_covers_compute_entry_points():
    utility = {"afb_abi_version", "afb_last_error", "afb_clear_error", "afb_set_pdl", "afb_get_pdl",
               "afb_take_device_status",
               "afb_device_status"}
    assert set(HEADER_FUNCS) - utility == set(_lib.SIGNATURES) | set(_lib.WORKSPACE_QUERIES)


def test_workspace_queries():
    lib = _lib.load()
    # [B][chunks of 28 rows][3][D] fp32 (the row scalars stay in shared memory)
    assert lib.afb_residual_adaln_bwd_workspace(1, 4096, 2048) == 1 * 147 * 3 * 2048 * 4
    assert lib.afb_adaln_bwd_workspace(2, 17, 256) == 2 * 1 * 2 * 256 * 4
    # sizes whose workspace does not fit in size_t report SIZE_MAX instead of wrapping
    assert lib.afb_residual_adaln_bwd_workspace(2**62, 2**40, 2048) == 2**64 - 1
    # [chunks of 8 tokens][sections][128] fp32
    assert lib.afb_qkv_norm_rope_bwd_workspace(1, 4096, 16, 128) == 512 * 2 * 128 * 4
    assert lib.afb_head_norm_bwd_workspace(1, 4096, 16, 128) == 512 * 1 * 128 * 4


def test_backward_rejects_small_workspace():
    rc, msg = _status("afb_adaln_bwd", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 32, 2048, 1e-6,
                      FAKE, 16, None)
    assert rc == 1 and "workspace too small" in msg


def _status(name, *args):
    lib = _lib.load()
    rc = getattr(lib, name)(*args)
    return rc, lib.afb_last_error().decode()


FAKE = 4096  # a 16-byte aligned non-null address; validation rejects before any use


def test_rejects_bad_dim_before_launch():
    rc, msg = _status("afb_residual_adaln", *([FAKE] * 7), 1, 4, 2047, 1e-6, None)
    assert rc == 1 and "afb_residual_adaln" in msg and "dim must be" in msg


def test_rejects_null_and_misaligned_pointers():
    rc, msg = _status("afb_adaln", None, FAKE, FAKE, FAKE, 1, 4, 2048, 1e-6, None)
    assert rc == 1 and "z is null" in msg
    rc, msg = _status("afb_adaln", FAKE + 2, FAKE, FAKE, FAKE, 1, 4, 2048, 1e-6, None)
    assert rc == 1 and "not 16-byte aligned" in msg


def test_rejects_bad_head_dim_and_K():
    rc, msg = _status("afb_qkv_norm_rope", *([FAKE] * 7), None, 1, 4, 16, 96, 1e-5, None)
    assert rc == 1 and "head_dim" in msg
    rc, msg = _status("afb_rowquant", FAKE, FAKE, FAKE, 4, 24, 0, None)
    assert rc == 1 and "K must be" in msg
    rc, msg = _status("afb_rowquant", FAKE, FAKE, FAKE, 4, 32768, 1, None)
    assert rc == 1 and "K must be" in msg


def test_ctx_scale_rejects_bad_shapes():
    rc, msg = _status("afb_ctx_scale", FAKE, FAKE, FAKE, FAKE, 1, 4, 16, 96, None)
    assert rc == 1 and "afb_ctx_scale" in msg and "head_dim" in msg
    rc, msg = _status("afb_ctx_scale_bwd", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 4, 32, 128, None)
    assert rc == 1 and "heads * head_dim" in msg
    rc, msg = _status("afb_ctx_scale", FAKE, FAKE + 2, FAKE, FAKE, 1, 4, 16, 128, None)
    assert rc == 1 and "lse is not 4-byte aligned" in msg
    assert _status("afb_ctx_scale", FAKE, FAKE, FAKE, FAKE, 0, 4, 16, 128, None)[0] == 0


def test_ctx_scale_rowquant_rejects_bad_shapes():
    rc, msg = _status("afb_ctx_scale_rowquant", FAKE, FAKE, FAKE, FAKE, FAKE, 1, 4, 16, 96, None)
    assert rc == 1 and "afb_ctx_scale_rowquant" in msg and "head_dim" in msg
    rc, msg = _status("afb_ctx_scale_rowquant", FAKE, FAKE, FAKE, FAKE, FAKE, 1, 4, 256, 128, None)
    assert rc == 1 and "heads * head_dim" in msg
    rc, msg = _status("afb_ctx_scale_rowquant", FAKE, FAKE, FAKE, FAKE, FAKE + 2, 1, 4, 16, 128, None)
    assert rc == 1 and "s is not 4-byte aligned" in msg
    assert _status("afb_ctx_scale_rowquant", FAKE, FAKE, FAKE, FAKE, FAKE, 0, 4, 16, 128, None)[0] == 0


def test_rms_silu_rejects_bad_channels_and_grid():
    rc, msg = _status("afb_rms_silu", FAKE, None, FAKE, None, FAKE, 4, 0, 0, 100, 0, None)
    assert rc == 1 and "afb_rms_silu" in msg and "multiple of 8" in msg
    rc, msg = _status("afb_rms_silu", FAKE, None, FAKE, FAKE, FAKE, 12, 3, 4, 96, 1, None)
    assert rc == 1 and "even output grid" in msg
    # C = 96: 4 lanes per row, 8 rows per tile, 8 tiles per chunk; the chunk
    # doubles once 32768 chunks are exceeded
    assert lib_ws("afb_rms_silu_bwd_workspace", 1024 * 1024, 96) == (1024 * 1024 // 64) * 96 * 4
    assert lib_ws("afb_rms_silu_bwd_workspace", 4096 * 1024, 96) == (4096 * 1024 // 128) * 96 * 4
    rc, msg = _status("afb_rms_silu_bwd", FAKE, FAKE, FAKE, None, FAKE, FAKE, 4096, 0, 0, 96, 0, FAKE, 16, None)
    assert rc == 1 and "workspace too small" in msg


def lib_ws(name, *args):
    return int(getattr(_lib.load(), name)(*args))


def test_empty_inputs_are_a_no_op():
    assert _status("afb_residual_adaln", *([FAKE] * 7), 0, 4, 2048, 1e-6, None)[0] == 0
    assert _status("afb_rowquant", FAKE, FAKE, FAKE, 0, 2048, 1, None)[0] == 0


def test_pdl_switch():
    _lib.set_pdl(False)
    assert _lib.load().afb_get_pdl() == 0
    _lib.set_pdl(True)
    assert _lib.load().afb_get_pdl() == 1


def test_call_raises_runtime_error_with_message():
    with pytest.raises(RuntimeError, match="dim must be"):
        _lib.call("afb_adaln", FAKE, FAKE, FAKE, FAKE, 1, 1, 12, 1e-6, None)


# ----------------------------------------------------------- Python boundary --
def _cpu_args(B=1, S=4, D=2048):
    bf = torch.bfloat16
    return (torch.zeros(B, S, D, dtype=bf), torch.zeros(B, S, D, dtype=bf),
            torch.zeros(B, D, dtype=bf), torch.zeros(B, D, dtype=bf), torch.ones(B, D, dtype=bf))


def test_cpu_tensors_raise_value_error_like_the_reference():
    x, res, gate, shift, scale = _cpu_args()
    with pytest.raises(ValueError, match="CUDA tensors required"):
        afb.residual_adaln(x, res, gate, shift, scale)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        afb.adaln(res, shift, scale)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        afb.rowquant(x)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        afb.head_norm(x.view(1, 4, 2048), torch.ones(128), 16)


@pytest.mark.parametrize(
    "op,args",
    [
        ("residual_adaln", lambda a: a),
        ("residual_adaln_fp8", lambda a: a),
        ("adaln", lambda a: (a[1], a[3], a[4])),
        ("adaln_fp8", lambda a: (a[1], a[3], a[4])),
    ],
)
def test_fake_impls_give_reference_shapes(op, args):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = args(tuple(t.to("meta") for t in _cpu_args(B=2, S=5)))
        out = getattr(torch.ops.anima_flat_b200, op)(*a, 1e-6)
    outs = out if isinstance(out, (tuple, list)) else (out,)
    shapes = [tuple(o.shape) for o in outs]
    if op.endswith("fp8"):
        assert shapes[0] == (2, 5, 2048) and shapes[1] == (10, 1)
        assert outs[0].dtype == torch.float8_e4m3fn and outs[1].dtype == torch.float32
    else:
        assert all(s == (2, 5, 2048) for s in shapes)


def test_fake_impls_rope():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        qkv = torch.empty(2, 6, 3 * 16 * 128, dtype=torch.bfloat16, device="meta")
        w = torch.empty(128, device="meta")
        cs = torch.empty(6, 64, device="meta")
        q, k = torch.ops.anima_flat_b200.qkv_norm_rope(qkv, w, w, cs, cs, 16, 1e-5)
        q2, k2, v2 = torch.ops.anima_flat_b200.qkv_norm_rope_v(qkv, w, w, cs, cs, 16, 1e-5)
        y = torch.ops.anima_flat_b200.head_norm(qkv[..., :2048], w, 16, 1e-5)
        qq, ss = torch.ops.anima_flat_b200.rowquant(qkv[..., :2048], True)
    assert q.shape == k.shape == v2.shape == y.shape == (2, 6, 16, 128)
    assert qq.shape == (2, 6, 2048) and ss.shape == (12, 1)

"""The allocation-free backward entry point, through the C ABI.

afb_residual_adaln_bwd_noalloc serves callers that cannot allocate device
memory (a binding without a device allocator of its own, or a process that
reserves all device memory up front and forbids allocation on the hot path):
it keeps its partial sums in a fixed array inside the library instead of a
caller-provided workspace.  Its outputs must equal those of
afb_residual_adaln_bwd (the workspace entry point) exactly, on two calls in a
row with different inputs, so that nothing left in the shared array from the
first call leaks into the second.  This file is collected last so that a run
stopping at the first failure has already run every other test; it also runs
alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from anima_flat_b200 import _lib
from tests.conftest import from_bits, to_bits

pytestmark = pytest.mark.gpu


def _inputs(seed: int, B: int, S: int, D: int, device):
    r = np.random.default_rng(seed)
    bf = lambda a: from_bits(to_bits(torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)), device)
    return dict(
        gh=bf(r.standard_normal((B, S, D)) * 1e-2),
        gz=bf(r.standard_normal((B, S, D)) * 1e-2),
        z=bf(r.standard_normal((B, S, D))),
        x=bf(r.standard_normal((B, S, D))),
        gate=bf(r.standard_normal((B, D)) * 0.1),
        scale=bf(1.0 + r.standard_normal((B, D)) * 0.1),
    )


def _outputs(t):
    B, S, D = t["z"].shape
    return [torch.empty_like(t["x"]), torch.empty_like(t["z"]), torch.empty_like(t["gate"]),
            torch.empty_like(t["scale"]), torch.empty_like(t["scale"])]


def _ptrs(t, outs):
    return [t["gh"].data_ptr(), t["gz"].data_ptr(), t["z"].data_ptr(), t["x"].data_ptr(),
            t["gate"].data_ptr(), t["scale"].data_ptr()] + [o.data_ptr() for o in outs]


@pytest.mark.parametrize("B,S,D", [(1, 4096, 2048), (2, 37, 1024)])
def test_noalloc_matches_workspace_entry_point_on_two_calls(B, S, D, cuda_dev):
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((101, 202)):
        t = _inputs(seed + B + S, B, S, D, cuda_dev)
        ref = _outputs(t)
        nbytes = int(_lib.load().afb_residual_adaln_bwd_workspace(B, S, D))
        ws = torch.empty(max(1, nbytes // 4), dtype=torch.float32, device=cuda_dev)
        _lib.call("afb_residual_adaln_bwd", *_ptrs(t, ref), B, S, D, 1e-6, ws.data_ptr(), nbytes,
                  stream)
        got = _outputs(t)
        _lib.call("afb_residual_adaln_bwd_noalloc", *_ptrs(t, got), B, S, D, 1e-6, stream)
        torch.cuda.synchronize()
        for name, a, b in zip(("dx", "dres", "dgate", "dshift", "dscale"), got, ref):
            assert torch.equal(a, b), f"call {call}: {name} differs from the workspace entry point"


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_dev):
    # a valid backward shape whose scratch does not fit:
    # 16 * 4096/32 * 3 * 2048 * 4 bytes = 48 MiB > 16 MiB
    lib = _lib.load()
    rc = lib.afb_residual_adaln_bwd_noalloc(*([16] * 11), 16, 4096, 2048, 1e-6, None)
    assert rc == 1
    assert "more than the" in lib.afb_last_error().decode()
    # sizes whose scratch does not even fit in size_t are rejected the same way
    rc = lib.afb_residual_adaln_bwd_noalloc(*([16] * 11), 2**62, 2**40, 2048, 1e-6, None)
    assert rc == 1
    assert "more than the" in lib.afb_last_error().decode()

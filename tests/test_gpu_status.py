"""After the GPU parity tests: no bounded wait in any kernel ever gave up."""

from __future__ import annotations

import ctypes

import pytest
import torch

from anima_flat_b200 import _lib

pytestmark = pytest.mark.gpu


def test_device_status_clean(cuda_dev):
    torch.cuda.synchronize()
    lib = _lib.load()
    status = ctypes.c_int(-1)
    assert lib.afb_device_status(ctypes.byref(status)) == 0
    assert status.value == 0

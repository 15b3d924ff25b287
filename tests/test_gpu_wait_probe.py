"""The give-up branch of the bounded waits, run on purpose without a fault.

Every kernel waits on its bulk copies with mbar_wait, which gives up after a
bounded number of try_wait rounds, sets the device status word, and lets the
kernel drain its copies in flight and return.  afb_wait_probe takes that
branch: it waits, with a short limit, on an mbarrier that nothing arrives on,
while a real bulk copy is in flight on another.  The test checks that the
wait gave up, that the copy was drained, that the status word reports the
timeout, and that afb_take_device_status reports it once and clears it.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from anima_flat_b200 import _lib

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1  # kStatusWaitTimeout


def _status(take: bool) -> int:
    lib = _lib.load()
    v = ctypes.c_int(-1)
    fn = lib.afb_take_device_status if take else lib.afb_device_status
    assert fn(ctypes.byref(v)) == 0, lib.afb_last_error().decode()
    return v.value


@pytest.mark.parametrize("spins", [1, 64, 512])
def test_bounded_wait_gives_up_and_drains(spins, cuda_dev):
    torch.cuda.synchronize()
    before = _status(take=False)
    result = torch.full((2,), -1, dtype=torch.int32, device=cuda_dev)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("afb_wait_probe", spins, result.data_ptr(), stream)
    torch.cuda.synchronize()  # the kernel returned: the give-up path ends
    assert result.tolist() == [1, 1]
    assert _status(take=False) & WAIT_TIMEOUT
    # reported once, then cleared (the words of the other files included)
    assert _status(take=True) & WAIT_TIMEOUT
    assert _status(take=False) == 0
    assert before == 0, "a kernel's bounded wait gave up before this test"
    # the context stays usable: an ordinary launch still works
    x = torch.ones(4, device=cuda_dev)
    assert float((x * 2).sum()) == 8.0

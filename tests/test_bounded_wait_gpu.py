"""A wait that runs out (B200): the bounded mbarrier wait every kernel uses, on a barrier nothing
completes, gives up after its limit, reports RW4_DEVERR_TIMEOUT through the device status word and
returns; the context stays usable.  Nothing traps, faults or hangs."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_reports_and_returns(cuda):
    from rocketllm_b200 import _lib, kernels
    kernels.device_status(clear=True)
    _lib.call("rw4_wait_selftest", 1, kernels._stream())      # the phase completes: no report
    assert kernels.device_status(clear=True) == 0
    t0 = time.monotonic()
    _lib.call("rw4_wait_selftest", 0, kernels._stream())      # nothing arrives
    word = kernels.device_status(clear=True)                  # synchronises
    elapsed = time.monotonic() - t0
    assert word & 1, word
    assert 0.9 < elapsed < 30, elapsed
    assert kernels.device_status() == 0                       # cleared
    x = torch.ones(4, device=cuda)                            # the context still works
    assert float((x * 2).sum()) == 8.0

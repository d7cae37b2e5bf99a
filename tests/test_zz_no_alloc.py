"""rw4_linear_noalloc, the GEMV entry point that allocates nothing, through the C ABI.

It exists for callers that cannot allocate device memory per call: a host that plans every byte of
VRAM up front, or a C caller without an allocator to hand a workspace from.  Its scratch is a fixed
array in the library's device image, shared by every call and never cleared, so the GPU test makes
two calls in a row (the second finds the first call's leftovers) and checks each against the
ordinary entry point (rw4_linear_ws with a torch-allocated workspace) within the tolerance of
tests/test_linear_gpu.py.  The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from rocketllm_b200 import _lib, kernels
from rocketllm_b200.synthetic import make_activation, make_weight


def within_tolerance(y, ref):
    """|y - ref| <= |ref| / 128 + 2e-3 * rms(ref): one bf16 rounding plus accumulation-order noise."""
    y, ref = y.float().cpu().numpy(), ref.float().cpu().numpy()
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-12
    err = np.abs(y - ref)
    bound = np.abs(ref) / 128 + 2e-3 * rms
    assert np.all(err <= bound), f"max err {err.max():.4g}, worst excess {(err - bound).max():.4g}"


def noalloc(x, packed, scale, zero, out):
    m, k = x.shape
    _lib.call("rw4_linear_noalloc", x.data_ptr(), m, k, packed.data_ptr(), scale.data_ptr(),
              zero.data_ptr(), packed.shape[0], 64, out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n", [(1, 4096, 4096), (3, 4096, 4096), (16, 14336, 4096),
                                   (40, 8192, 1024), (1, 53248, 16384), (64, 16384, 512)])
def test_noalloc_matches_linear_on_two_calls_in_a_row(cuda, m, k, n):
    packed, scale, zero = make_weight(n, k, device=cuda, seed=m + k)
    for call in range(2):
        x = make_activation(m, k, device=cuda, seed=100 * call + m)
        if call:
            x = (x.float() * 1e-3).to(torch.bfloat16)  # a different row exponent on the second call
        y = noalloc(x, packed, scale, zero, torch.empty(m, n, dtype=torch.bfloat16, device=cuda))
        ref = kernels.linear(x, packed, scale, zero)
        torch.cuda.synchronize()
        assert kernels.device_status() == 0
        within_tolerance(y, ref)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """Checked on the host before any device call (the pointers are never dereferenced)."""
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    assert lib.rw4_linear_noalloc(p, 65, 4096, p, p, p, 4096, 64, p, None) == _lib.RW4_EINVAL
    assert "at most 64 rows" in _lib.last_error()
    assert lib.rw4_linear_noalloc(p, 64, 53248, p, p, p, 4096, 64, p, None) == _lib.RW4_EINVAL
    assert "scratch" in _lib.last_error()

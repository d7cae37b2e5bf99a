"""The C-ABI library: it loads, exports every symbol include/rw4.h declares, and rejects bad
arguments before launching anything (these calls need no GPU)."""
import ctypes
import os
import re

import pytest

from rocketllm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "rw4.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rw4_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert "rw4_linear" in names and "rw4_xfer_send" in names and "rw4_moe_grouped" in names
    missing = [n for n in names if getattr(lib, n, None) is None]
    assert not missing, f"declared in rw4.h but not exported: {missing}"
    assert set(names) <= set(_lib.SIGNATURES), "ctypes signatures out of sync with rw4.h"


def test_version_and_path_selection():
    lib = _lib.lib()
    assert lib.rw4_version() >= 100
    assert lib.rw4_linear_path(1, 4096, 4096) == 1
    assert lib.rw4_linear_path(16, 4096, 4096) == 1
    assert lib.rw4_linear_path(64, 4096, 4096) in (2, 3)
    assert lib.rw4_linear_path(1, 100, 4096) == _lib.RW4_EINVAL


def test_invalid_arguments_are_rejected_before_launch():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    st = lib.rw4_linear(p, 1, 4096, p, p, p, 4096, 32, p, None)
    assert st == _lib.RW4_EINVAL
    assert "group" in _lib.last_error()
    st = lib.rw4_linear(p, 1, 100, p, p, p, 4096, 64, p, None)
    assert st == _lib.RW4_EINVAL and "multiple of 64" in _lib.last_error()
    st = lib.rw4_linear(ctypes.c_void_p(258), 1, 4096, p, p, p, 4096, 64, p, None)
    assert st == _lib.RW4_EINVAL and "aligned" in _lib.last_error()
    assert lib.rw4_dequant(p, p, p, 4, 64, 3, p, 1, None) == _lib.RW4_EINVAL
    assert lib.rw4_quantize(p, 7, 4, 64, 64, p, p, p, None) == _lib.RW4_EINVAL


def test_errors_raise_with_message():
    with pytest.raises(_lib.RW4Error, match="RW4_EINVAL"):
        _lib.call("rw4_linear", 256, 1, 4096, 256, 256, 256, 4096, 32, 256, None)


def test_kv_and_expert_routing_entry_points_reject_bad_arguments():
    """The int4-KV attention and device-side expert routing entry points validate shapes, counts
    and pointers on the host, before any device call."""
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    kv = lib.rw4_kv_attention_decode
    # 6 query heads over 4 kv heads
    assert kv(p, 0, 0, 1, 6, 4, 128, p, p, p, p, 1, 1, p, p, 64, 1, 1.0, p, 0, 0, None) \
        == _lib.RW4_EINVAL
    # head_dim 96 and 32 query heads per kv head are not built
    assert kv(p, 0, 0, 1, 8, 2, 96, p, p, p, p, 1, 1, p, p, 64, 1, 1.0, p, 0, 0, None) \
        == _lib.RW4_EUNSUPPORTED
    assert kv(p, 0, 0, 1, 64, 2, 128, p, p, p, p, 1, 1, p, p, 64, 1, 1.0, p, 0, 0, None) \
        == _lib.RW4_EUNSUPPORTED
    # more groups than the capacity, more window tokens than the window, nothing at all
    assert kv(p, 0, 0, 1, 8, 2, 128, p, p, p, p, 1, 2, p, p, 64, 1, 1.0, p, 0, 0, None) \
        == _lib.RW4_EINVAL
    assert kv(p, 0, 0, 1, 8, 2, 128, p, p, p, p, 1, 1, p, p, 64, 65, 1.0, p, 0, 0, None) \
        == _lib.RW4_EINVAL
    assert kv(p, 0, 0, 1, 8, 2, 128, p, p, p, p, 1, 0, p, p, 64, 0, 1.0, p, 0, 0, None) \
        == _lib.RW4_EINVAL
    # misaligned packed storage
    odd = ctypes.c_void_p(264)
    assert kv(p, 0, 0, 1, 8, 2, 128, odd, p, p, p, 1, 1, p, p, 64, 1, 1.0, p, 0, 0, None) \
        == _lib.RW4_EINVAL

    out = ctypes.c_void_p()
    arr = (ctypes.c_void_p * 1)(256)
    assert lib.rw4_slot_maps_create(arr, arr, arr, 0, 4096, 2048, 1, ctypes.byref(out)) \
        == _lib.RW4_EINVAL                                    # no slots
    assert lib.rw4_slot_maps_create(arr, arr, arr, 81, 4096, 2048, 1, ctypes.byref(out)) \
        == _lib.RW4_EINVAL                                    # more than fit the parameters
    assert lib.rw4_slot_maps_create(arr, arr, arr, 1, 4000, 2048, 1, ctypes.byref(out)) \
        == _lib.RW4_EINVAL                                    # K % 512
    assert out.value is None
    assert lib.rw4_moe_grouped_slots(p, p, 8, 1, None, p, p, None) == _lib.RW4_EINVAL
    assert lib.rw4_expert_residency(p, 0, 0, p, p, p, 8, p, p, p, p, p, p, None) \
        == _lib.RW4_EINVAL
    lfu = lib.rw4_expert_residency_lfu
    assert lfu(p, 8, 3, 24, p, p, 8, p, p, p, 4096, p, p, p, p, p, None) \
        == _lib.RW4_EINVAL                                    # layer 3 of a 3-layer table
    assert lfu(p, 8, 0, 24, p, p, 8, p, p, p, 0, p, p, p, p, p, None) \
        == _lib.RW4_EINVAL                                    # aging interval 0
    assert lfu(p, 8, 0, 24, p, p, 8, None, p, p, 4096, p, p, p, p, p, None) \
        == _lib.RW4_EINVAL                                    # no count table
    # a blob larger than a slot, a blob that is not whole 16-byte vectors
    assert lib.rw4_expert_copy(p, p, p, 0, 8, p, 1 << 21, p, 1 << 20, 4, 8, None) \
        == _lib.RW4_EINVAL
    assert lib.rw4_expert_copy(p, p, p, 0, 8, p, 1000, p, 1 << 20, 4, 8, None) \
        == _lib.RW4_EINVAL
    dev = ctypes.c_void_p()
    assert lib.rw4_host_ptr_device(None, ctypes.byref(dev)) == _lib.RW4_EINVAL


def test_ring_rejects_bad_arguments_before_touching_the_device():
    lib = _lib.lib()
    out = ctypes.c_void_p()
    assert lib.rw4_ring_create(0, 2, 1, ctypes.byref(out)) == _lib.RW4_EINVAL
    assert lib.rw4_ring_create(1 << 20, 0, 1, ctypes.byref(out)) == _lib.RW4_EINVAL
    assert lib.rw4_ring_create(1 << 20, 65, 1, ctypes.byref(out)) == _lib.RW4_EINVAL
    assert lib.rw4_ring_create(1 << 20, 2, 9, ctypes.byref(out)) == _lib.RW4_EINVAL
    assert lib.rw4_ring_create(1 << 20, 2, 1, None) == _lib.RW4_EINVAL
    assert out.value is None
    assert lib.rw4_ring_stage(None, 0, 0, None, 0) == _lib.RW4_EINVAL
    assert lib.rw4_ring_submit(None, 0, None, 0, None) == _lib.RW4_EINVAL
    assert lib.rw4_ring_wait_compute(None, None) == _lib.RW4_EINVAL
    assert lib.rw4_ring_destroy(None) == _lib.RW4_OK

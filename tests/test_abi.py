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

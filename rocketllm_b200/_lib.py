"""Loader for ``librw4.so``, the RW4 C-ABI library, and the ctypes signatures of its entry points.

There is no fallback: if the library is missing or fails to load, every caller gets a
``RuntimeError`` telling it how to build the library.  Nothing in this package computes the hot
path any other way.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librw4.so")

RW4_OK = 0
RW4_EINVAL = -1
RW4_ECUDA = -2
RW4_ENOMEM = -3
RW4_ETIMEOUT = -4
RW4_EBUSY = -5
RW4_EUNSUPPORTED = -6

RW4_F32 = 0
RW4_BF16 = 1
RW4_F16 = 2

_ERRNAMES = {RW4_EINVAL: "RW4_EINVAL", RW4_ECUDA: "RW4_ECUDA", RW4_ENOMEM: "RW4_ENOMEM",
             RW4_ETIMEOUT: "RW4_ETIMEOUT", RW4_EBUSY: "RW4_EBUSY",
             RW4_EUNSUPPORTED: "RW4_EUNSUPPORTED"}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/rw4.h
SIGNATURES = {
    "rw4_version": (ctypes.c_int, []),
    "rw4_last_error": (ctypes.c_int, [ctypes.c_char_p, _size]),
    "rw4_dequant": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, _c_void_p,
                                   _i32, _c_void_p]),
    "rw4_quantize": (ctypes.c_int, [_c_void_p, _i32, _i64, _i64, _i32, _c_void_p, _c_void_p,
                                    _c_void_p, _c_void_p]),
    "rw4_linear": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64,
                                  _i32, _c_void_p, _c_void_p]),
    "rw4_linear_path": (ctypes.c_int, [_i64, _i64, _i64]),
    "rw4_linear_on_path": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p,
                                          _i64, _i32, _c_void_p, _i32, _c_void_p]),
    "rw4_linear_workspace_size": (ctypes.c_int, [_i64, _i64, _i64, _i32,
                                                 ctypes.POINTER(_size)]),
    "rw4_linear_ws": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64,
                                     _i32, _c_void_p, _i32, _c_void_p, _size, _c_void_p]),
    "rw4_linear_noalloc": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p,
                                          _i64, _i32, _c_void_p, _c_void_p]),
    "rw4_rmsnorm": (ctypes.c_int, [_c_void_p, _c_void_p, _i64, _i64, ctypes.c_float, _c_void_p,
                                   _c_void_p]),
    "rw4_rope_kv": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32,
                                   _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p,
                                   _c_void_p, _c_void_p]),
    "rw4_silu_mul": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p]),
    "rw4_linear_rmsnorm_workspace_size": (ctypes.c_int, [_i64, _i64, _i64,
                                                         ctypes.POINTER(_size)]),
    "rw4_linear_rmsnorm_ws": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, ctypes.c_float,
                                             _c_void_p, _c_void_p, _c_void_p, _i64, _i32,
                                             _c_void_p, _c_void_p, _size, _c_void_p]),
    "rw4_linear_rmsnorm_swiglu_workspace_size": (ctypes.c_int, [_i64, _i64, _i64,
                                                                ctypes.POINTER(_size)]),
    "rw4_linear_rmsnorm_swiglu_ws": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p,
                                                    ctypes.c_float, _c_void_p, _c_void_p,
                                                    _c_void_p, _i64, _i32, _c_void_p, _c_void_p,
                                                    _size, _c_void_p]),
    "rw4_decode_attention": (ctypes.c_int, [_c_void_p, _i32, _i32, _i32, _i32, _c_void_p,
                                            _c_void_p, _i64, _c_void_p, ctypes.c_float,
                                            _c_void_p, _c_void_p]),
    "rw4_linear_residual_ws": (ctypes.c_int, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p,
                                              _c_void_p, _i64, _i32, _c_void_p, _c_void_p,
                                              _c_void_p, _size, _c_void_p]),
    "rw4_argmax_rows": (ctypes.c_int, [_c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p]),
    "rw4_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _i32, _c_void_p]),
    "rw4_wait_selftest": (ctypes.c_int, [_i32, _c_void_p]),
    "rw4_moe_permute": (ctypes.c_int, [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p,
                                       _c_void_p, _c_void_p]),
    "rw4_moe_gather": (ctypes.c_int, [_c_void_p, _c_void_p, _i64, _i32, _i64, _c_void_p,
                                      _c_void_p]),
    "rw4_moe_grouped": (ctypes.c_int, [_c_void_p, _c_void_p, _i32, _i64, _c_void_p, _c_void_p,
                                       _c_void_p, _i64, _i64, _i32, _i32, _c_void_p, _c_void_p]),
    "rw4_moe_combine": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64,
                                       _i32, _i64, _c_void_p, _c_void_p]),
    "rw4_slot_maps_create": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i32, _i64, _i64,
                                            _i32, ctypes.POINTER(_c_void_p)]),
    "rw4_slot_maps_destroy": (ctypes.c_int, [_c_void_p]),
    "rw4_moe_grouped_slots": (ctypes.c_int, [_c_void_p, _c_void_p, _i32, _i64, _c_void_p,
                                             _c_void_p, _c_void_p, _c_void_p]),
    "rw4_expert_residency": (ctypes.c_int, [_c_void_p, _i32, _i32, _c_void_p, _c_void_p,
                                            _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p,
                                            _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "rw4_expert_residency_lfu": (ctypes.c_int, [_c_void_p, _i32, _i32, _i32, _c_void_p,
                                                _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p,
                                                _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                                _c_void_p, _c_void_p]),
    "rw4_expert_residency_lfu_host": (ctypes.c_int, [_c_void_p, _i32, _i32, _i32, _c_void_p,
                                                     _c_void_p, _i32, _c_void_p, _c_void_p,
                                                     _c_void_p, _i64, _c_void_p, _c_void_p,
                                                     _c_void_p, _c_void_p, _c_void_p]),
    "rw4_expert_copy": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p,
                                       _i64, _c_void_p, _i64, _i32, _i32, _c_void_p]),
    "rw4_host_ptr_device": (ctypes.c_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "rw4_kv_attention": (ctypes.c_int, [_c_void_p, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                                        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                                        _c_void_p, _c_void_p, _i64, _i64, ctypes.c_float,
                                        _c_void_p, _i64, _i64, _i64, _c_void_p]),
    "rw4_kv_attention_decode": (ctypes.c_int, [_c_void_p, _i64, _i64, _i32, _i32, _i32, _i32,
                                               _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64,
                                               _i64, _c_void_p, _c_void_p, _i64, _i64,
                                               ctypes.c_float, _c_void_p, _i64, _i64, _c_void_p]),
    "rw4_ring_create": (ctypes.c_int, [_size, _i32, _i32, ctypes.POINTER(_c_void_p)]),
    "rw4_ring_destroy": (ctypes.c_int, [_c_void_p]),
    "rw4_ring_slot": (ctypes.c_int, [_c_void_p, _i32, ctypes.POINTER(_c_void_p)]),
    "rw4_ring_stage": (ctypes.c_int, [_c_void_p, _i32, _size, _c_void_p, _size]),
    "rw4_ring_submit": (ctypes.c_int, [_c_void_p, _i32, _c_void_p, _size, _c_void_p]),
    "rw4_ring_wait_compute": (ctypes.c_int, [_c_void_p, _c_void_p]),
    "rw4_pool_create": (ctypes.c_int, [_size, ctypes.POINTER(_c_void_p)]),
    "rw4_pool_destroy": (ctypes.c_int, [_c_void_p]),
    "rw4_pool_lease": (ctypes.c_int, [_c_void_p, _size, ctypes.POINTER(_i32),
                                      ctypes.POINTER(_c_void_p)]),
    "rw4_pool_release": (ctypes.c_int, [_c_void_p, _i32]),
    "rw4_pool_stats": (ctypes.c_int, [_c_void_p, ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                      ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64)]),
    "rw4_xfer_create": (ctypes.c_int, [_i32, _i32, ctypes.POINTER(_c_void_p)]),
    "rw4_xfer_destroy": (ctypes.c_int, [_c_void_p]),
    "rw4_xfer_send": (ctypes.c_int, [_c_void_p, _c_void_p, _c_void_p, _size, _size, _c_void_p,
                                     ctypes.POINTER(ctypes.c_uint64)]),
    "rw4_xfer_wait": (ctypes.c_int, [_c_void_p, ctypes.c_uint64, _c_void_p]),
    "rw4_xfer_query": (ctypes.c_int, [_c_void_p, ctypes.c_uint64]),
    "rw4_xfer_sync": (ctypes.c_int, [_c_void_p, ctypes.c_uint64, _i64]),
    "rw4_xfer_stats": (ctypes.c_int, [_c_void_p, ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_i32)]),
}

_lib = None
_lock = threading.Lock()


class RW4Error(RuntimeError):
    """A failed RW4 C-ABI call; ``status`` is the negative RW4_E* code."""

    def __init__(self, what, status, message):
        self.status = status
        super().__init__(f"{what} failed with {_ERRNAMES.get(status, status)}: {message}")


def lib():
    """The loaded library, with argument types declared.  Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing; build it with `python -m rocketllm_b200.csrc.build` "
                    f"(nvcc, sm_100a). There is no non-CUDA path for RW4 weights.")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def last_error():
    buf = ctypes.create_string_buffer(1024)
    lib().rw4_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status, what):
    """Raise :class:`RW4Error` for a non-zero status; return ``status`` otherwise."""
    if status < 0:
        raise RW4Error(what, status, last_error())
    return status


def call(name, *args):
    """Call entry point ``name`` and raise on a negative status."""
    return check(getattr(lib(), name)(*args), name)

"""Torch-tensor front end of the RW4 C ABI: device pointers and the current stream in, no copies.

Each function validates that its tensors live on a CUDA device with the layout the C ABI expects
and calls the matching ``rw4_*`` entry point on ``torch.cuda.current_stream()``.  Shapes follow
RocketLLM's int4 codec (``rocketllm/quant/kv_cache.py:190-272``) applied to a Linear weight
``W[N, K]``: ``packed`` uint8 ``[N, Kp/2]``, ``scale``/``zero`` fp16 ``[N, Kp/64]``.
"""
import ctypes

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.RW4_F32, torch.bfloat16: _lib.RW4_BF16,
               torch.float16: _lib.RW4_F16}


def _stream():
    return ctypes_stream(torch.cuda.current_stream())


def ctypes_stream(stream):
    return stream.cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("RW4 kernels take CUDA tensors only (there is no CPU path); got a "
                             f"{t.device} tensor of shape {tuple(t.shape)}")
        if not t.is_contiguous():
            raise ValueError(f"RW4 kernels need contiguous tensors; got strides {t.stride()}")


def _check_weight(packed, scale, zero):
    if packed.dtype != torch.uint8:
        raise TypeError(f"packed must be uint8, not {packed.dtype}")
    if scale.dtype != torch.float16 or zero.dtype != torch.float16:
        raise TypeError("scale and zero must be float16")
    if packed.dim() != 2 or scale.shape != zero.shape or scale.shape[0] != packed.shape[0]:
        raise ValueError(f"inconsistent RW4 weight: packed {tuple(packed.shape)}, scale "
                         f"{tuple(scale.shape)}, zero {tuple(zero.shape)}")


def dequantize(packed, scale, zero, k=None, dtype=torch.bfloat16, out=None):
    """Expand an RW4 weight to ``[N, k]`` in ``dtype``; bit-exact with the reference codec."""
    _require_cuda(packed, scale, zero)
    _check_weight(packed, scale, zero)
    n = packed.shape[0]
    kp = packed.shape[1] * 2
    k = kp if k is None else int(k)
    group = kp // scale.shape[1] if scale.shape[1] else 64
    if out is None:
        out = torch.empty((n, k), dtype=dtype, device=packed.device)
    _require_cuda(out)
    _lib.call("rw4_dequant", packed.data_ptr(), scale.data_ptr(), zero.data_ptr(), n, k, group,
              out.data_ptr(), _DTYPE_CODE[out.dtype], _stream())
    return out


def quantize(w, group=64):
    """Encode ``w[N, K]`` (fp32, bf16 or fp16, CUDA) as ``(packed, scale, zero, padding)``.

    Bit-exact with the reference ``quantize(w, 1, group)``, whose scale arithmetic runs in the
    tensor's own dtype.
    """
    _require_cuda(w)
    if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"quantize takes float32, bfloat16 or float16, not {w.dtype}")
    n, k = w.shape
    g = min(group, k) if k else group
    groups = (k + g - 1) // g if k else 0
    packed = torch.empty((n, groups * g // 2), dtype=torch.uint8, device=w.device)
    scale = torch.empty((n, groups), dtype=torch.float16, device=w.device)
    zero = torch.empty((n, groups), dtype=torch.float16, device=w.device)
    _lib.call("rw4_quantize", w.data_ptr(), _DTYPE_CODE[w.dtype], n, k, group, packed.data_ptr(),
              scale.data_ptr(), zero.data_ptr(), _stream())
    return packed, scale, zero, groups * g - k


_WS_BYTES = {}


def linear_workspace_bytes(m, k, n, path=0):
    """Device workspace bytes ``rw4_linear_ws`` needs for this call (0 for the tensor-core GEMM and
    for one row that the GEMV converts itself)."""
    key = (m, k, n, path)
    b = _WS_BYTES.get(key)
    if b is None:
        v = ctypes.c_size_t()
        _lib.call("rw4_linear_workspace_size", m, k, n, path, ctypes.byref(v))
        b = _WS_BYTES[key] = v.value
    return b


def linear(x, packed, scale, zero, out=None, path=None):
    """``y = x . W^T`` with ``x`` bf16 ``[..., K]`` and W in RW4; returns bf16 ``[..., N]``.

    ``x`` may be a strided view (e.g. the last position of every sequence); it is compacted first.
    ``path`` forces a kernel (1 / 3 GEMV, 2 tcgen05 GEMM, 4 tcgen05 decode GEMM for 17-64 rows)
    instead of the library's choice.  The
    GEMV's workspace (the converted activations) comes from torch's allocator on the current
    stream, so the call also works inside a CUDA-graph capture.
    """
    if not x.is_cuda:
        raise ValueError("RW4 kernels take CUDA tensors only (there is no CPU path); got a "
                         f"{x.device} activation")
    _require_cuda(packed, scale, zero)
    _check_weight(packed, scale, zero)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"rw4 linear takes bf16 activations, not {x.dtype}")
    k = x.shape[-1]
    n = packed.shape[0]
    if packed.shape[1] * 2 != k:
        raise ValueError(f"x has K={k} but the weight packs {packed.shape[1] * 2} values per row")
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m = x2.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], n), dtype=torch.bfloat16, device=x.device)
    p = 0 if path is None else int(path)
    wsb = linear_workspace_bytes(m, k, n, p) if m and n else 0
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device) if wsb else None
    _lib.call("rw4_linear_ws", x2.data_ptr(), m, k, packed.data_ptr(), scale.data_ptr(),
              zero.data_ptr(), n, 64, out.data_ptr(), p, ws.data_ptr() if ws is not None else None,
              wsb, _stream())
    return out


def linear_path(m, k, n):
    """Which kernel :func:`linear` launches: 1 GEMV, 2 tcgen05 GEMM, 3 GEMV slices, 4 tcgen05
    decode GEMM (17-64 rows)."""
    return _lib.check(_lib.lib().rw4_linear_path(m, k, n), "rw4_linear_path")


def device_status(clear=True):
    """The library's device status word (bit 1: a bounded wait timed out). Synchronises."""
    word = ctypes.c_uint32()
    _lib.call("rw4_device_status", ctypes.byref(word), int(clear), _stream())
    return word.value


# ---- routed experts ------------------------------------------------------------------------------

def argmax_rows(scores, out=None):
    """Greedy choice per row of bf16 ``scores [R, V]`` (``rw4_argmax_rows``): int64 ``[R, 1]``, the
    first index among equal maxima, NaN above every number -- ``scores.argmax(-1, keepdim=True)``.
    Rows may be a strided view (unit stride along V)."""
    if not scores.is_cuda:
        raise ValueError(f"RW4 kernels take CUDA tensors only; got a {scores.device} tensor")
    if scores.dtype != torch.bfloat16 or scores.dim() != 2 or scores.stride(1) != 1:
        raise TypeError("scores must be a 2-D bf16 tensor with unit stride along V")
    r, v = scores.shape
    if out is None:
        out = torch.empty(r, 1, dtype=torch.int64, device=scores.device)
    _lib.call("rw4_argmax_rows", scores.data_ptr(), r, v, scores.stride(0), out.data_ptr(),
              _stream())
    return out


def moe_permute(topk_idx, num_experts):
    """``(perm, inv, offsets)`` int32 for ``topk_idx`` int64 ``[T, k]`` (stable, by expert)."""
    _require_cuda(topk_idx)
    if topk_idx.dtype != torch.int64:
        raise TypeError("topk_idx must be int64")
    t, k = topk_idx.shape
    dev = topk_idx.device
    perm = torch.empty(t * k, dtype=torch.int32, device=dev)
    inv = torch.empty(t * k, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    _lib.call("rw4_moe_permute", topk_idx.data_ptr(), t, k, num_experts, perm.data_ptr(),
              inv.data_ptr(), offsets.data_ptr(), _stream())
    return perm, inv, offsets


def moe_gather(x, perm, k):
    """``x_perm[row] = x[perm[row] // k]`` for bf16 ``x [T, H]``."""
    _require_cuda(x, perm)
    t, h = x.shape
    out = torch.empty((perm.numel(), h), dtype=x.dtype, device=x.device)
    _lib.call("rw4_moe_gather", x.data_ptr(), perm.data_ptr(), t, k, h, out.data_ptr(), _stream())
    return out


def moe_grouped(x_perm, offsets, weights, act=0, max_rows=None, out=None):
    """Grouped RW4 GEMV over routed experts.

    ``weights`` is a list of ``(packed, scale, zero)`` per expert (all ``[N, K]``); ``act=1`` treats
    them as stacked gate/up (``N = 2I``) and returns the SwiGLU activation ``[rows, I]``.
    """
    _require_cuda(x_perm, offsets)
    e = len(weights)
    n = weights[0][0].shape[0]
    k = x_perm.shape[1]
    rows = x_perm.shape[0]
    n_out = n // 2 if act == 1 else n
    if out is None:
        out = torch.empty((rows, n_out), dtype=torch.bfloat16, device=x_perm.device)
    ptrs = [(ctypes.c_void_p * e)(*[w[i].data_ptr() for w in weights]) for i in range(3)]
    _lib.call("rw4_moe_grouped", x_perm.data_ptr(), offsets.data_ptr(), e,
              rows if max_rows is None else int(max_rows), ptrs[0], ptrs[1], ptrs[2], k, n, 64,
              int(act), out.data_ptr(), _stream())
    return out


def moe_combine(y_perm, inv, topk_idx, topk_w, out=None):
    """Weighted combine of expert rows back to tokens, bf16 ``[T, H]``."""
    _require_cuda(y_perm, inv, topk_w)
    t, k = topk_w.shape
    h = y_perm.shape[1]
    if out is None:
        out = torch.empty((t, h), dtype=torch.bfloat16, device=y_perm.device)
    wd = {torch.float32: _lib.RW4_F32, torch.bfloat16: _lib.RW4_BF16}[topk_w.dtype]
    _lib.call("rw4_moe_combine", y_perm.data_ptr(), inv.data_ptr(),
              topk_idx.data_ptr() if topk_idx is not None else None, topk_w.data_ptr(), wd, t, k,
              h, out.data_ptr(), _stream())
    return out


# ---- int4 KV cache attention ------------------------------------------------------------------

def kv_attention_decode(query, k_codes, k_sz, v_codes, v_sz, groups, k_res, v_res, res_len,
                        scaling, out=None):
    """Attention of ``q_len`` query positions over an int4 KV cache (``rw4_kv_attention``): the
    queries are the window's last ``q_len`` tokens and attend causally (``q_len = 1``: a decode
    step).

    ``query`` bf16 ``[b, h, q_len, d]`` (any strides with a unit last stride).  The cache arrays are
    the layouts ``include/rw4.h`` documents: ``k_codes [b, kvh, gcap, d, 32]``, ``k_sz [b, kvh,
    gcap, d, 2]`` f16, ``v_codes [b, kvh, gcap*64, d/2]``, ``v_sz [b, kvh, gcap*64, d/64, 2]`` f16,
    ``k_res`` / ``v_res`` bf16 ``[b, kvh, rcap, d]``; ``groups`` and ``res_len`` say how much of
    each is valid.  Returns bf16 ``[b, q_len, h, d]`` (the layout transformers' attention
    returns).
    """
    _require_cuda(k_codes, k_sz, v_codes, v_sz, k_res, v_res)
    if not query.is_cuda or query.dtype != torch.bfloat16 or query.stride(-1) != 1:
        raise ValueError("query must be a CUDA bf16 tensor with unit last stride")
    b, h, q_len, d = query.shape
    kvh, gcap = k_codes.shape[1], k_codes.shape[2]
    rcap = k_res.shape[2]
    if out is None:
        out = torch.empty((b, q_len, h, d), dtype=torch.bfloat16, device=query.device)
    _lib.call("rw4_kv_attention", query.data_ptr(), query.stride(0), query.stride(1),
              query.stride(2), b, h, kvh, d, q_len, k_codes.data_ptr(), k_sz.data_ptr(),
              v_codes.data_ptr(), v_sz.data_ptr(), gcap, int(groups), k_res.data_ptr(),
              v_res.data_ptr(), rcap, int(res_len), float(scaling), out.data_ptr(),
              out.stride(0), out.stride(2), out.stride(1), _stream())
    return out


# ---- device-side routing into the expert cache ---------------------------------------------------

class SlotMaps:
    """Tensor maps of every slot of a device expert cache for one projection (``[N, K]`` RW4
    weights at per-slot device addresses), encoded once (``rw4_slot_maps_create``)."""

    def __init__(self, packed_ptrs, scale_ptrs, zero_ptrs, k, n, act):
        s = len(packed_ptrs)
        arrs = [(ctypes.c_void_p * s)(*p) for p in (packed_ptrs, scale_ptrs, zero_ptrs)]
        handle = ctypes.c_void_p()
        _lib.call("rw4_slot_maps_create", arrs[0], arrs[1], arrs[2], s, int(k), int(n), int(act),
                  ctypes.byref(handle))
        self.handle, self.slots, self.k, self.n, self.act = handle, s, int(k), int(n), int(act)

    def close(self):
        if self.handle:
            _lib.call("rw4_slot_maps_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def moe_grouped_slots(x_perm, offsets, maps, slot_of, max_rows=None, out=None):
    """Grouped RW4 GEMV where routed expert ``e`` reads the weight in slot ``slot_of[e]``."""
    _require_cuda(x_perm, offsets, slot_of)
    rows = x_perm.shape[0]
    n_out = maps.n // 2 if maps.act == 1 else maps.n
    if out is None:
        out = torch.empty((rows, n_out), dtype=torch.bfloat16, device=x_perm.device)
    _lib.call("rw4_moe_grouped_slots", x_perm.data_ptr(), offsets.data_ptr(),
              offsets.numel() - 1, rows if max_rows is None else int(max_rows), maps.handle,
              slot_of.data_ptr(), out.data_ptr(), _stream())
    return out


def expert_residency(offsets, layer, where, owner, stamp, clock, slot_of, copy_expert, copy_slot,
                     ncopy, counters):
    """Device-side residency step of one MoE layer (``rw4_expert_residency``)."""
    _require_cuda(offsets, where, owner, stamp, clock, slot_of, copy_expert, copy_slot, ncopy,
                  counters)
    _lib.call("rw4_expert_residency", offsets.data_ptr(), offsets.numel() - 1, int(layer),
              where.data_ptr(), owner.data_ptr(), stamp.data_ptr(), owner.numel(),
              clock.data_ptr(), slot_of.data_ptr(), copy_expert.data_ptr(), copy_slot.data_ptr(),
              ncopy.data_ptr(), counters.data_ptr(), _stream())


def expert_residency_lfu(offsets, layer, where, owner, uses, admitted, state, aging_interval,
                         slot_of, copy_expert, copy_slot, ncopy, counters):
    """Device-side residency step of one MoE layer under LFU with aging
    (``rw4_expert_residency_lfu``); ``uses`` float64, ``state`` int64 [3]."""
    _require_cuda(offsets, where, owner, uses, admitted, state, slot_of, copy_expert, copy_slot,
                  ncopy, counters)
    if uses.dtype != torch.float64 or state.dtype != torch.int64 or state.numel() != 3:
        raise TypeError("uses must be float64 and state int64 [3]")
    _lib.call("rw4_expert_residency_lfu", offsets.data_ptr(), offsets.numel() - 1, int(layer),
              where.numel(), where.data_ptr(), owner.data_ptr(), owner.numel(), uses.data_ptr(),
              admitted.data_ptr(), state.data_ptr(), int(aging_interval), slot_of.data_ptr(),
              copy_expert.data_ptr(), copy_slot.data_ptr(), ncopy.data_ptr(), counters.data_ptr(),
              _stream())


def expert_copy(copy_expert, copy_slot, ncopy, layer, num_experts, host_blobs, blob_bytes, slots,
                slot_bytes, ctas_per_expert=64):
    """Copy the listed experts' mapped host blobs into their slots (``rw4_expert_copy``)."""
    _lib.call("rw4_expert_copy", copy_expert.data_ptr(), copy_slot.data_ptr(), ncopy.data_ptr(),
              int(layer), int(num_experts), host_blobs.data_ptr(), int(blob_bytes),
              slots.data_ptr(), int(slot_bytes), slots.numel() // int(slot_bytes),
              int(ctas_per_expert), _stream())


def host_ptr_device(ptr):
    """The device-visible address of pinned host memory at ``ptr`` (raises if it is not mapped)."""
    out = ctypes.c_void_p()
    _lib.call("rw4_host_ptr_device", ctypes.c_void_p(ptr), ctypes.byref(out))
    return out.value

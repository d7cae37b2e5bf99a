"""Device-routed expert streaming (``DeviceExpertStreamer``, LFU policy) driven on the CPU.

The residency step is the library's own: the call ``kernels.expert_residency_lfu`` makes is
redirected to ``rw4_expert_residency_lfu_host``, the same compiled step on host tables, with the
very arguments the wrapper marshals.  The other device kernels are restated in torch (the copy
kernel copies the listed blobs into their slots; the slot-indexed grouped GEMV reads each routed
expert's weights at the slot addresses its tensor maps were built from), pinning is the identity.
Every layer call must give exactly the output of the same arithmetic over the module's own
weights, and the slot table must follow :class:`ExpertSlotCache` with whole-set protection.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import rw4_oracle as o
from rocketllm_b200 import _lib, expert_stream, kernels
from test_expert_stream_cpu import (E, H, INTER, LAYERS, TOP_K, _combine, _direct, _Experts,
                                    _gather, _permute)


def _raw(ptr, shape, dtype):
    n = int(np.prod(shape)) * np.dtype(dtype).itemsize
    buf = (ctypes.c_uint8 * n).from_address(ptr)
    return np.frombuffer(buf, dtype=np.uint8).view(dtype).reshape(shape).copy()


class _Maps:
    def __init__(self, packed_ptrs, scale_ptrs, zero_ptrs, k, n, act):
        self.ptrs = list(zip(packed_ptrs, scale_ptrs, zero_ptrs))
        self.k, self.n, self.act = int(k), int(n), int(act)

    def close(self):
        pass


def _grouped_slots(xp, offsets, maps, slot_of, max_rows=None):
    n, k = maps.n, maps.k
    out = torch.zeros(xp.shape[0], n // 2 if maps.act == 1 else n)
    for e in range(offsets.numel() - 1):
        a, b = int(offsets[e]), int(offsets[e + 1])
        if a == b:
            continue
        p, s, z = maps.ptrs[int(slot_of[e])]
        w = o.dequantize(_raw(p, (n, k // 2), np.uint8), _raw(s, (n, k // 64), np.float16),
                         _raw(z, (n, k // 64), np.float16))
        y = xp[a:b].float() @ torch.from_numpy(w).T
        if maps.act == 1:
            y = torch.nn.functional.silu(y[:, :n // 2]) * y[:, n // 2:]
        out[a:b] = y
    return out.to(torch.bfloat16)


def _copy(blobs_by_ptr):
    def copy(ce, cs, nc, layer, n_exp, host_ptrs, blob_bytes, slots, slot_bytes, ctas=64):
        for i in range(int(nc[0])):
            e, s = int(ce[i]), int(cs[i])
            host = blobs_by_ptr[int(host_ptrs[layer * n_exp + e])]
            slots[s * slot_bytes:s * slot_bytes + blob_bytes].copy_(host[:blob_bytes])
    return copy


@pytest.mark.parametrize("slots,aging", [(E, 4096), (8, 5), (11, 3)])
def test_device_routed_lfu_streaming_on_host_tables(monkeypatch, slots, aging):
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self, *a, **k: self)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: None)
    monkeypatch.setattr(kernels, "_require_cuda", lambda *tensors: None)
    monkeypatch.setattr(kernels, "_stream", lambda: None)
    monkeypatch.setattr(kernels, "host_ptr_device", lambda ptr: ptr)
    monkeypatch.setattr(kernels, "SlotMaps", _Maps)
    real_call = _lib.call

    def call(name, *args):
        if name == "rw4_expert_residency_lfu":       # the same step on host tables
            assert args[-1] is None
            return real_call("rw4_expert_residency_lfu_host", *args[:-1])
        return real_call(name, *args)

    monkeypatch.setattr(_lib, "call", call)
    for name, fn in (("moe_permute", _permute), ("moe_gather", _gather),
                     ("moe_grouped_slots", _grouped_slots), ("moe_combine", _combine)):
        monkeypatch.setattr(kernels, name, fn)

    modules = [_Experts(20 + i) for i in range(LAYERS)]
    copies = [_Experts(20 + i) for i in range(LAYERS)]
    st = expert_stream.DeviceExpertStreamer(list(enumerate(modules)), "cpu", slots,
                                            policy="lfu", aging_interval=aging)
    monkeypatch.setattr(kernels, "expert_copy",
                        _copy({b.host.data_ptr(): b.host for b in st.blobs}))
    cache = expert_stream.ExpertSlotCache(slots, "lfu", aging)
    rng = np.random.default_rng(slots * 7 + aging)
    popular = [rng.permutation(E) for _ in range(LAYERS)]
    p = 1.0 / np.arange(1, E + 1) ** 1.2
    p /= p.sum()
    for call_i in range(36):
        layer = int(rng.integers(0, LAYERS))
        t = int(rng.integers(1, 4))
        x = torch.randn(t, H, generator=torch.Generator().manual_seed(call_i)).to(torch.bfloat16)
        idx = torch.tensor(np.stack([rng.choice(popular[layer], TOP_K, replace=False, p=p)
                                     for _ in range(t)]), dtype=torch.int64)
        w = torch.softmax(torch.randn(t, TOP_K, generator=torch.Generator().manual_seed(call_i)),
                          -1)
        got = modules[layer](x, idx, w)
        assert torch.equal(got, _direct(copies[layer], x, idx, w)), call_i
        routed = sorted(set(idx.reshape(-1).tolist()))
        for e in routed:
            cache.claim((layer, e), {(layer, r) for r in routed})
        assert st.owner.tolist() == [-1 if k is None else k[0] * E + k[1] for k in cache.owner]
    stats = st.stats()
    assert stats["policy"] == "lfu" and stats["agings"] == cache.agings
    assert stats["fetches"] + stats["hits"] == cache.accesses
    assert st.uses.tolist() == [cache.uses.get((k // E, k % E), 0.0) for k in range(LAYERS * E)]

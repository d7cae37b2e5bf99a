"""Host-routed expert streaming on the CPU: ``ExpertStreamer`` and ``streamed_experts_forward``.

The device kernels of the experts path (permute, gather, grouped RW4 GEMV, combine) are replaced by
torch restatements over the oracle (``oracle.moe_permute`` / ``dequantize``), the copy engine by a
fake that copies at once, pinning by the identity.  What runs for real is the streamer: the
per-expert blobs, the slot cache with its LFU eviction under whole-set protection, the sends into
the slots and the per-expert weight views the grouped GEMV is handed.  With far fewer slots than
experts, every layer call must give exactly the output of the same arithmetic over the module's
own (never streamed) weights.
"""
import numpy as np
import pytest
import torch

from oracle import rw4_oracle as o
from rocketllm_b200 import expert_stream

H, INTER, E, LAYERS, TOP_K = 64, 64, 6, 3, 2


class _Experts(torch.nn.Module):
    """A stacked-experts module in RW4 form (the parameters the RW4 experts function reads)."""

    rw4 = True

    def __init__(self, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        for name, n, k in (("gate_up_proj", 2 * INTER, H), ("down_proj", H, INTER)):
            packed = torch.randint(0, 256, (E, n, k // 2), dtype=torch.uint8, generator=g)
            scale = (0.005 + 0.015 * torch.rand(E, n, k // 64, generator=g)).to(torch.float16)
            zero = (-8.0 * scale.float()).to(torch.float16)
            for sfx, t in (("_packed", packed), ("_scale", scale), ("_zero_point", zero)):
                self.register_parameter(name + sfx, torch.nn.Parameter(t, requires_grad=False))


def _dequant(triple):
    p, s, z = (t.contiguous().numpy() for t in triple)
    return torch.from_numpy(o.dequantize(p, s, z))


def _permute(idx, n_exp):
    perm, offsets = o.moe_permute(idx.numpy(), n_exp)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.shape[0], dtype=perm.dtype)
    return torch.from_numpy(perm), torch.from_numpy(inv), torch.from_numpy(offsets)


def _gather(x, perm, k):
    return x[perm.long() // k]


def _grouped(xp, offsets, weights, act=0, max_rows=None):
    n = weights[0][0].shape[0]
    out = torch.zeros(xp.shape[0], n // 2 if act == 1 else n)
    for e in range(len(weights)):
        a, b = int(offsets[e]), int(offsets[e + 1])
        if a == b:
            continue                              # an expert no row routed to is never read
        y = xp[a:b].float() @ _dequant(weights[e]).T
        if act == 1:
            y = torch.nn.functional.silu(y[:, :n // 2]) * y[:, n // 2:]
        out[a:b] = y
    return out.to(torch.bfloat16)


def _combine(yp, inv, idx, w):
    t, k = w.shape
    rows = inv.long().view(t, k)
    out = (w.float()[..., None] * yp.float()[rows]).sum(1)
    return out.to(torch.bfloat16)


class _Handle:
    def resolve(self, stream=None):
        return None


class _CopyAtOnce:
    def __init__(self):
        self.sends = 0

    def send_buffer(self, host, lease=None, out=None, after=None):
        out.copy_(host.view(-1)[:out.numel()])
        self.sends += 1
        return _Handle()


def _direct(module_copy, x, idx, w):
    """The same arithmetic over the module's own stacked weights (nothing streamed)."""
    perm, inv, offsets = _permute(idx, E)
    xp = _gather(x, perm, TOP_K)
    triples = {name: [tuple(getattr(module_copy, name + sfx)[e]
                            for sfx in ("_packed", "_scale", "_zero_point")) for e in range(E)]
               for name in ("gate_up_proj", "down_proj")}
    act = _grouped(xp, offsets, triples["gate_up_proj"], act=1)
    yp = _grouped(act, offsets, triples["down_proj"], act=0)
    return _combine(yp, inv, idx, w)


@pytest.mark.parametrize("slots,policy,aging", [(E, "lfu", 4096), (8, "lfu", 5), (8, "lru", 4096),
                                                (LAYERS * E, "lfu", 3)])
def test_streamed_experts_give_the_modules_own_output(monkeypatch, slots, policy, aging):
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self, *a, **k: self)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: None)
    for name, fn in (("moe_permute", _permute), ("moe_gather", _gather),
                     ("moe_grouped", _grouped), ("moe_combine", _combine)):
        monkeypatch.setattr(expert_stream.kernels, name, fn)
    modules = [_Experts(10 + i) for i in range(LAYERS)]
    copies = [_Experts(10 + i) for i in range(LAYERS)]          # the same weights, kept whole
    xfer = _CopyAtOnce()
    st = expert_stream.ExpertStreamer(list(enumerate(modules)), "cpu", slots, xfer,
                                      policy=policy, aging_interval=aging)
    assert all(m.gate_up_proj_packed.shape[0] == 0 for m in modules)   # weights left the modules
    rng = np.random.default_rng(slots + aging)
    popular = [rng.permutation(E) for _ in range(LAYERS)]
    for call in range(40):
        layer = call % LAYERS
        t = int(rng.integers(1, 4))
        x = torch.randn(t, H, generator=torch.Generator().manual_seed(call)).to(torch.bfloat16)
        p = 1.0 / np.arange(1, E + 1) ** 1.3
        p /= p.sum()
        idx = torch.tensor(np.stack([rng.choice(popular[layer], TOP_K, replace=False, p=p)
                                     for _ in range(t)]), dtype=torch.int64)
        w = torch.softmax(torch.randn(t, TOP_K, generator=torch.Generator().manual_seed(99 + call)),
                          -1)
        got = modules[layer](x, idx, w)
        want = _direct(copies[layer], x, idx, w)
        assert torch.equal(got, want), (call, layer)
    stats = st.stats()
    assert stats["fetches"] == xfer.sends and stats["resident"] <= slots
    assert stats["policy"] == policy and stats["routing"]["firings"] == 40
    if slots < LAYERS * E:
        assert stats["fetches"] > stats["resident"]             # slots were recycled
    else:
        assert stats["fetches"] == stats["resident"]            # each expert crossed once

"""Modules that hold RW4 weights and compute on them through the C ABI.

``RW4Linear`` replaces ``nn.Linear`` (what transformers' attention / MLP / lm_head forwards call,
e.g. transformers ``models/llama/modeling_llama.py:171-184``); ``rw4_experts_forward`` replaces the
stacked-expert forward of ``MixtralExperts`` (``models/mixtral/modeling_mixtral.py:62-98``) through
transformers' experts-implementation registry.  Parameter names follow the checkpoint's companion
suffixes (``weight_packed`` / ``weight_scale`` / ``weight_zero_point``), so a pre-quantized shard
loads into them by name.  There is no CPU path: a forward on a non-CUDA tensor raises.
"""
import types

import torch
from torch import nn

from .. import kernels

GROUP = 64


def _param(shape, dtype, device):
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class RW4Linear(nn.Module):
    """``y = x W^T (+ b)`` with ``W [out, in]`` stored as RW4 (group 64)."""

    def __init__(self, in_features, out_features, bias=False, device=None, dtype=torch.bfloat16):
        super().__init__()
        if in_features % GROUP:
            raise ValueError(f"RW4Linear needs in_features % {GROUP} == 0, got {in_features}")
        self.in_features = in_features
        self.out_features = out_features
        self.weight_packed = _param((out_features, in_features // 2), torch.uint8, device)
        self.weight_scale = _param((out_features, in_features // GROUP), torch.float16, device)
        self.weight_zero_point = _param((out_features, in_features // GROUP), torch.float16,
                                        device)
        self.bias = _param((out_features,), dtype, device) if bias else None

    @classmethod
    def from_linear(cls, linear, device=None):
        return cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                   device=device if device is not None else linear.weight.device,
                   dtype=linear.weight.dtype if linear.weight.is_floating_point()
                   else torch.bfloat16)

    def forward(self, x):
        dtype = x.dtype
        xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        y = kernels.linear(xb, self.weight_packed, self.weight_scale, self.weight_zero_point)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y if dtype == torch.bfloat16 else y.to(dtype)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, rw4 group {GROUP}")


def rw4_experts_params(experts, device=None):
    """Swap a stacked-experts module's dense ``gate_up_proj [E, 2I, H]`` / ``down_proj [E, H, I]``
    for their RW4 triples (``*_packed`` / ``*_scale`` / ``*_zero_point``)."""
    for name in ("gate_up_proj", "down_proj"):
        dense = getattr(experts, name)
        e, n, k = dense.shape
        if k % GROUP:
            raise ValueError(f"{name}: K={k} is not a multiple of {GROUP}")
        dev = device if device is not None else dense.device
        del experts._parameters[name]
        # An empty, non-persistent stand-in keeps code that initialises the dense weight by name
        # (transformers' _init_weights) working, without a state-dict entry.
        experts.register_buffer(name, torch.empty(0, device=dev), persistent=False)
        experts.register_parameter(f"{name}_packed", _param((e, n, k // 2), torch.uint8, dev))
        experts.register_parameter(f"{name}_scale", _param((e, n, k // GROUP), torch.float16, dev))
        experts.register_parameter(f"{name}_zero_point",
                                   _param((e, n, k // GROUP), torch.float16, dev))
    experts.rw4 = True
    # Bound on the instance: transformers may re-resolve config._experts_implementation after the
    # quantizer ran, and the stock forwards read the dense parameters this module no longer has.
    experts.forward = types.MethodType(rw4_experts_forward, experts)
    return experts


def _expert_triples(experts, name):
    p = getattr(experts, f"{name}_packed")
    s = getattr(experts, f"{name}_scale")
    z = getattr(experts, f"{name}_zero_point")
    return [(p[e], s[e], z[e]) for e in range(p.shape[0])]


def rw4_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """Routed experts on RW4 weights: permute -> gather -> grouped gate/up with fused SwiGLU ->
    grouped down -> ordered weighted combine.  Signature of transformers' experts interface
    (``integrations/moe.py:432-455``): ``(hidden [T, H], top_k_index [T, k], top_k_weights [T, k])``.
    Experts no token routed to are never read."""
    t, h = hidden_states.shape
    k = top_k_index.shape[1]
    x = hidden_states if hidden_states.dtype == torch.bfloat16 else hidden_states.to(torch.bfloat16)
    if not x.is_contiguous():
        x = x.contiguous()
    idx = top_k_index.to(torch.int64).contiguous()
    w = top_k_weights.contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    n_exp = getattr(self, "num_experts", None) or self.gate_up_proj_packed.shape[0]
    perm, inv, offsets = kernels.moe_permute(idx, n_exp)
    # rows per expert: a token's top-k experts are distinct, so every expert gets at most one row
    # per token (known on the host: no device read)
    rows = t
    xp = kernels.moe_gather(x, perm, k)
    act = kernels.moe_grouped(xp, offsets, _expert_triples(self, "gate_up_proj"), act=1,
                              max_rows=rows)
    yp = kernels.moe_grouped(act, offsets, _expert_triples(self, "down_proj"), act=0,
                             max_rows=rows)
    out = kernels.moe_combine(yp, inv, idx, w)
    return out if hidden_states.dtype == torch.bfloat16 else out.to(hidden_states.dtype)

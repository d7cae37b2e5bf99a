"""One-time conversion of a dense transformers model to an RW4 checkpoint.

Every ``nn.Linear`` weight (and stacked-expert weight) is encoded with ``rw4_quantize`` -- bit-exact
with the reference ``quantize(W, axis=1, group_size=64)`` (``rocketllm/quant/kv_cache.py:190-221``)
-- and stored under the companion-suffix names the RW4 backend groups (``X.weight_packed``,
``X.weight_scale``, ``X.weight_zero_point``); everything else (embeddings, norms, routers, biases) is
kept as it is.  The checkpoint's ``config.json`` declares ``quantization_config = {"quant_method":
"rw4", ...}``, which is what selects the RW4 backend and quantizer at load.
"""
import json
import os

import torch
from torch import nn

from .. import kernels
from .hf import QUANT_METHOD, RW4Config, _is_stacked_experts


def _quantize(w, device):
    w = w.detach().to(device)
    if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        w = w.float()
    packed, scale, zero, padding = kernels.quantize(w.contiguous(), 64)
    if padding:
        raise ValueError("RW4 Linear weights need in_features % 64 == 0")
    return packed.cpu(), scale.cpu(), zero.cpu()


def quantize_state_dict(model, device="cuda", modules_to_not_convert=()):
    """``(state_dict, quantization_config)`` of ``model`` with every Linear / experts weight in RW4."""
    sd = {}
    handled = set()
    skip = tuple(modules_to_not_convert)
    for name, module in model.named_modules():
        if any(name == s or name.endswith("." + s) for s in skip):
            continue
        if isinstance(module, nn.Linear):
            p, s, z = _quantize(module.weight, device)
            sd[f"{name}.weight_packed"], sd[f"{name}.weight_scale"] = p, s
            sd[f"{name}.weight_zero_point"] = z
            handled.add(f"{name}.weight")
        elif _is_stacked_experts(module):
            for wname in ("gate_up_proj", "down_proj"):
                dense = getattr(module, wname)
                parts = [_quantize(dense[e], device) for e in range(dense.shape[0])]
                for i, suffix in enumerate(("_packed", "_scale", "_zero_point")):
                    sd[f"{name}.{wname}{suffix}"] = torch.stack([t[i] for t in parts])
                handled.add(f"{name}.{wname}")
    for pname, param in model.state_dict().items():
        if pname not in handled and pname not in sd:
            sd[pname] = param.detach().cpu()
    return sd, RW4Config(modules_to_not_convert=list(skip)).to_dict()


def save_rw4_checkpoint(model, path, device="cuda", modules_to_not_convert=()):
    """Write ``config.json`` + ``model.safetensors`` of the RW4-encoded ``model`` to ``path``."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    sd, qcfg = quantize_state_dict(model, device, modules_to_not_convert)
    # tied embeddings share storage with lm_head in some models; safetensors refuses aliases
    seen = {}
    for k, v in list(sd.items()):
        key = (v.data_ptr(), v.numel()) if v.numel() else None
        if key is not None and key in seen:
            sd[k] = v.clone()
        elif key is not None:
            seen[key] = k
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(path, "model.safetensors"),
              metadata={"format": "pt"})
    cfg = model.config.to_dict()
    cfg["quantization_config"] = qcfg
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path


__all__ = ["quantize_state_dict", "save_rw4_checkpoint", "QUANT_METHOD"]

"""transformers integration: the ``rw4`` quantization config, its quantizer and experts function.

RocketLLM builds every model on the meta device and, when the checkpoint declares a
``quantization_config``, calls ``AutoHfQuantizer.from_config(...).preprocess_model(...)``
(``rocketllm/base.py:680-690``) -- the hook through which a format swaps ``nn.Linear`` for its own
module before any weight is read.  Registering ``rw4`` here makes that path (and plain
``AutoModelForCausalLM.from_pretrained``) build ``RW4Linear`` modules whose parameters are the
checkpoint's packed tensors, placed verbatim (``param_needs_quantization`` is False, so the engine's
coalesced placement copies them as stored, ``rocketllm/quant/registry.py:486-501``).

Stacked-expert modules (``MixtralExperts`` style: ``gate_up_proj [E, 2I, H]``, ``down_proj
[E, H, I]``) get RW4 triples for both weights and the model's experts implementation is pointed at
``rw4`` in transformers' ``ALL_EXPERTS_FUNCTIONS`` (``integrations/moe.py:432-515``).
"""
import torch
from torch import nn
from transformers.integrations.moe import ALL_EXPERTS_FUNCTIONS
from transformers.quantizers.auto import (AUTO_QUANTIZATION_CONFIG_MAPPING, AUTO_QUANTIZER_MAPPING,
                                          register_quantization_config, register_quantizer)
from transformers.quantizers.base import HfQuantizer
from transformers.utils.quantization_config import QuantizationConfigMixin

from .modules import RW4Linear, rw4_experts_forward, rw4_experts_params

QUANT_METHOD = "rw4"


class RW4Config(QuantizationConfigMixin):
    """``{"quant_method": "rw4", "bits": 4, "group_size": 64, "modules_to_not_convert": [...]}``."""

    def __init__(self, bits=4, group_size=64, modules_to_not_convert=None, **kwargs):
        if bits != 4 or group_size != 64:
            raise ValueError(f"rw4 is 4-bit with group 64, got bits={bits} group={group_size}")
        self.quant_method = QUANT_METHOD
        self.bits = bits
        self.group_size = group_size
        self.modules_to_not_convert = list(modules_to_not_convert or [])

    def to_dict(self):
        return {"quant_method": QUANT_METHOD, "bits": self.bits, "group_size": self.group_size,
                "modules_to_not_convert": list(self.modules_to_not_convert)}


def _is_stacked_experts(module):
    gu = getattr(module, "gate_up_proj", None)
    dn = getattr(module, "down_proj", None)
    return (isinstance(gu, nn.Parameter) and isinstance(dn, nn.Parameter) and gu.dim() == 3
            and dn.dim() == 3)


def convert_modules(model, modules_to_not_convert=()):
    """Replace every ``nn.Linear`` (and stacked-experts weight) not excluded by name with its RW4
    counterpart, on whatever device the skeleton lives (normally meta).  Returns the converted
    names."""
    converted = []
    skip = tuple(modules_to_not_convert)
    for name, module in list(model.named_modules()):
        if any(name == s or name.endswith("." + s) or name.startswith(s + ".") for s in skip):
            continue
        if isinstance(module, nn.Linear):
            parent_name, _, leaf = name.rpartition(".")
            parent = model.get_submodule(parent_name) if parent_name else model
            setattr(parent, leaf, RW4Linear.from_linear(module))
            converted.append(name)
        elif _is_stacked_experts(module):
            rw4_experts_params(module)
            converted.append(name)
    if any(getattr(m, "rw4", False) for m in model.modules()):
        model.config._experts_implementation = QUANT_METHOD
    return converted


class RW4HfQuantizer(HfQuantizer):
    """Pre-quantized RW4 checkpoints only; packed tensors load verbatim into RW4 modules."""

    requires_calibration = True

    def validate_environment(self, *args, **kwargs):
        return

    def update_dtype(self, dtype):
        return torch.bfloat16 if dtype is None else dtype

    def param_needs_quantization(self, model, param_name, **kwargs):
        return False

    def _process_model_before_weight_loading(self, model, **kwargs):
        convert_modules(model, self.quantization_config.modules_to_not_convert)
        return model

    def _process_model_after_weight_loading(self, model, **kwargs):
        return model

    @property
    def is_serializable(self):
        return True

    @property
    def is_trainable(self):
        return False


def register():
    """Register config, quantizer and experts function with transformers (idempotent)."""
    if QUANT_METHOD not in AUTO_QUANTIZATION_CONFIG_MAPPING:
        register_quantization_config(QUANT_METHOD)(RW4Config)
    if QUANT_METHOD not in AUTO_QUANTIZER_MAPPING:
        register_quantizer(QUANT_METHOD)(RW4HfQuantizer)
    ALL_EXPERTS_FUNCTIONS._global_mapping[QUANT_METHOD] = rw4_experts_forward


register()

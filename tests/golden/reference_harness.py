"""Run the reference's own RocketLLM code (imported from its source tree) in this process.

Test infrastructure for the fixture scripts beside it and for the CPU tests that exercise the
reference-side integration; it needs the reference's source tree (``RW4_REFERENCE_ROOT``, default
``/root/reference``) and is never imported by the package, ``bench.py`` or a GPU test.

Two things the reference imports are not installed here and are stood in for:

* ``accelerate`` (``rocketllm/base.py:12-13``, ``rocketllm/quant/registry.py:23``): only
  ``init_empty_weights`` and ``accelerate.utils.modeling.set_module_tensor_to_device`` are used.
  :func:`install_accelerate_standin` provides both, written from their documented behaviour: the
  first makes parameters registered inside it land on the meta device (buffers stay real unless
  ``include_buffers``); the second puts a value (or the current tensor) for one named parameter or
  buffer on a device, casting a floating value to ``dtype`` -- or, with no ``dtype``, to the
  existing parameter's dtype, the behaviour the reference's ``_move_coalesced`` comment describes
  (``rocketllm/base.py:982-986``) -- and never casting a non-float value.
* a quantizer for the ``rw4`` checkpoint format.  :func:`register_dequant_rw4` registers, in
  transformers, a quantizer that gives every ``nn.Linear`` homes for ``weight_packed`` /
  ``weight_scale`` / ``weight_zero_point`` (so the reference's loader keeps those tensors), and, in
  the reference's own registry (``register_backend``, ``rocketllm/quant/registry.py:634-638``), a
  ``QuantBackend`` whose ``prepare_layer`` -- the reference's dequant-to-scratch seam
  (``rocketllm/base.py:848-855``) -- expands each triple with the reference's codec
  ``QuantizedTensor.dequantize`` (``rocketllm/quant/kv_cache.py:249-257``) into ``X.weight`` in the
  compute dtype.  The model then runs the stock ``nn.Linear`` over those weights: the reference's
  CPU path for a packed checkpoint.
"""
import contextlib
import importlib.machinery
import os
import sys
import types
from collections import OrderedDict

import torch

REFERENCE_ROOT = os.environ.get("RW4_REFERENCE_ROOT", "/root/reference")


def reference_available():
    return os.path.isfile(os.path.join(REFERENCE_ROOT, "rocketllm", "base.py"))


@contextlib.contextmanager
def _init_empty_weights(include_buffers=False):
    module_cls = torch.nn.Module
    register_parameter = module_cls.register_parameter
    register_buffer = module_cls.register_buffer

    def parameter_on_meta(module, name, param):
        register_parameter(module, name, param)
        p = module._parameters.get(name)
        if p is not None and p.device.type != "meta":
            module._parameters[name] = torch.nn.Parameter(p.detach().to("meta"),
                                                          requires_grad=p.requires_grad)

    def buffer_on_meta(module, name, tensor, persistent=True):
        if tensor is not None:
            tensor = tensor.to("meta")
        register_buffer(module, name, tensor, persistent=persistent)

    module_cls.register_parameter = parameter_on_meta
    if include_buffers:
        module_cls.register_buffer = buffer_on_meta
    try:
        yield
    finally:
        module_cls.register_parameter = register_parameter
        module_cls.register_buffer = register_buffer


def _set_module_tensor_to_device(module, tensor_name, device, value=None, dtype=None, **_):
    owner = module
    path = tensor_name.split(".")
    for part in path[:-1]:
        owner = getattr(owner, part)
    leaf = path[-1]
    is_param = leaf in owner._parameters
    if not is_param and leaf not in owner._buffers:
        raise ValueError(f"{type(owner).__name__} has no parameter or buffer named {leaf!r} "
                         f"({tensor_name})")
    old = owner._parameters[leaf] if is_param else owner._buffers[leaf]
    if value is None:
        if old is None or old.device.type == "meta" and str(device) != "meta":
            raise ValueError(f"{tensor_name} is on meta; a value is needed to place it")
        value = old
    if value.is_floating_point():
        if dtype is not None:
            value = value.to(dtype)
        elif old is not None and old.is_floating_point():
            value = value.to(old.dtype)
    value = value.to(device)
    if is_param:
        owner._parameters[leaf] = torch.nn.Parameter(
            value, requires_grad=bool(old is not None and old.requires_grad
                                      and value.is_floating_point()))
    else:
        owner._buffers[leaf] = value


def install_accelerate_standin():
    """Put the stand-in ``accelerate`` modules in ``sys.modules`` (after transformers is imported,
    so its own probe for accelerate still finds none)."""
    import transformers  # noqa: F401 - must see the real (absent) accelerate first
    import transformers.modeling_utils  # noqa: F401
    if "accelerate" in sys.modules:
        return
    acc = types.ModuleType("accelerate")
    utils = types.ModuleType("accelerate.utils")
    modeling = types.ModuleType("accelerate.utils.modeling")
    for m in (acc, utils, modeling):
        m.__spec__ = importlib.machinery.ModuleSpec(m.__name__, None)
    acc.init_empty_weights = _init_empty_weights
    modeling.set_module_tensor_to_device = _set_module_tensor_to_device
    acc.utils, utils.modeling = utils, modeling
    sys.modules.update({"accelerate": acc, "accelerate.utils": utils,
                        "accelerate.utils.modeling": modeling})


def import_reference():
    """Import the reference package from its source tree; returns the ``rocketllm`` module."""
    if not reference_available():
        raise RuntimeError(f"the reference source tree is not at {REFERENCE_ROOT}")
    install_accelerate_standin()
    if REFERENCE_ROOT not in sys.path:
        sys.path.insert(0, REFERENCE_ROOT)
    import rocketllm
    import rocketllm.base  # noqa: F401
    return rocketllm


_TRIPLE = ("_packed", "_scale", "_zero_point")


def register_dequant_rw4():
    """Register the dequant-to-scratch ``rw4`` quantizer (transformers) and backend (the
    reference's registry).  Idempotent; not combinable in one process with the package's own
    ``rw4`` registration (both claim the name)."""
    import_reference()
    from rocketllm.quant.kv_cache import QuantizedTensor
    from rocketllm.quant.registry import QuantBackend, register_backend, registered_backends
    from transformers.quantizers.auto import (AUTO_QUANTIZATION_CONFIG_MAPPING,
                                              AUTO_QUANTIZER_MAPPING,
                                              register_quantization_config, register_quantizer)
    from transformers.quantizers.base import HfQuantizer
    from transformers.utils.quantization_config import QuantizationConfigMixin

    if AUTO_QUANTIZER_MAPPING.get("rw4") is not None and \
            getattr(AUTO_QUANTIZER_MAPPING["rw4"], "_dequant_harness", False):
        return

    class DequantRW4Config(QuantizationConfigMixin):
        def __init__(self, bits=4, group_size=64, modules_to_not_convert=None, **kwargs):
            self.quant_method = "rw4"
            self.bits, self.group_size = bits, group_size
            self.modules_to_not_convert = list(modules_to_not_convert or [])

        def to_dict(self):
            return {"quant_method": "rw4", "bits": self.bits, "group_size": self.group_size,
                    "modules_to_not_convert": self.modules_to_not_convert}

    class DequantRW4Quantizer(HfQuantizer):
        _dequant_harness = True
        requires_calibration = True

        def validate_environment(self, *args, **kwargs):
            return

        def update_dtype(self, dtype):
            return dtype

        def param_needs_quantization(self, model, param_name, **kwargs):
            return False

        def _process_model_before_weight_loading(self, model, **kwargs):
            skip = tuple(self.quantization_config.modules_to_not_convert)
            for name, module in model.named_modules():
                if not isinstance(module, torch.nn.Linear) or any(
                        name == s or name.endswith("." + s) for s in skip):
                    continue
                n, k = module.weight.shape
                for suffix, shape, dt in (("_packed", (n, k // 2), torch.uint8),
                                          ("_scale", (n, k // 64), torch.float16),
                                          ("_zero_point", (n, k // 64), torch.float16)):
                    module.register_parameter(
                        "weight" + suffix,
                        torch.nn.Parameter(torch.empty(shape, dtype=dt, device="meta"),
                                           requires_grad=False))
            return model

        def _process_model_after_weight_loading(self, model, **kwargs):
            return model

        @property
        def is_serializable(self):
            return True

        @property
        def is_trainable(self):
            return False

    class DequantRW4Backend(QuantBackend):
        """The reference's dequant-to-scratch path for an RW4 checkpoint."""
        format = "rw4-dequant"
        quant_methods = ("rw4",)

        def needs_scratch(self, weight):
            return True

        def prepare_layer(self, state_dict):
            out = OrderedDict()
            for name, value in state_dict.items():
                base, suffix = None, None
                for s in _TRIPLE:
                    if name.endswith(s):
                        base, suffix = name[:-len(s)], s
                if base is not None and base + "_packed" in state_dict:
                    if suffix == "_packed":
                        n, half = value.shape
                        q = QuantizedTensor(packed=value, scale=state_dict[base + "_scale"],
                                            zero=state_dict[base + "_zero_point"], axis=1,
                                            group=64, length=2 * half, padding=0,
                                            shape=(n, 2 * half), dtype=self.compute_dtype)
                        out[base] = q.dequantize()
                    continue
                out[name] = value
            return out

    if "rw4" not in AUTO_QUANTIZATION_CONFIG_MAPPING:
        register_quantization_config("rw4")(DequantRW4Config)
    else:
        AUTO_QUANTIZATION_CONFIG_MAPPING["rw4"] = DequantRW4Config
    AUTO_QUANTIZER_MAPPING["rw4"] = DequantRW4Quantizer
    if not any(getattr(b, "format", None) == "rw4-dequant" for b in registered_backends()):
        register_backend(DequantRW4Backend)


def reference_cpu_model(path, threads=None, dtype=torch.float32):
    """The reference's ``RocketModel`` on the CPU in ``dtype`` (fp32 by default) over the checkpoint
    at ``path`` (its own per-layer shard split, streaming and caching), without a tokenizer (token
    ids only, as the reference's own CPU generation test builds it,
    ``tests/test_cpu_generation.py:37-45``)."""
    rocketllm = import_reference()
    register_dequant_rw4()
    if threads:
        torch.set_num_threads(int(threads))

    class TokenIdModel(rocketllm.base.RocketModel):
        def get_tokenizer(self, hf_token=None):
            return None

    return TokenIdModel(str(path), device="cpu", dtype=dtype)


def phase_marker(force=None):
    """A logits processor that records every step's scores and a timestamp: transformers calls it
    once per generated token, the first call at the end of prefill -- the reference harness's
    decode-rate method (``tests/bench_streaming.py:474-502``).  With ``force`` (a token sequence)
    it then leaves only that step's token, so the run follows ``force`` (teacher forcing) and its
    recorded scores are comparable step by step with the run that produced ``force``."""
    import time

    from transformers import LogitsProcessor

    class Marker(LogitsProcessor):
        def __init__(self):
            self.times, self.scores = [], []

        def __call__(self, input_ids, scores):
            self.times.append(time.perf_counter())
            self.scores.append(scores.detach().float().clone())
            if force is None:
                return scores
            forced = torch.full_like(scores, float("-inf"))
            forced[:, int(force[len(self.scores) - 1])] = 0
            return forced

        def decode_tokens_per_second(self):
            if len(self.times) < 2:
                return None
            return (len(self.times) - 1) / (self.times[-1] - self.times[0])

    return Marker()

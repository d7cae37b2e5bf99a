"""RW4 quantization plugin surface: registry + backend, transformers quantizer, modules, converter.

Importing this package registers the ``rw4`` backend (``register_backend``) and the transformers
``rw4`` quantization config / quantizer / experts implementation.
"""
from .registry import (COMPANION_SUFFIXES, PackedWeight, QuantBackend, TensorSpec, decision_table,
                       detect_backend, quant_method_of, register_backend, registered_backends)
from .rw4 import RW4Backend
from .modules import RW4Linear, rw4_experts_forward, rw4_experts_params
from .hf import RW4Config, RW4HfQuantizer, convert_modules

__all__ = ["COMPANION_SUFFIXES", "PackedWeight", "QuantBackend", "TensorSpec", "decision_table",
           "detect_backend", "quant_method_of", "register_backend", "registered_backends",
           "RW4Backend", "RW4Linear", "rw4_experts_forward", "rw4_experts_params", "RW4Config",
           "RW4HfQuantizer", "convert_modules"]

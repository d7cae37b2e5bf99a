"""The RW4 quant backend: RocketLLM's int4 codec applied to Linear weights, computed packed.

A logical weight ``X.weight`` is stored as three checkpoint tensors (the companion-suffix
convention of ``rocketllm/quant/registry.py:33``):

    X.weight_packed       uint8 [N, K/2]   two codes per byte, even index in the low nibble
    X.weight_scale        fp16  [N, K/64]
    X.weight_zero_point   fp16  [N, K/64]

exactly the ``packed`` / ``scale`` / ``zero`` of ``rocketllm/quant/kv_cache.py:190-221`` with
``axis=1, group_size=64``.  The backend reports ``needs_scratch = False``: the sm_100a library
multiplies the packed form directly (``fused_packed``), so ``prepare_layer`` is the identity and a
layer's packed bytes are all that ever crosses PCIe.
"""
import torch

from .registry import QuantBackend, register_backend

GROUP = 64


@register_backend
class RW4Backend(QuantBackend):
    format = "rw4"
    quant_methods = ("rw4",)
    PAYLOAD_SUFFIXES = ("_packed",)

    @classmethod
    def example_config(cls):
        return {"quant_method": "rw4", "bits": 4, "group_size": GROUP}

    def bits(self, weight):
        payload = weight.payload
        if payload.dtype == torch.uint8 and payload.name.endswith("_packed"):
            return 4
        return super().bits(weight)

    def values_per_item(self, weight):
        return 2 if self.bits(weight) == 4 else super().values_per_item(weight)

    def logical_shape(self, weight):
        p = weight.payload
        if p.dtype == torch.uint8 and p.name.endswith("_packed") and len(p.shape) >= 2:
            return tuple(p.shape[:-1]) + (p.shape[-1] * 2,)
        return None

    def needs_scratch(self, weight):
        """Never: the RW4 library computes on the packed weight (no dequant-to-scratch)."""
        return False

    def prepare_layer(self, state_dict):
        return state_dict

    def decision(self):
        from .. import _lib
        try:
            _lib.lib()
            available, reason = True, "librw4.so loaded: dequant-GEMV / tcgen05 GEMM on packed weights"
        except RuntimeError as exc:
            available, reason = False, str(exc)
        return {"format": self.format, "capability": "rw4 sm_100a kernels (librw4.so)",
                "available": available, "path": "fused_packed" if available else "unavailable",
                "reason": reason}

"""The quant-registry plugin surface, with the RW4 backend registered in it.

Same interface as RocketLLM's ``rocketllm/quant/registry.py`` (``TensorSpec`` :51-97,
``PackedWeight`` :100-262, ``QuantBackend`` :265-560, ``register_backend`` / ``detect_backend`` /
``decision_table`` :631-690): a backend groups a shard's checkpoint tensors into logical weights,
sizes them in packed bytes, says whether the running device can compute on them as stored
(``needs_scratch``), places them, and reports its decision.  The names and argument meanings are
kept so engine code written against the reference calls this unchanged; the implementation is this
package's own, restricted to what the RW4 hot path needs (no accelerate dependency: placement binds
the tensor onto the module directly).
"""
import logging
from collections import OrderedDict

import torch

log = logging.getLogger(__name__)

#: Companion-tensor suffixes, longest first (``registry.py:33``).
COMPANION_SUFFIXES = ("_scale_inv", "_zero_point", "_packed", "_scale", "_shape", "_g_idx")
BIT_WIDTH_KEYS = ("bits", "w_bit", "num_bits", "weight_bits")


def _itemsize(dtype):
    return int(torch.empty((), dtype=dtype).element_size())


class TensorSpec:
    """One checkpoint tensor described without its data (``registry.py:51-97``)."""

    __slots__ = ("name", "shape", "dtype")

    def __init__(self, name, shape, dtype):
        self.name = name
        self.shape = tuple(int(d) for d in shape)
        self.dtype = dtype

    @classmethod
    def of(cls, name, tensor):
        return cls(name, tuple(tensor.shape), tensor.dtype)

    @property
    def numel(self):
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def itemsize(self):
        return _itemsize(self.dtype)

    @property
    def nbytes(self):
        return self.numel * self.itemsize

    @property
    def is_floating_point(self):
        return self.dtype.is_floating_point

    def __eq__(self, other):
        return (isinstance(other, TensorSpec) and (self.name, self.shape, self.dtype)
                == (other.name, other.shape, other.dtype))

    def __hash__(self):
        return hash((self.name, self.shape, self.dtype))

    def __repr__(self):
        return f"<TensorSpec {self.name} {self.shape} {self.dtype}>"


class PackedWeight:
    """One logical weight and the checkpoint tensors it spans (``registry.py:100-262``).

    Sizes are packed bytes (what crosses the link); ``expanded_bytes`` is the dequantized size.
    """

    __slots__ = ("name", "specs", "backend", "_values", "_shard")

    def __init__(self, name, specs, backend, values=None, shard=None):
        self.name = name
        self.specs = tuple(specs)
        self.backend = backend
        self._values = values
        self._shard = shard

    format = property(lambda self: self.backend.format)
    tensor_names = property(lambda self: tuple(s.name for s in self.specs))
    payload = property(lambda self: self.specs[0])
    companions = property(lambda self: self.specs[1:])
    bits = property(lambda self: self.backend.bits(self))
    logical_shape = property(lambda self: self.backend.logical_shape(self))
    packed_bytes = property(lambda self: sum(s.nbytes for s in self.specs))
    expanded_bytes = property(lambda self: self.backend.expanded_bytes(self))
    needs_scratch = property(lambda self: self.backend.needs_scratch(self))
    has_values = property(lambda self: self._values is not None)

    @property
    def scratch_bytes(self):
        return self.expanded_bytes if self.needs_scratch else 0

    def value_of(self, tensor_name):
        if self._values is None:
            raise ValueError(
                f"{self.name} was planned from checkpoint metadata alone, so it has no tensor data "
                f"to place; build it from a state dict to materialise it")
        return self._values[tensor_name]

    def place(self, tensor_name, device, shard=None):
        return self.backend.place(tensor_name, self.value_of(tensor_name), device,
                                  shard if shard is not None else self._shard or self._values)

    @property
    def placed_names(self):
        return [s.name for s in self.specs if not self.backend.is_consumed(s.name, self.name)]

    def materialize(self, device, shard=None):
        placed = []
        for name in self.placed_names:
            self.place(name, device, shard)
            placed.append(name)
        return placed

    def placements(self):
        out = []
        for name in self.placed_names:
            if self.backend.needs_quantizer(name):
                continue
            value = self.value_of(name)
            out.append((name, value, self.backend.target_dtype(name, value)))
        return out

    def quantizer_names(self):
        return [n for n in self.placed_names if self.backend.needs_quantizer(n)]

    def describe(self):
        return {"name": self.name, "format": self.format, "tensors": list(self.tensor_names),
                "bits": self.bits, "packed_bytes": self.packed_bytes,
                "expanded_bytes": self.expanded_bytes, "needs_scratch": self.needs_scratch,
                "logical_shape": self.logical_shape}

    def __repr__(self):
        return (f"<PackedWeight {self.name} {self.format} {len(self.specs)} tensors "
                f"{self.packed_bytes}B packed>")


def set_module_tensor(model, tensor_name, value):
    """Bind ``value`` as the parameter or buffer ``tensor_name`` of ``model`` (no copy)."""
    module_name, _, leaf = tensor_name.rpartition(".")
    module = model.get_submodule(module_name) if module_name else model
    if leaf in module._parameters:
        module._parameters[leaf] = torch.nn.Parameter(value, requires_grad=False)
    elif leaf in module._buffers:
        module._buffers[leaf] = value
    else:
        raise KeyError(f"{tensor_name}: no such parameter or buffer")


class QuantBackend:
    """How one storage format becomes weights on a device (``registry.py:265-560``).

    This base is the unquantized format; subclasses declare ``quant_methods`` and override the
    per-format answers.
    """

    format = "dense"
    quant_methods = ()
    PAYLOAD_SUFFIXES = ("_packed",)

    def __init__(self, config=None, caps=None, model=None, hf_quantizer=None, compute_dtype=None,
                 device=None, shape_adopter=None):
        self.config = config
        self.model = model
        self.hf_quantizer = hf_quantizer
        self.device = device
        self._caps = caps
        self._compute_dtype = compute_dtype
        self._shape_adopter = shape_adopter
        self._config_dict = _as_dict(config)
        self._declared_bits = _find_int(self._config_dict, BIT_WIDTH_KEYS)

    @classmethod
    def matches(cls, quant_method, config):
        return quant_method in cls.quant_methods

    @classmethod
    def example_config(cls):
        return {"quant_method": cls.quant_methods[0]} if cls.quant_methods else None

    @property
    def caps(self):
        return self._caps

    @property
    def compute_dtype(self):
        if self._compute_dtype is not None:
            return self._compute_dtype
        return getattr(self._caps, "compute_dtype", None) or torch.bfloat16

    # -- layout ------------------------------------------------------------------------------------

    def logical_name(self, tensor_name, known=()):
        module, _, leaf = tensor_name.rpartition(".")
        for suffix in COMPANION_SUFFIXES:
            if leaf.endswith(suffix) and leaf != suffix:
                stem = leaf[: -len(suffix)]
                return f"{module}.{stem}" if module else stem
        return tensor_name

    def is_payload(self, tensor_name, logical_name):
        return tensor_name == logical_name or any(
            tensor_name == logical_name + s for s in self.PAYLOAD_SUFFIXES)

    def is_consumed(self, tensor_name, logical_name):
        return False

    def _group(self, items, name_of):
        known = {name_of(i) for i in items}
        groups = OrderedDict()
        for item in items:
            groups.setdefault(self.logical_name(name_of(item), known), []).append(item)
        for logical, members in groups.items():
            payload = next((m for m in members if self.is_payload(name_of(m), logical)),
                           members[0])
            yield logical, [payload] + [m for m in members if m is not payload]

    def plan(self, state_dict):
        weights = []
        for logical, names in self._group(list(state_dict), lambda n: n):
            specs = [TensorSpec.of(n, state_dict[n]) for n in names]
            weights.append(PackedWeight(logical, specs, self,
                                        values={n: state_dict[n] for n in names},
                                        shard=state_dict))
        return weights

    def plan_from_specs(self, specs):
        return [PackedWeight(logical, group, self)
                for logical, group in self._group(list(specs), lambda s: s.name)]

    # -- sizing --------------------------------------------------------------------------------------

    def declared_bits(self):
        return self._declared_bits

    def bits(self, weight):
        payload = weight.payload
        stored = payload.itemsize * 8
        if payload.is_floating_point and stored >= 16:
            return stored
        return self.declared_bits() or stored

    def values_per_item(self, weight):
        stored = weight.payload.itemsize * 8
        bits = self.bits(weight)
        return max(1, stored // bits) if bits else 1

    def logical_shape(self, weight):
        return None

    def logical_numel(self, weight):
        shape = weight.logical_shape
        if shape is not None:
            n = 1
            for d in shape:
                n *= d
            return n
        return weight.payload.numel * self.values_per_item(weight)

    def expanded_bytes(self, weight):
        return self.logical_numel(weight) * _itemsize(self.compute_dtype)

    # -- the per-device decision ---------------------------------------------------------------------

    def needs_scratch(self, weight):
        return self.bits(weight) < 16

    # -- placement -----------------------------------------------------------------------------------

    def needs_quantizer(self, tensor_name):
        q = self.hf_quantizer
        return bool(q is not None and q.param_needs_quantization(self.model, tensor_name))

    def load_verbatim(self, tensor_name, value):
        """Packed integers, 1-byte floats and companions keep their dtype (``registry.py:486-512``)."""
        if not value.is_floating_point():
            return True
        if value.element_size() == 1:
            return True
        return tensor_name.endswith(COMPANION_SUFFIXES)

    def target_dtype(self, tensor_name, value):
        return value.dtype if self.load_verbatim(tensor_name, value) else self.compute_dtype

    def place(self, tensor_name, value, device, shard=None):
        if self._shape_adopter is not None:
            self._shape_adopter(tensor_name, value)
        dtype = self.target_dtype(tensor_name, value)
        set_module_tensor(self.model, tensor_name, value.to(device=device, dtype=dtype))
        return tensor_name

    def prepare_layer(self, state_dict):
        return state_dict

    # -- reporting -----------------------------------------------------------------------------------

    def decision(self):
        return {"format": self.format,
                "capability": "none: stored weights are already in a computable dtype",
                "available": True, "path": "as_stored",
                "reason": "an unquantized checkpoint is placed as it is, cast to the compute dtype"}

    def summary(self):
        info = dict(self.decision())
        info.update({"quant_method": quant_method_of(self.config),
                     "declared_bits": self._declared_bits,
                     "compute_dtype": str(self.compute_dtype).replace("torch.", ""),
                     "hf_quantizer": type(self.hf_quantizer).__name__ if self.hf_quantizer
                     else None})
        return info

    def __repr__(self):
        return f"<{type(self).__name__} {self.format}>"


def _as_dict(config):
    if config is None:
        return {}
    if isinstance(config, dict):
        return config
    for attr in ("to_dict", "to_diff_dict"):
        fn = getattr(config, attr, None)
        if callable(fn):
            try:
                out = fn()
                if isinstance(out, dict):
                    return out
            except Exception:  # noqa: BLE001 - an unserialisable config is still usable
                pass
    return {k: v for k, v in vars(config).items() if not k.startswith("_")}


def _find_int(node, keys, depth=0):
    if depth > 6 or not isinstance(node, (dict, list, tuple)):
        return None
    if isinstance(node, dict):
        for key in keys:
            v = node.get(key)
            if isinstance(v, int) and not isinstance(v, bool):
                return int(v)
        children = node.values()
    else:
        children = node
    for child in children:
        found = _find_int(child, keys, depth + 1)
        if found is not None:
            return found
    return None


def quant_method_of(quantization_config):
    """The declared ``quant_method``, lowercased, or ``None`` (``registry.py:605-626``)."""
    if quantization_config is None:
        return None
    if isinstance(quantization_config, dict):
        method = quantization_config.get("quant_method")
    else:
        method = getattr(quantization_config, "quant_method", None)
        if method is None:
            method = _as_dict(quantization_config).get("quant_method")
    method = getattr(method, "value", method)
    return str(method).lower() if method is not None else None


_BACKENDS = []


def register_backend(cls):
    """Register a backend for detection; first match wins (``registry.py:634-638``)."""
    if cls not in _BACKENDS:
        _BACKENDS.append(cls)
    return cls


def _load_backends():
    if not _BACKENDS:
        from . import rw4  # noqa: F401 - imported for its registration


def registered_backends():
    _load_backends()
    return tuple(_BACKENDS)


def detect_backend(quantization_config=None, **context):
    """The backend for what the checkpoint declares about itself (``registry.py:656-675``).

    A declared method nothing here recognises raises: this package computes RW4 only and has no
    delegating fallback path.
    """
    _load_backends()
    method = quant_method_of(quantization_config)
    for cls in _BACKENDS:
        if cls.matches(method, quantization_config):
            return cls(config=quantization_config, **context)
    if method is not None:
        raise ValueError(f"quant_method {method!r} is not served by rocketllm_b200 "
                         f"(known: {[c.quant_methods for c in _BACKENDS]})")
    return QuantBackend(config=quantization_config, **context)


def decision_table(caps=None, compute_dtype=None):
    _load_backends()
    return [cls(config=cls.example_config(), caps=caps, compute_dtype=compute_dtype).decision()
            for cls in list(_BACKENDS) + [QuantBackend]]

"""Layer streaming engine and the ``AutoModel`` / ``RocketModel`` entry points.

Counterpart of RocketLLM's engine hooks (``rocketllm/base.py``: forward pre-hook ``_pre_hook``
:1916-1926 -> ``cache.acquire`` -> ``_move_coalesced`` :952-991 -> bind; ``prefetch_window``
``memory/cache.py:254-272``) for RW4 checkpoints on B200, built the device-first way:

* every streamed decoder layer is packed ONCE into a single pinned host blob (its RW4 codes, fp16
  scales / zeros and bf16 norms at 256-byte aligned offsets) -- the host tier the reference
  stages into a leased buffer on every fetch;
* the device holds ``window`` slots, each the size of the largest blob; layer ``i`` always lives
  in slot ``i % window`` and its parameters are bound ONCE as views into that slot, so a layer
  fetch is one chunked host->device send and no Python rebinding;
* the pre-hook of layer ``i`` makes the compute stream wait (device-side) for layer ``i``'s send
  and issues the sends of layers ``i+1 .. i+window-1`` into their slots, ordered after the compute
  already queued (the slot's previous occupant) -- so the next layers cross PCIe while this one
  computes, and the loop wraps around to layer 0 for the next token.

Transformers still owns the forward, attention, KV cache and ``generate``.  Resident mode (the
whole model fits the VRAM budget) moves everything to the device and installs no hooks.
"""
import os

import torch

from . import quant  # noqa: F401 - registers the rw4 quantizer with transformers
from .expert_stream import (DeviceExpertStreamer, ExpertStreamer, expert_blob_bytes,
                            is_rw4_experts)
from .streaming import WeightTransfer

ALIGN = 256


class _LayerBlob:
    __slots__ = ("host", "entries", "nbytes")

    def __init__(self, host, entries, nbytes):
        self.host = host          # pinned uint8 [nbytes]
        self.entries = entries    # [(module, leaf, kind, dtype, shape, offset)]
        self.nbytes = nbytes


def _layer_tensors(layer, skip_experts=False):
    out = []
    for mname, module in layer.named_modules():
        if skip_experts and is_rw4_experts(module):
            continue  # streamed per expert (expert_stream.py)
        for leaf, p in module._parameters.items():
            if p is not None:
                out.append((module, leaf, "param", p))
        for leaf, b in module._buffers.items():
            if b is not None and b.numel() and leaf not in module._non_persistent_buffers_set:
                out.append((module, leaf, "buffer", b))
    return out


def _pack_layer(layer, skip_experts=False):
    tensors = _layer_tensors(layer, skip_experts)
    entries, off = [], 0
    for module, leaf, kind, t in tensors:
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        entries.append((module, leaf, kind, t.dtype, tuple(t.shape), off))
        off += t.numel() * t.element_size()
    nbytes = (off + ALIGN - 1) // ALIGN * ALIGN
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    for (module, leaf, kind, dtype, shape, o), (_, _, _, t) in zip(entries, tensors):
        n = t.numel() * t.element_size()
        host[o:o + n].copy_(t.detach().contiguous().view(-1).view(torch.uint8))
    return _LayerBlob(host, entries, nbytes)


def _bind(blob, slot):
    for module, leaf, kind, dtype, shape, off in blob.entries:
        n = 1
        for d in shape:
            n *= d
        view = slot[off:off + n * torch.empty((), dtype=dtype).element_size()].view(dtype)
        view = view.view(shape)
        if kind == "param":
            module._parameters[leaf] = torch.nn.Parameter(view, requires_grad=False)
        else:
            module._buffers[leaf] = view


class LayerStreamer:
    """Streams decoder layers from pinned host blobs through ``window`` device slots.

    The last ``pinned`` layers are kept resident instead (uploaded once, no hooks): every token
    reads every dense layer, so each resident byte saves one streamed byte per token -- the
    reference's pin placement for dense blocks (``rocketllm/memory/placement.py``).  They are the
    last ones so that their compute covers the prefetch of the next token's first streamed
    layers."""

    def __init__(self, layers, device, window=2, copy_streams=2, chunk_bytes=16 << 20,
                 prefetching=True, expert_slots=None, blobs=None, pinned=0,
                 expert_routing="host", expert_policy=None, storage=None):
        if window < 1:
            raise ValueError("window must be >= 1")
        self.layers = list(layers)
        self.device = torch.device(device)
        self.pinned = max(0, min(int(pinned), len(self.layers)))
        self.streamed = len(self.layers) - self.pinned
        self.window = min(window, self.streamed)
        self.prefetching = prefetching
        # routed experts stream one by one (expert_stream.py) when expert_slots is given
        stream_experts = expert_slots is not None
        # blobs: prebuilt host blobs (read from layer shards on disk); else packed from the layers
        self.blobs = blobs if blobs is not None else [_pack_layer(layer, stream_experts)
                                                      for layer in self.layers]
        self.slot_bytes = max((b.nbytes for b in self.blobs[:self.streamed]), default=0)
        self.slots = [torch.empty(self.slot_bytes, dtype=torch.uint8, device=self.device)
                      for _ in range(self.window)]
        for i in range(self.streamed):
            _bind(self.blobs[i], self.slots[i % self.window])
        self.resident = []   # device storage of the pinned layers
        for i in range(self.streamed, len(self.layers)):
            blob = self.blobs[i]
            dev = torch.empty(blob.nbytes, dtype=torch.uint8, device=self.device)
            dev.copy_(blob.host[:blob.nbytes])
            _bind(blob, dev)
            self.resident.append(dev)
            self.blobs[i] = _LayerBlob(None, blob.entries, blob.nbytes)  # host copy released
        # storage tier (shards.LayerStager): streamed layers with no host blob are read from their
        # shard files ahead of use into leases of the stager's pool; the transfer engine releases
        # a lease once its copy has finished (and reclaims finished ones when the pool runs dry)
        self.storage = storage
        if any(self.blobs[i].host is None for i in range(self.streamed)) and storage is None:
            raise ValueError("streamed layers without a host blob need a storage tier")
        self.xfer = WeightTransfer(device=self.device, copy_streams=copy_streams,
                                   chunk_bytes=chunk_bytes,
                                   pool=storage.pool if storage is not None else None)
        self.experts = None
        if stream_experts:
            moe = [(i, m) for i, layer in enumerate(self.layers) for m in layer.modules()
                   if is_rw4_experts(m)]
            if moe and expert_routing == "device":
                self.experts = DeviceExpertStreamer(moe, self.device, expert_slots,
                                                    policy=expert_policy or "lru")
            elif moe:
                self.experts = ExpertStreamer(moe, self.device, expert_slots, self.xfer,
                                              policy=expert_policy or "lfu")
        self.tickets = [None] * len(self.layers)
        self.resident_slot = [None] * self.window   # which layer's bytes a slot holds (issued)
        self.fetches = 0
        self.bytes = 0
        self.hits = 0
        self._handles = [self.layers[i].register_forward_pre_hook(self._make_pre_hook(i))
                         for i in range(self.streamed)]

    def _send(self, i, compute):
        s = i % self.window
        if self.resident_slot[s] == i:
            return
        blob = self.blobs[i]
        if blob.host is None:
            lease = self.storage.take(i)
            handle = self.xfer.send_buffer(lease.view, lease=lease,
                                           out=self.slots[s][:blob.nbytes], after=compute)
        else:
            handle = self.xfer.send_buffer(blob.host, out=self.slots[s][:blob.nbytes],
                                           after=compute)
        self.tickets[i] = handle
        self.resident_slot[s] = i
        self.fetches += 1
        self.bytes += blob.nbytes

    def _make_pre_hook(self, i):
        def hook(module, args):
            compute = torch.cuda.current_stream(self.device)
            if self.resident_slot[i % self.window] != i:
                self._send(i, compute)
            else:
                self.hits += 1
            handle = self.tickets[i]
            if handle is not None:
                handle.resolve(compute)
                self.tickets[i] = None
            if self.prefetching:
                n = self.streamed
                for d in range(1, self.window):
                    j = (i + d) % n
                    # never into the slot of the layer about to run (only possible when the
                    # layer count is not a multiple of the window and the loop wraps)
                    if j % self.window != i % self.window:
                        self._send(j, compute)
            return None
        return hook

    def stats(self):
        return {"layers": len(self.layers), "pinned": self.pinned, "streamed": self.streamed,
                "window": self.window, "slot_bytes": self.slot_bytes,
                "fetches": self.fetches, "bytes": self.bytes, "slot_hits": self.hits,
                "experts": self.experts.stats() if self.experts else None,
                "storage": self.storage.stats() if self.storage else None,
                "transfer": self.xfer.stats()}

    def close(self):
        for h in self._handles:
            h.remove()
        self._handles = []
        if hasattr(self.experts, "close"):
            self.experts.close()
        self.xfer.close()
        if self.storage is not None:
            self.storage.close()
            self.storage.pool.close()
            self.storage = None


def _layers_path(model):
    for path in ("model.layers", "model.decoder.layers", "transformer.h"):
        try:
            model.get_submodule(path)
            return path
        except AttributeError:
            continue
    raise ValueError("cannot find the decoder layers of this model")


def _decoder_layers(model):
    return model.get_submodule(_layers_path(model))


def footprint(model, skip_experts=False):
    """``(resident_bytes, [bytes of each decoder layer])`` of ``model`` (without the routed
    experts' stacked weights when ``skip_experts``)."""
    layers = _decoder_layers(model)
    layer_bytes = [sum(t.numel() * t.element_size() for *_, t in _layer_tensors(l))
                   for l in layers]
    if skip_experts:
        dense = [sum(t.numel() * t.element_size() for *_, t in _layer_tensors(l, True))
                 for l in layers]
        total = sum(p.numel() * p.element_size() for p in model.parameters())
        total += sum(b.numel() * b.element_size() for b in model.buffers())
        return total - sum(layer_bytes), dense
    total = sum(p.numel() * p.element_size() for p in model.parameters())
    total += sum(b.numel() * b.element_size() for b in model.buffers())
    return total - sum(layer_bytes), layer_bytes


# Constructor knobs of the reference's RocketModel (rocketllm/base.py:203-208) that have no
# counterpart here (its hardware-profile overrides, shard-path and tokenizer options): accepted so
# that code written for the reference runs unchanged, and ignored.  Anything else is an error.
REFERENCE_ONLY_KNOBS = ("max_seq_len", "layer_shards_saving_path", "profiling_mode",
                        "compression", "hf_token", "delete_original", "vram_reserve",
                        "host_cache_gb", "window_max", "shard_handle_limit", "pin_policy",
                        "expert_residency")


class RocketModel:
    """An RW4 ``*ForCausalLM`` with layer streaming (the reference's ``RocketModel`` surface:
    ``generate``, ``__call__``/``forward``, ``stats``, ``close``).

    ``vram_budget`` (bytes) bounds the model's device footprint: if the whole model fits it (or it
    is None) every layer is resident; otherwise the non-layer modules stay resident and at most
    ``window`` layer slots fit in what is left (at least one); the last layers that still fit
    beside those slots stay resident (pinned) and the others stream from pinned host memory every
    token.  In a mixture-of-experts model the routed experts stream one by one
    (``expert_streaming``): the layer slots hold the attention / router / norms only, and the rest
    of the budget becomes an expert cache of at least one layer's experts.  ``expert_routing``:
    ``"host"`` reads the routed set back per MoE layer and issues the sends from the host (the
    reference's scheme); ``"device"`` decides residency and copies on the device
    (:class:`~rocketllm_b200.expert_stream.DeviceExpertStreamer`, at most 80 expert slots).
    ``expert_policy``: which resident expert gives way, ``"lfu"`` (the reference's LFU with aging)
    or ``"lru"``; None takes ``"lfu"`` with host routing and ``"lru"`` with device routing.
    ``io_workers``: threads that read each layer's blob from a layer-shard directory (adjacent,
    byte-balanced stretches of the blob: the reference loader's ``io_workers``).
    ``host_budget`` (bytes; layer-shard directories only): pinned host memory for streamed layer
    blobs.  Streamed layers past it form the storage tier: they stay in their files and are read
    ``storage_depth`` layers ahead of use into leased staging buffers on every pass
    (:class:`~rocketllm_b200.shards.LayerStager`).  None keeps every blob in host memory.  The
    staging pool those reads land in is pinned on top of ``host_budget``: ``storage_depth + window
    + 1`` buffers of the largest layer blob's power-of-two size class (``stats()["staging_pool"]``).
    ``read_faults`` (layer-shard directories; tests of failure handling): host-side injected read
    failures, ``shards.parse_faults`` -- e.g. ``"read:layer=3:pass=2"``, or ``"env"`` for the
    ``RW4_FAULT`` variable; None (default) injects nothing.

    ``kv_cache`` (``rocketllm/base.py:208-411``, ``quant/kv_cache.py:449-503``): ``"int4"`` gives
    every ``generate`` an :class:`~rocketllm_b200.kv_cache.RW4KVCache` whose decode attention reads
    the packed history; ``"fp16"`` keeps transformers' own cache; ``"auto"`` (default) quantizes the
    context exactly when the weights do not fit the budget (they stream).  ``hqq`` / ``quanto``
    (transformers' optional caches) fall back to the stock cache.

    ``draft_model`` / ``speculative`` (``rocketllm/spec/draft.py``): with a draft (a path, a
    transformers model or a :class:`~rocketllm_b200.speculative.DraftModel`) one-sequence
    ``generate`` calls run :class:`~rocketllm_b200.speculative.SpeculativeDecoder` -- ``"on"``
    always, ``"auto"`` when the weights stream, ``"off"`` never; ``lookahead`` proposals per pass
    to start, adapted up to ``max_lookahead``.
    """

    def __init__(self, model_or_path, device="cuda", dtype=torch.bfloat16, vram_budget=None,
                 window=2, prefetching=True, copy_streams=2, chunk_bytes=16 << 20,
                 expert_streaming=True, kv_cache="auto", draft_model=None, speculative="auto",
                 lookahead=4, max_lookahead=8, expert_routing="host", expert_policy=None,
                 io_workers=4, host_budget=None, storage_depth=2, read_faults=None,
                 **reference_knobs):
        from .kv_cache import KV_CHOICES
        from .shards import INDEX
        from .speculative import SPEC_CHOICES
        unknown = sorted(set(reference_knobs) - set(REFERENCE_ONLY_KNOBS))
        if unknown:
            raise TypeError(f"RocketModel got unknown argument(s) {', '.join(unknown)}; "
                            f"the reference's other constructor knobs ("
                            f"{', '.join(REFERENCE_ONLY_KNOBS)}) are accepted and have no effect "
                            f"here")
        if reference_knobs.get("compression") is not None:
            raise ValueError("compression= is not supported: RocketLLM reads pre-quantized "
                             "checkpoints only (rocketllm/utils.py:31-56); convert with "
                             "rocketllm_b200.quant.convert.save_rw4_checkpoint")
        if kv_cache not in KV_CHOICES:
            raise ValueError(f"kv_cache must be one of {', '.join(KV_CHOICES)}, not {kv_cache!r}")
        if expert_routing not in ("host", "device"):
            raise ValueError(f"expert_routing must be 'host' or 'device', not {expert_routing!r}")
        if expert_policy is None:
            expert_policy = "lru" if expert_routing == "device" else "lfu"
        if expert_policy not in ("lfu", "lru"):
            raise ValueError(f"expert_policy must be 'lfu' or 'lru', not {expert_policy!r}")
        if speculative not in SPEC_CHOICES:
            raise ValueError(f"speculative must be one of {', '.join(SPEC_CHOICES)}, not "
                             f"{speculative!r}")
        self.kv_cache_setting = kv_cache
        self._kv_attention = False
        self.speculative_setting = speculative
        self._draft_arg = draft_model
        self._draft = None
        self.lookahead, self.max_lookahead = lookahead, max_lookahead
        self.speculation = None   # SpeculationStats of the last speculative generate
        if isinstance(model_or_path, (str, os.PathLike)) and \
                os.path.exists(os.path.join(str(model_or_path), INDEX)):
            self._init_from_shards(str(model_or_path), device, dtype, vram_budget, window,
                                   prefetching, copy_streams, chunk_bytes, io_workers,
                                   host_budget, storage_depth, expert_streaming, read_faults)
            return
        if host_budget is not None:
            raise ValueError("host_budget applies to a layer-shard directory "
                             "(shards.split_rw4_layers): a checkpoint or model loads whole into "
                             "host memory")
        if isinstance(model_or_path, (str, os.PathLike)):
            from transformers import AutoModelForCausalLM
            model = AutoModelForCausalLM.from_pretrained(str(model_or_path), dtype=dtype)
        else:
            model = model_or_path
        self.model = model.eval()
        self.device = torch.device(device)
        layers = _decoder_layers(model)
        rest, layer_bytes = footprint(model)   # embeddings, final norm, lm_head: resident
        total = rest + sum(layer_bytes)
        self.streamer = None
        stream = vram_budget is not None and total > vram_budget
        if not stream:
            self.model.to(self.device)
            return
        experts = [m for m in layers.modules() if is_rw4_experts(m)]
        expert_slots = None
        if experts and expert_streaming:
            # attention / norms / router of every layer before routed experts (the reference's
            # priority classes): window slots, then as many dense parts pinned as fit beside one
            # layer's worth of expert slots, then the rest of the budget as expert cache
            _, dense_bytes = footprint(model, skip_experts=True)
            per_layer = max(m.gate_up_proj_packed.shape[0] for m in experts)
            eb = max(expert_blob_bytes(m) for m in experts)
            left = max(0, vram_budget - rest - per_layer * eb)
            window = max(1, min(window, int(left // max(dense_bytes))))
            pinned = self._pin_count(dense_bytes, left, window)
            used = rest + self._plan_bytes(dense_bytes, window, pinned)
            expert_slots = max(per_layer, int((vram_budget - used) // eb))
        else:
            left = max(0, vram_budget - rest)
            window = max(1, min(window, int(left // max(layer_bytes))))
            pinned = self._pin_count(layer_bytes, left, window)
        # everything outside the decoder layers is resident: move the model with its layer
        # list detached, then hand the layers to the streamer (they stay on the host)
        parent_path, _, leaf = _layers_path(model).rpartition(".")
        parent = self.model.get_submodule(parent_path) if parent_path else self.model
        setattr(parent, leaf, torch.nn.ModuleList())
        self.model.to(self.device)
        setattr(parent, leaf, layers)
        self.streamer = LayerStreamer(layers, self.device, window=window,
                                      copy_streams=copy_streams, chunk_bytes=chunk_bytes,
                                      prefetching=prefetching, expert_slots=expert_slots,
                                      pinned=pinned, expert_routing=expert_routing,
                                      expert_policy=expert_policy)

    @staticmethod
    def _plan_bytes(layer_bytes, window, pinned):
        """Device bytes of ``window`` slots for the streamed layers plus the pinned last layers."""
        n = len(layer_bytes)
        streamed = layer_bytes[:n - pinned]
        return (window * max(streamed) if streamed else 0) + sum(layer_bytes[n - pinned:])

    @classmethod
    def _pin_count(cls, layer_bytes, free, window):
        """How many of the last layers fit resident beside the window slots in ``free`` bytes."""
        pinned = 0
        while pinned < len(layer_bytes) and \
                cls._plan_bytes(layer_bytes, window, pinned + 1) <= free:
            pinned += 1
        return pinned

    def _init_from_shards(self, root, device, dtype, vram_budget, window, prefetching,
                          copy_streams, chunk_bytes, io_workers=1, host_budget=None,
                          storage_depth=2, expert_streaming=True, read_faults=None):
        """Layer shards written by ``shards.split_rw4_layers``: the model is built on the meta
        device, the non-layer tensors come from ``rest.safetensors`` straight to the device, and
        each layer's blob is read from its file into pinned memory by positioned reads over
        ``io_workers`` threads (no CPU copy of the model ever exists).  Routed experts stream with
        their layer."""
        from .shards import LayerShardReader, _materialize_rest, build_skeleton
        self.device = torch.device(device)
        reader = LayerShardReader(root, io_workers=io_workers, faults=read_faults)
        self.shards = reader
        model = build_skeleton(root, dtype).eval()
        self.model = model
        layers_path = reader.index["layers_path"]
        _materialize_rest(model, root, self.device, layers_path)
        layers = model.get_submodule(layers_path)
        plans = [reader.plan(i) for i in range(len(reader))]
        rest = sum(p.numel() * p.element_size() for n, p in model.named_parameters()
                   if not n.startswith(layers_path + "."))
        layer_bytes = [nbytes for _, nbytes in plans]
        self.streamer = None

        def resolve(layer, entries):
            return [(layer.get_submodule(m) if m else layer, leaf, kind, dt, shape, off)
                    for m, leaf, kind, dt, shape, off in entries]

        if vram_budget is None or rest + sum(layer_bytes) <= vram_budget:
            staging = torch.empty(max(layer_bytes), dtype=torch.uint8).pin_memory()
            for i, layer in enumerate(layers):
                entries, nbytes = plans[i]
                reader.read_into(i, staging)
                slot = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                slot.copy_(staging[:nbytes])   # synchronous: the staging buffer is reused
                _bind(_LayerBlob(None, resolve(layer, entries), nbytes), slot)
            reader.close()
            return
        if expert_streaming and any(is_rw4_experts(m) for m in layers.modules()):
            reader.close()
            raise ValueError(
                "this layer-shard directory holds routed experts and the layers do not fit the "
                "VRAM budget: per-expert streaming (only the routed experts cross PCIe) is built "
                "for a checkpoint directory or a loaded model, not yet from layer shards.  Load "
                "the checkpoint directory instead, or pass expert_streaming=False to stream whole "
                "layers (every expert) from the shards")
        left = max(0, vram_budget - rest)
        window = max(1, min(window, int(left // max(layer_bytes))))
        pinned = self._pin_count(layer_bytes, left, window)
        streamed = len(layers) - pinned
        # host tier: streamed blobs in pinned host memory while host_budget lasts (in scan order);
        # the storage tier takes the rest, read from their files on every pass
        host_left = float("inf") if host_budget is None else max(0, int(host_budget))
        blobs, storage_layers = [], []
        for i, layer in enumerate(layers):
            entries, nbytes = plans[i]
            if i < streamed and (storage_layers or nbytes > host_left):
                blobs.append(_LayerBlob(None, resolve(layer, entries), nbytes))
                storage_layers.append(i)
                continue
            host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
            reader.read_into(i, host)
            if i < streamed:
                host_left -= nbytes
            blobs.append(_LayerBlob(host, resolve(layer, entries), nbytes))
        storage = None
        if storage_layers:
            from .shards import LayerStager
            from .streaming import HostStagingPool
            cls = HostStagingPool._size_class(max(layer_bytes[i] for i in storage_layers))
            pool = HostStagingPool(budget_bytes=(storage_depth + window + 1) * cls)
            storage = LayerStager(reader, storage_layers, pool, depth=storage_depth)
            for i in storage_layers[:storage_depth]:
                storage.request(i)
        else:
            reader.close()
        self.streamer = LayerStreamer(layers, self.device, window=window,
                                      copy_streams=copy_streams, chunk_bytes=chunk_bytes,
                                      prefetching=prefetching, blobs=blobs, pinned=pinned,
                                      storage=storage)

    @property
    def config(self):
        return self.model.config

    @property
    def kv_cache_choice(self):
        from .kv_cache import KV_AUTO, KV_FP16, KV_INT4
        if self.kv_cache_setting != KV_AUTO:
            return self.kv_cache_setting
        return KV_INT4 if self.streamer is not None else KV_FP16

    def draft(self):
        """The draft model (loaded on first use), or None."""
        from .speculative import DraftModel
        if self._draft is None and self._draft_arg is not None:
            d = self._draft_arg
            if isinstance(d, DraftModel):
                self._draft = d
            elif isinstance(d, (str, os.PathLike)):
                self._draft = DraftModel.load(str(d), target_config=self.model.config,
                                              device=self.device, dtype=torch.bfloat16)
            else:
                self._draft = DraftModel(d.to(self.device).eval())
        return self._draft

    def speculation_enabled(self):
        from .speculative import resolve_speculation
        return resolve_speculation(self.speculative_setting, self._draft_arg,
                                   streamed=self.streamer is not None)

    def generate(self, *args, **kwargs):
        from .kv_cache import KV_INT4, RW4KVCache, enable_kv_attention
        int4 = self.kv_cache_choice == KV_INT4
        if int4 and not self._kv_attention:
            enable_kv_attention(self.model)
            self._kv_attention = True
        ids = args[0] if args else kwargs.get("input_ids")
        if ids is not None and ids.shape[0] == 1 and self.speculation_enabled()[0]:
            return self._speculative_generate(ids, int4, **kwargs)
        fast = self._fused_greedy(ids, int4, kwargs)
        if fast is not None:
            return fast
        # a quantized context has to be handed in (transformers builds its own cache otherwise);
        # a cache the caller passed is kept
        if kwargs.get("past_key_values") is None and int4:
            kwargs["past_key_values"] = RW4KVCache(fused=True)
            kwargs.setdefault("use_cache", True)
        return self.model.generate(*args, **kwargs)

    # generate() arguments the fused greedy path honours; anything else goes to transformers
    _FUSED_KWARGS = frozenset(("input_ids", "max_new_tokens", "do_sample", "eos_token_id",
                               "pad_token_id", "min_new_tokens", "attention_mask", "use_cache"))

    def _fused_greedy(self, ids, int4, kwargs):
        """Greedy ``generate`` on the fused, CUDA-graphed decode step
        (:class:`~rocketllm_b200.fused_decode.FusedDecoder`) when it applies: a resident RW4 Llama
        model with the stock cache, greedy decoding, an explicit ``max_new_tokens`` and no
        argument the fused path does not honour (no padding mask, logits processors, streamers,
        dictionary outputs).  Returns the sequences as transformers does -- prompt, then the new
        tokens, rows that produced an end-of-sequence token padded after it, and the output cut
        where every row has ended -- or None to take transformers' loop."""
        from .fused_decode import FusedDecoder, fusable
        gc = self.model.generation_config
        if ids is None or ids.dim() != 2 or self.streamer is not None or int4:
            return None
        if set(kwargs) - self._FUSED_KWARGS or not kwargs.get("max_new_tokens"):
            return None
        do_sample = kwargs.get("do_sample", getattr(gc, "do_sample", False))
        if do_sample or getattr(gc, "num_beams", 1) not in (None, 1):
            return None
        mask = kwargs.get("attention_mask")
        if mask is not None and not bool(torch.all(mask == 1)):
            return None
        eos = kwargs.get("eos_token_id", getattr(gc, "eos_token_id", None))
        if eos is not None and kwargs.get("min_new_tokens"):
            return None   # transformers masks the end token below min_new_tokens; this path does not
        if not fusable(self.model):
            return None
        n = int(kwargs["max_new_tokens"])
        ids = ids.to(self.device)
        b, t = ids.shape
        dec = FusedDecoder(self.model, b, t + n + 1, device=self.device, use_graph=n > 2)
        new = dec.generate(ids, n)
        if eos is not None:
            eos = torch.tensor([eos] if isinstance(eos, int) else list(eos), device=self.device)
            pad = kwargs.get("pad_token_id", getattr(gc, "pad_token_id", None))
            pad = int(eos[0]) if pad is None else int(pad)
            hit = torch.isin(new, eos)
            done = hit.cumsum(1) > 0                    # at or after the first end token
            after = done & ~hit.logical_and(hit.cumsum(1) == 1)
            new = torch.where(after, torch.full_like(new, pad), new)
            if bool(done[:, -1].all()):
                last = int((~done).sum(1).max()) + 1   # every row has ended by here
                new = new[:, :last]
        return torch.cat([ids, new], dim=1)

    def _speculative_generate(self, ids, int4, max_new_tokens=None, generator=None,
                              past_key_values=None, **kwargs):
        from .kv_cache import RW4KVCache
        from .speculative import SamplingParams, SpeculativeDecoder
        gc = self.model.generation_config
        if max_new_tokens is None:
            max_new_tokens = getattr(gc, "max_new_tokens", None) or 20
        eos = kwargs.get("eos_token_id", getattr(gc, "eos_token_id", None))
        sampling = SamplingParams.from_generation(gc, **{k: kwargs.get(k) for k in (
            "do_sample", "temperature", "top_k", "top_p")})
        dec = SpeculativeDecoder(self, self.draft(), self.lookahead, self.max_lookahead,
                                 new_cache=(lambda: RW4KVCache(fused=True, causal_chunks=True))
                                 if int4 else None,
                                 eos_token_id=eos)
        out = dec.generate(ids.to(self.device), int(max_new_tokens), sampling, generator,
                           past_key_values, int(kwargs.get("min_new_tokens") or 0))
        self.speculation = dec.stats
        return out

    def forward(self, *args, **kwargs):
        return self.model(*args, **kwargs)

    __call__ = forward

    def stats(self):
        out = {"streaming": self.streamer.stats() if self.streamer else None,
               "staging_pool": None}
        storage = getattr(self.streamer, "storage", None) if self.streamer else None
        if storage is not None and getattr(storage, "pool", None) is not None:
            # pinned host memory of the storage tier's staging leases, beside host_budget
            out["staging_pool"] = storage.pool.stats()
        return out

    def close(self):
        if self.streamer is not None:
            self.streamer.close()
            self.streamer = None


class AutoModel:
    """``AutoModel.from_pretrained(path, **knobs) -> RocketModel`` (``rocketllm/auto_model.py``)."""

    def __init__(self):
        raise EnvironmentError("use AutoModel.from_pretrained(path)")

    @classmethod
    def from_pretrained(cls, pretrained_model_name_or_path, *args, **kwargs):
        return RocketModel(pretrained_model_name_or_path, *args, **kwargs)

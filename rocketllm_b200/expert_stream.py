"""Per-expert streaming of routed experts (the reference's fused expert-row reads and expert
residency: ``rocketllm/base.py:1375-1464``, ``rocketllm/moe/expert_cache.py:261-316``).

When an RW4 mixture-of-experts model does not fit the VRAM budget, each expert of each layer is
packed once into its own pinned host blob (gate/up and down codes, fp16 scales and zeros at
256-byte aligned offsets).  The device keeps a cache of expert slots.  In a streamed experts
forward the routing is permuted on the device, the routed set is read back (one device->host sync
per MoE layer, as the reference's ``.tolist()``), the sends of every routed expert that is not
resident are issued together on the copy streams (``on_router``), the token gather runs meanwhile,
and the grouped RW4 GEMV waits (device-side) for exactly those sends.  Experts no token routed to
never cross PCIe.  Which resident expert gives its slot up is the reference's expert policy, LFU
with aging (:class:`ExpertSlotCache`), never one holding an expert of the running layer; a send
into a slot is ordered after all compute already queued, so the previous occupant's last reader has
finished before its bytes are overwritten.

:class:`DeviceExpertStreamer` does the same with the routing decision on the device: nothing on the
host reads the routed set (see its docstring).
"""
import collections
import types

import torch

from . import kernels

ALIGN = 256
_NAMES = ("gate_up_proj", "down_proj")
_SUFFIXES = ("_packed", "_scale", "_zero_point")


def is_rw4_experts(module):
    return bool(getattr(module, "rw4", False))


def expert_tensors(module, e):
    """The six tensors of expert ``e`` of an RW4 stacked-experts module, in blob order."""
    return [getattr(module, name + sfx)[e] for name in _NAMES for sfx in _SUFFIXES]


class _ExpertBlob:
    __slots__ = ("host", "entries", "nbytes")

    def __init__(self, tensors):
        self.entries, off = [], 0
        for t in tensors:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            self.entries.append((t.dtype, tuple(t.shape), off))
            off += t.numel() * t.element_size()
        self.nbytes = (off + ALIGN - 1) // ALIGN * ALIGN
        self.host = torch.empty(self.nbytes, dtype=torch.uint8).pin_memory()
        for (dtype, shape, o), t in zip(self.entries, tensors):
            n = t.numel() * t.element_size()
            self.host[o:o + n].copy_(t.detach().contiguous().view(-1).view(torch.uint8))

    def views(self, slot):
        out = []
        for dtype, shape, off in self.entries:
            n = 1
            for d in shape:
                n *= d
            size = n * torch.empty((), dtype=dtype).element_size()
            out.append(slot[off:off + size].view(dtype).view(shape))
        return out


def expert_blob_bytes(module):
    """Bytes of one expert's blob (the device slot size it needs)."""
    off = 0
    for t in expert_tensors(module, 0):
        off = (off + ALIGN - 1) // ALIGN * ALIGN + t.numel() * t.element_size()
    return (off + ALIGN - 1) // ALIGN * ALIGN


class ExpertSlotCache:
    """Which device slot holds which expert, and which resident expert gives way to a routed one.

    ``policy="lfu"`` is the reference's expert policy (``rocketllm/memory/cache.py``: ``_touch``
    434-441, ``_age`` 443-453, ``_expert_victims`` 484-493, ``acquire`` 201-250): each routed use
    of an expert adds one to its count, every ``aging_interval``-th use halves every count, and the
    victim is the resident expert with the smallest count, ties to the one admitted first.  The
    victim is chosen before the incoming expert's use is counted, as ``acquire`` makes room before
    it touches.  Counts and admission order outlive an eviction, because the expert's pinned host
    blob stays, as an entry demoted to the reference's host tier keeps them (``cache.py:518-538``).
    ``policy="lru"`` recycles the least recently used slot instead (the device-routed default).
    Either way a free slot goes first, lowest index first, and no slot holding an expert of
    ``protect`` (the running layer's routed set, which one grouped launch reads at once, as the
    reference's refcount keeps an acquired entry on the device) is ever recycled.
    """

    def __init__(self, num_slots, policy="lfu", aging_interval=4096):
        if policy not in ("lfu", "lru"):
            raise ValueError(f"expert cache policy {policy!r}: 'lfu' or 'lru'")
        if num_slots < 1:
            raise ValueError(f"{num_slots} expert slots")
        self.policy = policy
        self.aging_interval = max(1, int(aging_interval))
        self.owner = [None] * num_slots    # slot -> key
        self.where = {}                    # key -> slot
        self.uses = {}                     # key -> aged use count (kept across evictions)
        self.admitted = {}                 # key -> first-admission ordinal (kept likewise)
        self.last_use = {}                 # key -> ordinal of its latest use
        self.accesses = 0
        self.agings = 0

    def _touch(self, key):
        self.accesses += 1
        self.last_use[key] = self.accesses
        self.uses[key] = self.uses.get(key, 0.0) + 1.0
        if self.accesses % self.aging_interval == 0:
            for k in self.uses:
                self.uses[k] *= 0.5
            self.agings += 1

    def _victim_slot(self, protect):
        for s, key in enumerate(self.owner):
            if key is None:
                return s
        candidates = [k for k in self.where if k not in protect]
        if not candidates:
            raise RuntimeError("no expert slot can be recycled")
        if self.policy == "lfu":
            key = min(candidates, key=lambda k: (self.uses[k], self.admitted[k]))
        else:
            key = min(candidates, key=self.last_use.__getitem__)
        return self.where[key]

    def claim(self, key, protect=()):
        """Count one use of ``key`` and give it a slot: ``(slot, hit, evicted)``.  ``hit`` is True
        when it was resident already; ``evicted`` is the key that gave the slot up, or None."""
        if key in self.where:
            self._touch(key)
            return self.where[key], True, None
        s = self._victim_slot(protect)
        old = self.owner[s]
        if old is not None:
            del self.where[old]
        self.admitted.setdefault(key, len(self.admitted))
        self.owner[s] = key
        self.where[key] = s
        self._touch(key)
        return s, False, old


class ExpertStreamer:
    """Routed experts of ``moe`` (a list of ``(layer_index, experts_module)``) streamed from pinned
    host blobs into ``num_slots`` device slots through ``xfer`` (a ``WeightTransfer``); which
    resident expert gives way follows ``policy`` (:class:`ExpertSlotCache`)."""

    def __init__(self, moe, device, num_slots, xfer, policy="lfu", aging_interval=4096):
        self.device = torch.device(device)
        self.xfer = xfer
        self.blobs = {}
        self.num_experts = {}
        for layer, module in moe:
            e_count = module.gate_up_proj_packed.shape[0]
            self.num_experts[layer] = e_count
            for e in range(e_count):
                self.blobs[(layer, e)] = _ExpertBlob(expert_tensors(module, e))
        max_e = max(self.num_experts.values())
        if num_slots < max_e:
            raise ValueError(f"{num_slots} expert slots cannot hold one layer's {max_e} experts")
        self.slot_bytes = max(b.nbytes for b in self.blobs.values())
        self.slots = [torch.empty(self.slot_bytes, dtype=torch.uint8, device=self.device)
                      for _ in range(min(num_slots, len(self.blobs)))]
        self.cache = ExpertSlotCache(len(self.slots), policy, aging_interval)
        self.where = self.cache.where             # (layer, expert) -> slot
        self.tickets = {}
        self.frequency = collections.Counter()    # routed count per (layer, expert)
        self.firings = 0                          # on_router calls (one per MoE layer call)
        self.fetches = 0
        self.hits = 0
        self.bytes = 0
        for layer, module in moe:
            # the stacked tensors now live in the host blobs; the module keeps empty stand-ins
            for name in _NAMES:
                for sfx in _SUFFIXES:
                    p = getattr(module, name + sfx)
                    module._parameters[name + sfx] = torch.nn.Parameter(
                        torch.empty((0,) + tuple(p.shape[1:]), dtype=p.dtype, device=self.device),
                        requires_grad=False)
            module._rw4_stream = (self, layer)
            module.forward = types.MethodType(streamed_experts_forward, module)

    # -- residency ---------------------------------------------------------------------------------

    def on_router(self, layer, selected, compute):
        """The layer's router chose ``selected``: issue the sends of the ones not resident, all
        together, ordered after the compute queued on ``compute``.  Returns how many started."""
        protect = {(layer, e) for e in selected}
        started = 0
        self.firings += 1
        for e in selected:
            key = (layer, e)
            self.frequency[key] += 1
            s, hit, old = self.cache.claim(key, protect)
            if hit:
                self.hits += 1
                continue
            if old is not None:
                self.tickets.pop(old, None)
            blob = self.blobs[key]
            self.tickets[key] = self.xfer.send_buffer(blob.host, out=self.slots[s][:blob.nbytes],
                                                      after=compute)
            self.fetches += 1
            self.bytes += blob.nbytes
            started += 1
        return started

    def wait(self, layer, selected, compute):
        """Make ``compute`` wait (device-side) for the sends of the selected experts."""
        for e in selected:
            handle = self.tickets.pop((layer, e), None)
            if handle is not None:
                handle.resolve(compute)

    def triples(self, layer, selected):
        """Per-expert ``(packed, scale, zero)`` lists for gate/up and down; experts outside
        ``selected`` get the first selected expert's views (the kernel never reads them)."""
        views = {e: self.blobs[(layer, e)].views(self.slots[self.where[(layer, e)]])
                 for e in selected}
        first = views[selected[0]]
        gate_up, down = [], []
        for e in range(self.num_experts[layer]):
            v = views.get(e, first)
            gate_up.append(tuple(v[0:3]))
            down.append(tuple(v[3:6]))
        return gate_up, down

    def stats(self):
        return {"expert_slots": len(self.slots), "slot_bytes": self.slot_bytes,
                "fetches": self.fetches, "hits": self.hits, "bytes": self.bytes,
                "resident": len(self.where), "policy": self.cache.policy,
                "agings": self.cache.agings,
                "routing": routing_distribution(self.frequency, len(self.blobs), self.firings)}


def routing_distribution(frequency, experts, firings):
    """How skewed the routing was -- what an expert cache's hit rate rests on -- from lifetime
    selection counts (``frequency``: key -> count over ``experts`` keys in all; ``firings``: router
    calls).  The reference's benchmark reports the same figures (``rocketllm/moe/expert_cache.py:
    171-200``): the share of selections taken by the most popular expert and by the most popular
    tenth (beside the tenth's share under uniform routing), and the Gini coefficient of the counts
    (0: uniform; (n-1)/n: one expert takes everything), here by its sorted-rank formula
    G = 2 * sum_i(i * x_i) / (n * sum(x)) - (n + 1) / n over the ascending counts x_1..x_n."""
    counts = sorted(frequency.values(), reverse=True)
    counts += [0] * max(0, experts - len(counts))
    total = sum(counts)
    n = len(counts)
    out = {"experts": n, "touched": sum(1 for c in counts if c), "firings": firings,
           "selections": total,
           "distinct_per_firing": total / firings if firings else 0.0}
    if not total:
        out.update(top_1_share=0.0, top_10pct_share=0.0, uniform_share=0.0, gini=0.0)
        return out
    head = max(1, n // 10)
    ascending = counts[::-1]
    out["top_1_share"] = counts[0] / total
    out["top_10pct_share"] = sum(counts[:head]) / total
    out["uniform_share"] = head / n
    out["gini"] = 2.0 * sum((i + 1) * x for i, x in enumerate(ascending)) / (n * total) \
        - (n + 1) / n
    return out


def streamed_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """``rw4_experts_forward`` for a module whose experts stream (same signature and result)."""
    streamer, layer = self._rw4_stream
    t, h = hidden_states.shape
    k = top_k_index.shape[1]
    x = hidden_states if hidden_states.dtype == torch.bfloat16 else hidden_states.to(torch.bfloat16)
    if not x.is_contiguous():
        x = x.contiguous()
    idx = top_k_index.to(torch.int64).contiguous()
    w = top_k_weights.contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    n_exp = streamer.num_experts[layer]
    compute = torch.cuda.current_stream(streamer.device)
    perm, inv, offsets = kernels.moe_permute(idx, n_exp)
    # rows per expert: a token's top-k experts are distinct, so one token gives each at most one
    # row (the one-row fp16 kernel); otherwise bound by all of the token-slot pairs
    rows = 1 if t == 1 else t * k
    counts = offsets.cpu().tolist()          # the routed set: one device->host sync per layer
    selected = [e for e in range(n_exp) if counts[e + 1] > counts[e]]
    if not selected:
        return torch.zeros_like(hidden_states)
    streamer.on_router(layer, selected, compute)
    xp = kernels.moe_gather(x, perm, k)      # runs while the experts cross PCIe
    streamer.wait(layer, selected, compute)
    gate_up, down = streamer.triples(layer, selected)
    act = kernels.moe_grouped(xp, offsets, gate_up, act=1, max_rows=rows)
    yp = kernels.moe_grouped(act, offsets, down, act=0, max_rows=rows)
    out = kernels.moe_combine(yp, inv, idx, w)
    return out if hidden_states.dtype == torch.bfloat16 else out.to(hidden_states.dtype)


class DeviceExpertStreamer:
    """Routed experts of ``moe`` streamed with device-side routing (no host sync per MoE layer).

    The experts' blobs stay in pinned host memory (mapped into the device address space); the
    device keeps ``num_slots`` expert slots (<= 80: one TMA tensor-map set per slot travels as
    kernel parameters) and the residency tables.  In a forward, everything runs on the compute
    stream without the host waiting: permute -> residency kernel (claims resident slots, assigns
    free / least-recently-used ones to the others, lists them) -> copy kernel (reads the listed
    blobs over PCIe into their slots) -> gather -> grouped GEMVs that reach each expert's weights
    through its slot index -> combine.  ``policy``: ``"lru"`` (least recently used: a free slot
    first, never a slot the running layer's routed experts hold; ties between slots last used in
    the same call go to the lower slot index) or ``"lfu"``, the reference's LFU with aging, the
    same decisions as :class:`ExpertSlotCache` with whole-set protection (an aged count and an
    admission ordinal per expert in device tables, ``rw4_expert_residency_lfu``).
    """

    MAX_SLOTS = 80

    def __init__(self, moe, device, num_slots, ctas_per_expert=64, policy="lru",
                 aging_interval=4096):
        if policy not in ("lfu", "lru"):
            raise ValueError(f"expert cache policy {policy!r}: 'lfu' or 'lru'")
        self.policy = policy
        self.aging_interval = max(1, int(aging_interval))
        self.device = torch.device(device)
        counts = {m.gate_up_proj_packed.shape[0] for _, m in moe}
        shapes = {(tuple(m.gate_up_proj_packed.shape[1:]), tuple(m.down_proj_packed.shape[1:]))
                  for _, m in moe}
        if len(counts) != 1 or len(shapes) != 1:
            raise ValueError("device-side routing needs every MoE layer to have the same experts")
        self.num_experts = counts.pop()
        self.index = {layer: i for i, (layer, _) in enumerate(moe)}
        e_count = self.num_experts
        slots = min(int(num_slots), self.MAX_SLOTS, len(moe) * e_count)
        if slots < e_count:
            raise ValueError(f"{slots} expert slots cannot hold one layer's {e_count} experts")
        self.blobs = []
        host = []
        for layer, module in moe:
            for e in range(e_count):
                blob = _ExpertBlob(expert_tensors(module, e))
                if blob.host.data_ptr() % 16:
                    raise RuntimeError("pinned expert blob is not 16-byte aligned")
                host.append(kernels.host_ptr_device(blob.host.data_ptr()))
                self.blobs.append(blob)
        self.blob_bytes = self.blobs[0].nbytes
        self.host_ptrs = torch.tensor(host, dtype=torch.int64, device=self.device)
        self.slots = torch.empty(slots * self.blob_bytes, dtype=torch.uint8, device=self.device)
        entries = self.blobs[0].entries          # every blob has the same layout
        base = self.slots.data_ptr()
        ptr = [[base + s * self.blob_bytes + off for s in range(slots)]
               for (_, _, off) in entries]
        gu_shape, dn_shape = shapes.pop()
        n_gu, k_gu = gu_shape[0], gu_shape[1] * 2
        n_dn, k_dn = dn_shape[0], dn_shape[1] * 2
        self.gate_up_maps = kernels.SlotMaps(ptr[0], ptr[1], ptr[2], k_gu, n_gu, act=1)
        self.down_maps = kernels.SlotMaps(ptr[3], ptr[4], ptr[5], k_dn, n_dn, act=0)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.where = torch.full((len(moe) * e_count,), -1, **i32)
        self.owner = torch.full((slots,), -1, **i32)
        self.stamp = torch.zeros(slots, **i32)
        self.clock = torch.zeros(1, **i32)
        keys = len(moe) * e_count
        self.uses = torch.zeros(keys if policy == "lfu" else 0, dtype=torch.float64,
                                device=self.device)
        self.admitted = torch.full((keys if policy == "lfu" else 0,), -1, **i32)
        self.lfu_state = torch.zeros(3, dtype=torch.int64, device=self.device)
        self.counters = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.slot_of = torch.empty(e_count, **i32)
        self.copy_expert = torch.empty(e_count, **i32)
        self.copy_slot = torch.empty(e_count, **i32)
        self.ncopy = torch.zeros(1, **i32)
        self.ctas_per_expert = ctas_per_expert
        for layer, module in moe:
            for name in _NAMES:
                for sfx in _SUFFIXES:
                    p = getattr(module, name + sfx)
                    module._parameters[name + sfx] = torch.nn.Parameter(
                        torch.empty((0,) + tuple(p.shape[1:]), dtype=p.dtype, device=self.device),
                        requires_grad=False)
            module._rw4_device_stream = (self, self.index[layer])
            module.forward = types.MethodType(device_streamed_experts_forward, module)

    def stats(self):
        """Counters (reading them synchronises the device)."""
        hits, fetches = self.counters.tolist()
        return {"expert_slots": self.owner.numel(), "slot_bytes": self.blob_bytes,
                "fetches": fetches, "hits": hits, "bytes": fetches * self.blob_bytes,
                "resident": int((self.owner >= 0).sum()), "routing": "device",
                "policy": self.policy, "agings": int(self.lfu_state[2])}

    def close(self):
        self.gate_up_maps.close()
        self.down_maps.close()


def device_streamed_experts_forward(self, hidden_states, top_k_index, top_k_weights):
    """``rw4_experts_forward`` with device-side routing into the expert cache (same result)."""
    st, li = self._rw4_device_stream
    t, h = hidden_states.shape
    k = top_k_index.shape[1]
    x = hidden_states if hidden_states.dtype == torch.bfloat16 else hidden_states.to(torch.bfloat16)
    if not x.is_contiguous():
        x = x.contiguous()
    idx = top_k_index.to(torch.int64).contiguous()
    w = top_k_weights.contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    perm, inv, offsets = kernels.moe_permute(idx, st.num_experts)
    if st.policy == "lfu":
        kernels.expert_residency_lfu(offsets, li, st.where, st.owner, st.uses, st.admitted,
                                     st.lfu_state, st.aging_interval, st.slot_of, st.copy_expert,
                                     st.copy_slot, st.ncopy, st.counters)
    else:
        kernels.expert_residency(offsets, li, st.where, st.owner, st.stamp, st.clock, st.slot_of,
                                 st.copy_expert, st.copy_slot, st.ncopy, st.counters)
    kernels.expert_copy(st.copy_expert, st.copy_slot, st.ncopy, li, st.num_experts, st.host_ptrs,
                        st.blob_bytes, st.slots, st.blob_bytes, st.ctas_per_expert)
    rows = 1 if t == 1 else t * k
    xp = kernels.moe_gather(x, perm, k)
    act = kernels.moe_grouped_slots(xp, offsets, st.gate_up_maps, st.slot_of, max_rows=rows)
    yp = kernels.moe_grouped_slots(act, offsets, st.down_maps, st.slot_of, max_rows=rows)
    out = kernels.moe_combine(yp, inv, idx, w)
    return out if hidden_states.dtype == torch.bfloat16 else out.to(hidden_states.dtype)

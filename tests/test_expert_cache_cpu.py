"""Expert residency on CPU: the streamed-expert slot cache against the reference's own weight cache.

``golden/reference_expert_cache.npz`` holds routing traces replayed through the reference's
``TieredWeightCache`` (``rocketllm/memory/cache.py``; made by ``golden/make_expert_cache_golden.py``):
per firing, which acquires hit the device and which experts were resident afterwards.  The LFU
policy with aging must reproduce them exactly under the reference's protection rule, and the same
residency with no fewer hits under the streamer's (the whole routed set); the reference's own
expert-policy cases
(``tests/test_cache_policy.py:381-439``) are restated below, and the host streamer's ``on_router``
is driven with a fake transfer engine.
"""
import collections
import os

import numpy as np
import pytest
import torch

from rocketllm_b200.expert_stream import ExpertSlotCache, ExpertStreamer

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_expert_cache.npz")


def replay(d, name, policy, whole_set=False):
    """Replay a trace.  ``whole_set=False`` protects, while an expert is placed, the experts of the
    firing acquired so far (the reference's refcount); ``whole_set=True`` protects the whole routed
    set (what the streamer does: one grouped launch reads them all)."""
    layers, experts, top_k, slots, aging = (int(x) for x in d[f"{name}.params"])
    cache = ExpertSlotCache(slots, policy, aging)
    hits, resident = [], []
    for layer, sel in zip(d[f"{name}.layer"], d[f"{name}.selected"]):
        keys = [(int(layer), int(e)) for e in sel]
        hits.append([cache.claim(k, set(keys if whole_set else keys[:j + 1]))[1]
                     for j, k in enumerate(keys)])
        row = np.zeros(layers * experts, dtype=np.uint8)
        for (l, e) in cache.where:
            row[l * experts + e] = 1
        resident.append(row)
    return np.array(hits, dtype=np.uint8), np.stack(resident), cache


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_lfu_with_aging_reproduces_the_reference_cache(golden):
    for name in golden["cases"]:
        hits, resident, cache = replay(golden, str(name), "lfu")
        np.testing.assert_array_equal(hits, golden[f"{name}.hits"], err_msg=str(name))
        np.testing.assert_array_equal(resident, golden[f"{name}.resident"], err_msg=str(name))
        assert cache.agings == int(golden[f"{name}.agings"]), name


def test_protecting_the_whole_routed_set_only_saves_reads(golden):
    """The reference may evict a routed expert not yet acquired and read it straight back; with
    counts and admission order kept across evictions, that detour ends in the same residency.  So
    protecting the whole set leaves every firing's resident set as the reference's, and only ever
    turns a miss into a hit."""
    saved = 0
    for name in golden["cases"]:
        hits, resident, _ = replay(golden, str(name), "lfu", whole_set=True)
        np.testing.assert_array_equal(resident, golden[f"{name}.resident"], err_msg=str(name))
        ref = golden[f"{name}.hits"]
        assert (hits >= ref).all(), name
        saved += int(hits.sum() - ref.sum())
    assert saved > 0


def test_the_traces_tell_lfu_from_lru(golden):
    """The pin means something: recency alone gives other residency on these traces."""
    differ = 0
    for name in golden["cases"]:
        hits, resident, _ = replay(golden, str(name), "lru")
        differ += not np.array_equal(resident, golden[f"{name}.resident"])
    assert differ >= 2


def test_the_least_popular_expert_is_evicted_first():
    """``test_cache_policy.py:410-418`` restated: 3 slots, uses 5 / 1 / 3, a fourth expert."""
    c = ExpertSlotCache(3)
    for e, n in ((1, 5), (2, 1), (3, 3)):
        for _ in range(n):
            c.claim((0, e))
    slot, hit, evicted = c.claim((0, 4))
    assert (hit, evicted) == (False, (0, 2)) and c.where[(0, 4)] == slot
    assert (0, 1) in c.where and (0, 3) in c.where


def test_aging_lets_a_newly_hot_expert_overtake_an_old_favourite():
    """``test_cache_policy.py:429-437`` restated, plus the overtaking itself."""
    c = ExpertSlotCache(2, aging_interval=4)
    for _ in range(8):
        c.claim((0, 1))
    before = c.uses[(0, 1)]
    for _ in range(8):
        c.claim((0, 2))
    assert c.uses[(0, 1)] < before and c.agings == 4
    assert c.uses[(0, 2)] > c.uses[(0, 1)]
    c.claim((0, 3))                                   # the old favourite gives way
    assert (0, 1) not in c.where and (0, 2) in c.where
    nc = ExpertSlotCache(2, aging_interval=1 << 20)   # without aging it would have stayed
    for e in (1, 2):
        for _ in range(8 + (e == 1)):
            nc.claim((0, e))
    nc.claim((0, 3))
    assert (0, 1) in nc.where and (0, 2) not in nc.where


def test_counts_outlive_an_eviction():
    """An evicted expert keeps its count (its host copy stays), so it returns ranked by it."""
    c = ExpertSlotCache(2, aging_interval=1 << 20)
    for _ in range(5):
        c.claim((0, 0))
    c.claim((0, 1))
    c.claim((0, 2), protect={(0, 2), (0, 1)})         # (0, 0) must go: the rest are protected
    assert (0, 0) not in c.where and c.uses[(0, 0)] == 5.0
    c.claim((0, 0))                                   # back, with 6: (0, 1) or (0, 2) goes next
    c.claim((0, 3))
    assert (0, 0) in c.where


def test_ties_go_to_the_expert_admitted_first():
    c = ExpertSlotCache(3)
    for e in (5, 3, 4):
        c.claim((1, e))
    assert c.claim((1, 9))[2] == (1, 5)
    assert c.claim((1, 8))[2] == (1, 3)


def test_a_protected_slot_is_never_recycled():
    c = ExpertSlotCache(2)
    c.claim((0, 0))
    c.claim((0, 1))
    for _ in range(3):
        c.claim((0, 0))
    assert c.claim((0, 2), protect={(0, 1), (0, 2)})[2] == (0, 0)   # the popular one, protected out
    with pytest.raises(RuntimeError, match="no expert slot"):
        c.claim((0, 3), protect={(0, 1), (0, 2), (0, 3)})
    with pytest.raises(ValueError):
        ExpertSlotCache(2, policy="mru")


def test_lru_recycles_the_least_recently_used():
    c = ExpertSlotCache(2, policy="lru")
    for _ in range(4):
        c.claim((0, 0))
    c.claim((0, 1))
    assert c.claim((0, 2))[2] == (0, 0)


class _FakeXfer:
    def __init__(self):
        self.sends = []

    def send_buffer(self, host, out, after=None):
        self.sends.append((int(host[0]), out.data_ptr()))
        return _Handle()


class _Handle:
    def resolve(self, stream):
        pass


def _streamer(num_slots, layers=2, experts=4, policy="lfu", aging=4096):
    """An ExpertStreamer without pinned blobs or a device: its residency and send wiring only."""
    s = object.__new__(ExpertStreamer)
    s.xfer = _FakeXfer()
    s.slots = [torch.zeros(64, dtype=torch.uint8) for _ in range(num_slots)]
    s.blobs = {}
    for layer in range(layers):
        for e in range(experts):
            host = torch.full((64,), layer * experts + e, dtype=torch.uint8)
            s.blobs[(layer, e)] = type("Blob", (), {"host": host, "nbytes": 64})()
    s.cache = ExpertSlotCache(num_slots, policy, aging)
    s.where = s.cache.where
    s.tickets, s.frequency = {}, collections.Counter()
    s.fetches = s.hits = s.bytes = s.firings = 0
    return s


def test_on_router_sends_only_what_is_missing_into_the_slot_it_was_given():
    s = _streamer(3)
    assert s.on_router(0, [0, 2], None) == 2
    assert s.on_router(0, [0, 2], None) == 0 and s.hits == 2
    assert s.on_router(1, [1, 3], None) == 2                 # one free slot, one recycled
    ptr = {sl.data_ptr(): i for i, sl in enumerate(s.slots)}
    sent = {blob: ptr[p] for blob, p in s.xfer.sends}
    assert sent[0] != sent[2]
    # (0, 2) and (0, 0) tied at two uses: the one admitted first gave its slot to (1, 3)
    assert (0, 0) not in s.where and s.where[(1, 3)] == sent[0]
    assert s.where[(1, 1)] == sent[1 * 4 + 1] and s.where[(0, 2)] == sent[2]
    assert (0, 0) not in s.tickets and s.fetches == 4 and s.bytes == 4 * 64
    assert s.frequency[(0, 0)] == 2


class _LfuTables:
    """Host tables for ``rw4_expert_residency_lfu_host``: the residency kernel's own step compiled
    for the host (one definition, ``csrc/rw4_residency.cuh``)."""

    def __init__(self, layers, experts, slots, aging):
        keys = layers * experts
        self.E, self.aging = experts, aging
        self.where = torch.full((keys,), -1, dtype=torch.int32)
        self.owner = torch.full((slots,), -1, dtype=torch.int32)
        self.uses = torch.zeros(keys, dtype=torch.float64)
        self.admitted = torch.full((keys,), -1, dtype=torch.int32)
        self.state = torch.zeros(3, dtype=torch.int64)
        self.counters = torch.zeros(2, dtype=torch.int64)
        self.slot_of = torch.empty(experts, dtype=torch.int32)
        self.copy_expert = torch.empty(experts, dtype=torch.int32)
        self.copy_slot = torch.empty(experts, dtype=torch.int32)
        self.ncopy = torch.zeros(1, dtype=torch.int32)

    def step(self, layer, routed):
        from rocketllm_b200 import _lib
        counts = torch.zeros(self.E, dtype=torch.int32)
        counts[list(routed)] = 1
        offsets = torch.zeros(self.E + 1, dtype=torch.int32)
        offsets[1:] = torch.cumsum(counts, 0)
        _lib.call("rw4_expert_residency_lfu_host", offsets.data_ptr(), self.E, int(layer),
                  self.where.numel(), self.where.data_ptr(), self.owner.data_ptr(),
                  self.owner.numel(), self.uses.data_ptr(), self.admitted.data_ptr(),
                  self.state.data_ptr(), self.aging, self.slot_of.data_ptr(),
                  self.copy_expert.data_ptr(), self.copy_slot.data_ptr(), self.ncopy.data_ptr(),
                  self.counters.data_ptr())
        n = int(self.ncopy[0])
        return (self.slot_of.tolist(),
                list(zip(self.copy_expert.tolist()[:n], self.copy_slot.tolist()[:n])))


def _same_step(t, cache, layer, routed):
    """One firing through the compiled step and through ExpertSlotCache: same slots, same copies,
    bit-identical counts and admission order."""
    slot_of, copies = t.step(layer, routed)
    protect = {(layer, e) for e in routed}
    want_copies = []
    for e in routed:
        s, hit, _ = cache.claim((layer, e), protect)
        if not hit:
            want_copies.append((e, s))
    assert copies == want_copies
    assert [slot_of[e] for e in routed] == [cache.where[(layer, e)] for e in routed]
    assert all(slot_of[e] == -1 for e in range(t.E) if e not in routed)
    keys = t.where.numel()
    assert t.owner.tolist() == [-1 if k is None else k[0] * t.E + k[1] for k in cache.owner]
    uses = [cache.uses.get((k // t.E, k % t.E), 0.0) for k in range(keys)]
    assert t.uses.tolist() == uses                                  # exact: same halvings
    assert t.admitted.tolist() == [cache.admitted.get((k // t.E, k % t.E), -1)
                                   for k in range(keys)]
    assert t.state.tolist() == [cache.accesses, len(cache.admitted), cache.agings]


def test_the_residency_kernels_lfu_step_is_the_policy_on_the_golden_traces(golden):
    for name in golden["cases"]:
        layers, experts, top_k, slots, aging = (int(x) for x in golden[f"{name}.params"])
        t = _LfuTables(layers, experts, slots, aging)
        cache = ExpertSlotCache(slots, "lfu", aging)
        hits = 0
        for layer, sel in zip(golden[f"{name}.layer"], golden[f"{name}.selected"]):
            before = int(t.counters[0])
            _same_step(t, cache, int(layer), [int(e) for e in sel])
            hits += int(t.counters[0]) - before
        _, resident, _ = replay(golden, str(name), "lfu", whole_set=True)
        rows = np.zeros(layers * experts, dtype=np.uint8)
        rows[[k for k in t.owner.tolist() if k >= 0]] = 1
        np.testing.assert_array_equal(rows, resident[-1])
        assert hits >= int(golden[f"{name}.hits"].sum())


@pytest.mark.parametrize("seed", range(4))
def test_the_residency_kernels_lfu_step_is_the_policy_on_random_routings(seed):
    rng = np.random.default_rng(seed)
    layers, experts = 3, int(rng.integers(4, 17))
    slots = int(rng.integers(experts, layers * experts + 3))
    aging = int(rng.integers(1, 40))
    t = _LfuTables(layers, experts, slots, aging)
    cache = ExpertSlotCache(slots, "lfu", aging)
    for _ in range(120):
        layer = int(rng.integers(0, layers))
        k = int(rng.integers(1, experts + 1))
        routed = sorted(rng.choice(experts, size=k, replace=False).tolist())
        _same_step(t, cache, layer, routed)


def test_the_host_lfu_step_rejects_what_it_cannot_place():
    """Three slots, all held by the layer's routed experts, and a fourth routed expert: no slot."""
    from rocketllm_b200 import _lib
    t = _LfuTables(2, 4, 3, 16)
    t.step(1, [0, 1, 2])
    with pytest.raises(_lib.RW4Error, match="found no slot"):
        t.step(1, [0, 1, 2, 3])
    with pytest.raises(_lib.RW4Error, match="RW4_EINVAL"):
        t.step(2, [0])                                   # layer 2 of a 2-layer table


def test_routing_distribution_figures():
    """The skew report (the reference's ``ExpertStats.distribution``): uniform routing has Gini 0
    and the top tenth at its uniform share; one expert taking everything has Gini (n-1)/n."""
    from rocketllm_b200.expert_stream import routing_distribution
    flat = routing_distribution(collections.Counter({(0, e): 5 for e in range(20)}), 20, 50)
    assert flat["gini"] == pytest.approx(0.0, abs=1e-12)
    assert flat["top_10pct_share"] == pytest.approx(flat["uniform_share"]) == pytest.approx(0.1)
    assert flat["distinct_per_firing"] == 2.0 and flat["touched"] == 20
    one = routing_distribution(collections.Counter({(1, 3): 7}), 20, 7)
    assert one["gini"] == pytest.approx(19 / 20) and one["top_1_share"] == 1.0
    assert one["touched"] == 1 and one["experts"] == 20
    empty = routing_distribution(collections.Counter(), 8, 0)
    assert empty["gini"] == 0.0 and empty["selections"] == 0
    s = _streamer(3)
    s.on_router(0, [0, 2], None)
    s.on_router(1, [2], None)
    got = routing_distribution(s.frequency, len(s.blobs), s.firings)
    assert got["firings"] == 2 and got["selections"] == 3 and got["experts"] == 8

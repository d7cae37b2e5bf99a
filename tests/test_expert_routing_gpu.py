"""Device-side routing into the expert cache (B200): the residency kernel follows the cache policy
exactly (checked against a step-by-step restatement over random routings), the copy kernel lands
every listed blob byte for byte, and a Mixtral-architecture RW4 model streaming its experts this way
produces exactly the resident model's logits and greedy tokens -- with no host read of the routing.
"""
import numpy as np
import pytest
import torch

from rocketllm_b200 import kernels
from rocketllm_b200.engine import AutoModel, RocketModel
from test_expert_stream_gpu import E, budget_for, checkpoint  # noqa: F401 - shared fixture

pytestmark = pytest.mark.gpu


def policy_step(routed, layer, n_exp, where, owner, stamp, clock):
    """One residency step restated: claim resident routed experts, then give each other routed
    expert the first free slot, else the least recently used slot not claimed in this step (lowest
    index on ties).  Mutates the tables; returns (slot_of, copies, hits)."""
    t = clock[0] = clock[0] + 1
    base = layer * n_exp
    slot_of = [-1] * n_exp
    hits = 0
    for e in routed:
        s = where[base + e]
        if s >= 0 and owner[s] == base + e:
            slot_of[e] = s
            stamp[s] = t
            hits += 1
    copies = []
    for e in routed:
        if slot_of[e] >= 0:
            continue
        best = -1
        for s in range(len(owner)):
            if owner[s] < 0:
                best = s
                break
            if stamp[s] != t and (best < 0 or stamp[s] < stamp[best]):
                best = s
        old = owner[best]
        if old >= 0:
            where[old] = -1
        owner[best] = base + e
        where[base + e] = best
        stamp[best] = t
        slot_of[e] = best
        copies.append((e, best))
    return slot_of, copies, hits


@pytest.mark.parametrize("slots", [8, 13, 24])
def test_residency_kernel_follows_the_policy(cuda, slots):
    n_exp, layers, steps = 8, 4, 60
    rng = np.random.default_rng(slots)
    dev = cuda
    i32 = dict(dtype=torch.int32, device=dev)
    where = torch.full((layers * n_exp,), -1, **i32)
    owner = torch.full((slots,), -1, **i32)
    stamp = torch.zeros(slots, **i32)
    clock = torch.zeros(1, **i32)
    counters = torch.zeros(2, dtype=torch.int64, device=dev)
    slot_of = torch.empty(n_exp, **i32)
    ce = torch.empty(n_exp, **i32)
    cs = torch.empty(n_exp, **i32)
    nc = torch.zeros(1, **i32)
    r_where, r_owner, r_stamp, r_clock = [-1] * (layers * n_exp), [-1] * slots, [0] * slots, [0]
    r_hits = r_fetch = 0
    for step in range(steps):
        layer = step % layers
        t = int(rng.integers(1, 4))                     # tokens routed in this layer call
        idx = np.stack([rng.choice(n_exp, 2, replace=False) for _ in range(t)])
        counts = np.bincount(idx.reshape(-1), minlength=n_exp)
        offsets = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), **i32)
        kernels.expert_residency(offsets, layer, where, owner, stamp, clock, slot_of, ce, cs, nc,
                                 counters)
        routed = [e for e in range(n_exp) if counts[e]]
        ref_slot, ref_copies, hits = policy_step(routed, layer, n_exp, r_where, r_owner, r_stamp,
                                                 r_clock)
        r_hits += hits
        r_fetch += len(ref_copies)
        n = int(nc.item())
        got = [s if counts[e] else -1 for e, s in enumerate(slot_of.tolist())]
        assert got == ref_slot, step
        assert list(zip(ce.tolist()[:n], cs.tolist()[:n])) == ref_copies, step
    assert where.tolist() == r_where and owner.tolist() == r_owner and stamp.tolist() == r_stamp
    assert counters.tolist() == [r_hits, r_fetch]
    assert kernels.device_status() == 0


@pytest.mark.parametrize("slots,aging", [(8, 5), (13, 4096), (24, 3)])
def test_lfu_residency_kernel_follows_the_policy(cuda, slots, aging):
    """The LFU-with-aging step on the device makes the host cache's decisions (whole routed set
    protected), with bit-identical aged counts."""
    from rocketllm_b200.expert_stream import ExpertSlotCache
    n_exp, layers, steps = 8, 4, 60
    rng = np.random.default_rng(100 + slots)
    i32 = dict(dtype=torch.int32, device=cuda)
    keys = layers * n_exp
    where = torch.full((keys,), -1, **i32)
    owner = torch.full((slots,), -1, **i32)
    uses = torch.zeros(keys, dtype=torch.float64, device=cuda)
    admitted = torch.full((keys,), -1, **i32)
    state = torch.zeros(3, dtype=torch.int64, device=cuda)
    counters = torch.zeros(2, dtype=torch.int64, device=cuda)
    slot_of = torch.empty(n_exp, **i32)
    ce = torch.empty(n_exp, **i32)
    cs = torch.empty(n_exp, **i32)
    nc = torch.zeros(1, **i32)
    cache = ExpertSlotCache(slots, "lfu", aging)
    r_hits = r_fetch = 0
    for step in range(steps):
        layer = int(rng.integers(0, layers))
        t = int(rng.integers(1, 4))
        idx = np.stack([rng.choice(n_exp, 2, replace=False) for _ in range(t)])
        counts = np.bincount(idx.reshape(-1), minlength=n_exp)
        offsets = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), **i32)
        kernels.expert_residency_lfu(offsets, layer, where, owner, uses, admitted, state, aging,
                                     slot_of, ce, cs, nc, counters)
        routed = [e for e in range(n_exp) if counts[e]]
        protect = {(layer, e) for e in routed}
        ref_copies = []
        for e in routed:
            s, hit, _ = cache.claim((layer, e), protect)
            r_hits += hit
            if not hit:
                ref_copies.append((e, s))
        r_fetch += len(ref_copies)
        n = int(nc.item())
        got = [s if counts[e] else -1 for e, s in enumerate(slot_of.tolist())]
        assert got == [cache.where[(layer, e)] if counts[e] else -1 for e in range(n_exp)], step
        assert list(zip(ce.tolist()[:n], cs.tolist()[:n])) == ref_copies, step
    assert owner.tolist() == [-1 if k is None else k[0] * n_exp + k[1] for k in cache.owner]
    assert uses.tolist() == [cache.uses.get((k // n_exp, k % n_exp), 0.0) for k in range(keys)]
    assert state.tolist() == [cache.accesses, len(cache.admitted), cache.agings]
    assert counters.tolist() == [r_hits, r_fetch]
    assert kernels.device_status() == 0


def test_copy_kernel_lands_listed_blobs(cuda):
    n_exp, blob = 4, 1 << 20
    host = [torch.randint(0, 256, (blob,), dtype=torch.uint8).pin_memory() for _ in range(n_exp)]
    ptrs = torch.tensor([kernels.host_ptr_device(h.data_ptr()) for h in host], dtype=torch.int64,
                        device=cuda)
    slots = torch.zeros(3 * blob, dtype=torch.uint8, device=cuda)
    i32 = dict(dtype=torch.int32, device=cuda)
    ce = torch.tensor([2, 0, 0, 0], **i32)
    cs = torch.tensor([1, 2, 0, 0], **i32)
    nc = torch.tensor([2], **i32)                          # two listed copies: 2 -> 1, 0 -> 2
    kernels.expert_copy(ce, cs, nc, 0, n_exp, ptrs, blob, slots, blob, ctas_per_expert=7)
    torch.cuda.synchronize()
    assert torch.equal(slots[blob:2 * blob].cpu(), host[2])
    assert torch.equal(slots[2 * blob:].cpu(), host[0])
    assert int(slots[:blob].sum()) == 0                    # unlisted slot untouched
    with pytest.raises(Exception):
        kernels.host_ptr_device(torch.zeros(16, dtype=torch.uint8).data_ptr())  # pageable


@pytest.mark.parametrize("slots,policy", [(E, "lru"), (2 * E, "lru"), (2 * E, "lfu")])
def test_device_routed_experts_equal_resident(checkpoint, slots, policy):  # noqa: F811
    ids = torch.randint(0, 2048, (1, 12), generator=torch.Generator().manual_seed(4)).cuda()
    resident = AutoModel.from_pretrained(checkpoint)
    budget = budget_for(resident.model, slots)
    streamed = RocketModel(checkpoint, vram_budget=budget, window=1, kv_cache="fp16",
                           expert_routing="device", expert_policy=policy)
    ex = streamed.streamer.experts
    assert type(ex).__name__ == "DeviceExpertStreamer"
    with torch.no_grad():
        assert torch.equal(resident(ids).logits, streamed(ids).logits)
        a = resident.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
        b = streamed.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
    assert torch.equal(a, b)
    st = ex.stats()
    assert st["routing"] == "device" and st["fetches"] > 0 and st["resident"] <= st["expert_slots"]
    assert st["policy"] == policy
    assert kernels.device_status() == 0
    streamed.close()

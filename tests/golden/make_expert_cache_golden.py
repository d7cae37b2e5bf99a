"""Generate ``reference_expert_cache.npz`` by running the REFERENCE weight cache on routing traces.

Run once in a checkout that has the RocketLLM sources (read-only is fine)::

    python tests/golden/make_expert_cache_golden.py /path/to/RocketLLM

It imports the reference's ``rocketllm/memory/cache.py`` (bound without the package ``__init__``,
as ``make_golden.py`` does) and drives its ``TieredWeightCache`` with seeded, skewed routing traces:
each firing acquires the layer's routed experts in ascending order, then releases them all (the
grouped launch reads the whole routed set at once, so none of it may be evicted while the layer is
being placed).  Every expert costs one byte, the device tier holds ``slots`` of them and the host
tier holds all of them (an expert's pinned host copy never leaves, as a streamed expert's pinned
blob never does).  Recorded per firing: which acquires hit the device tier and which experts are on
the device afterwards.
"""
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, layers, experts, top_k, slots, aging_interval, firings, zipf exponent, seed)
CASES = (("s12_age7", 2, 8, 2, 12, 7, 300, 1.2, 1),
         ("s5_age4096", 3, 6, 2, 5, 4096, 200, 1.0, 2),
         ("s20_age16_k4", 4, 16, 4, 20, 16, 400, 0.8, 3),
         ("s8_age3_uniform", 2, 8, 3, 8, 3, 250, 0.0, 4))


def bind_reference(root):
    for name, sub in (("rocketllm", "rocketllm"), ("rocketllm.memory", "rocketllm/memory")):
        if name not in sys.modules:
            pkg = types.ModuleType(name)
            pkg.__path__ = [os.path.join(root, sub)]
            sys.modules[name] = pkg
    sys.path.insert(0, root)
    from rocketllm.memory import cache
    return cache


def trace(layers, experts, top_k, firings, zipf, seed):
    """Seeded routing: per firing a layer (cyclic) and top_k distinct experts, Zipf-skewed with a
    per-layer permutation of which experts are popular; the ranking shifts halfway through."""
    rng = np.random.default_rng(seed)
    weight = 1.0 / np.arange(1, experts + 1) ** zipf
    perms = [rng.permutation(experts) for _ in range(layers)]
    rows = []
    for f in range(firings):
        layer = f % layers
        if f == firings // 2:
            perms = [rng.permutation(experts) for _ in range(layers)]
        p = np.empty(experts)
        p[perms[layer]] = weight / weight.sum()
        rows.append((layer, np.sort(rng.choice(experts, size=top_k, replace=False, p=p))))
    return rows


def main(root):
    cache_mod = bind_reference(root)
    out = {}
    for name, layers, experts, top_k, slots, aging, firings, zipf, seed in CASES:
        c = cache_mod.TieredWeightCache(fetch=lambda key: key, sizer=lambda key: 1,
                                        device_bytes=slots, host_bytes=layers * experts,
                                        window=1, aging_interval=aging)
        rows = trace(layers, experts, top_k, firings, zipf, seed)
        hits = np.zeros((firings, top_k), dtype=np.uint8)
        resident = np.zeros((firings, layers * experts), dtype=np.uint8)
        for f, (layer, sel) in enumerate(rows):
            keys = [(layer, cache_mod.expert_kind(int(e))) for e in sel]
            for j, key in enumerate(keys):
                before = c.stats["hits_device"]
                c.acquire(key)
                hits[f, j] = c.stats["hits_device"] > before
            for key in keys:
                c.release(key)
            for key in c.device.entries:
                resident[f, key[0] * experts + int(key[1].split(":")[1])] = 1
        out[f"{name}.params"] = np.array([layers, experts, top_k, slots, aging], dtype=np.int64)
        out[f"{name}.layer"] = np.array([r[0] for r in rows], dtype=np.int64)
        out[f"{name}.selected"] = np.stack([r[1] for r in rows]).astype(np.int64)
        out[f"{name}.hits"] = hits
        out[f"{name}.resident"] = resident
        out[f"{name}.agings"] = np.array(c.stats["agings"], dtype=np.int64)
    out["cases"] = np.array([c[0] for c in CASES])
    path = os.path.join(HERE, "reference_expert_cache.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(CASES)} traces")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ROCKETLLM_REFERENCE", "."))

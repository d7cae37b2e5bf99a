"""Generate ``reference_kv.npz`` by running the REFERENCE int4 KV cache and transformers' SDPA.

Run once in a checkout that has the RocketLLM sources (read-only is fine)::

    python tests/golden/make_kv_golden.py /path/to/RocketLLM

It feeds seeded bf16 keys / values through the reference's own ``QuantizedKVCache`` (a prefill
long enough to flush two groups at once, then decode steps until the window flushes again), and
records what ``update`` returned at the last step (the expanded history the model's
attention sees) plus the quantized blocks.  At the last step it also runs transformers' own
``sdpa_attention_forward`` (grouped-query, one query token) over that history.  The reference
package is bound without its ``__init__``, as ``make_golden.py`` does.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from make_golden import bind_reference, bits  # noqa: E402


def main(root):
    kv_cache, _ = bind_reference(root)
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    b, kvh, h, d = 1, 2, 8, 64
    prefill, steps = 260, 60
    g = torch.Generator().manual_seed(30)
    out = {"shape": np.array([b, kvh, h, d, prefill, steps], dtype=np.int64)}
    cache = kv_cache.QuantizedKVCache(kv_cache.KVCacheConfig(compute_dtype=torch.bfloat16))
    # keys with per-channel outliers (the reason K is grouped along tokens), values plain
    chan = 1.0 + 4.0 * (torch.rand(d, generator=g) > 0.9).float()

    def kv(t):
        k = (torch.randn(b, kvh, t, d, generator=g) * chan).to(torch.bfloat16)
        v = torch.randn(b, kvh, t, d, generator=g).to(torch.bfloat16)
        return k, v

    k, v = kv(prefill)
    out["k.0"], out["v.0"] = bits(k), bits(v)
    hk, hv = cache.update(k, v, 0)
    out["hist_len.0"] = np.int64(hk.shape[-2])
    for s in range(1, steps + 1):
        k, v = kv(1)
        out[f"k.{s}"], out[f"v.{s}"] = bits(k), bits(v)
        hk, hv = cache.update(k, v, 0)
    out["hist_k.last"], out["hist_v.last"] = bits(hk), bits(hv)
    kb, vb = cache._blocks[0]
    out["blocks"] = np.array([blk.length for blk in kb], dtype=np.int64)
    for i, (bk, bv) in enumerate(zip(kb, vb)):
        for name, blk in (("kb", bk), ("vb", bv)):
            out[f"{name}{i}.packed"] = bits(blk.packed)
            out[f"{name}{i}.scale"] = bits(blk.scale)
            out[f"{name}{i}.zero"] = bits(blk.zero)
    out["residual"] = np.int64(cache.key_cache[0].shape[-2])

    class Module:   # the attributes transformers' SDPA wrapper reads from an attention module
        num_key_value_groups = h // kvh
        is_causal = True
        training = False

    q = torch.randn(b, h, 1, d, generator=g).to(torch.bfloat16)
    attn, _ = sdpa_attention_forward(Module(), q, hk, hv, None, scaling=d ** -0.5)
    out["q"] = bits(q)
    out["attn"] = bits(attn)                       # [b, 1, h, d] bf16
    out["attn_f32"] = bits(sdpa_attention_forward(Module(), q.float(), hk.float(), hv.float(),
                                                  None, scaling=d ** -0.5)[0])
    path = os.path.join(HERE, "reference_kv.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ROCKETLLM_REFERENCE", "."))

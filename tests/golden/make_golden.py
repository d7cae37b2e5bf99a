"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Run once in a checkout that has the RocketLLM sources (read-only is fine)::

    python tests/golden/make_golden.py /path/to/RocketLLM

It imports the reference's own int4 codec (``rocketllm/quant/kv_cache.py``: ``quantize``,
``QuantizedTensor.dequantize``, ``_pack``, ``_unpack``) and router reader
(``rocketllm/moe/router.py``: ``RouterSelection.observe``), plus transformers' own
``MixtralTopKRouter`` (the model's router, which the reference reads), on seeded inputs, and writes
what they return to ``*.npz`` files.  The reference package is bound without running its
``__init__`` (which imports ``accelerate``, absent here) -- the same technique the reference's own
``tests/test_kimi_k3_split.py:22-29`` uses.

The fixtures are small and committed; the tests that read them need neither the reference nor a
GPU.  bf16 tensors are stored as their uint16 bit patterns.
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bind_reference(root):
    for name, sub in (("rocketllm", "rocketllm"), ("rocketllm.quant", "rocketllm/quant"),
                      ("rocketllm.moe", "rocketllm/moe")):
        if name not in sys.modules:
            pkg = types.ModuleType(name)
            pkg.__path__ = [os.path.join(root, sub)]
            sys.modules[name] = pkg
    sys.path.insert(0, root)
    from rocketllm.quant import kv_cache
    from rocketllm.moe import router
    return kv_cache, router


def bits(t):
    """A bf16 tensor's bit pattern as uint16, any other tensor as numpy."""
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def codec_case(kv_cache, w):
    q = kv_cache.quantize(w, 1, 64)
    deq = q.dequantize()
    return {
        "w": bits(w), "packed": bits(q.packed), "scale": bits(q.scale), "zero": bits(q.zero),
        "padding": np.int64(q.padding), "group": np.int64(q.group), "deq": bits(deq),
    }


def main(root):
    kv_cache, router = bind_reference(root)
    out = {}

    # 1. fp32 weights, N(0, 0.02): aligned and ragged K.
    g = torch.Generator().manual_seed(0)
    for name, (n, k) in {"f32_aligned": (16, 256), "f32_ragged": (6, 200)}.items():
        w = torch.randn(n, k, generator=g) * 0.02
        for key, val in codec_case(kv_cache, w).items():
            out[f"{name}.{key}"] = val

    # 2. bf16 weights: the scale is computed in bf16 arithmetic by the reference.
    for name, (n, k) in {"bf16_aligned": (8, 512), "bf16_ragged": (5, 100)}.items():
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        for key, val in codec_case(kv_cache, w).items():
            out[f"{name}.{key}"] = val

    # 2b. fp16 weights: the scale is computed in fp16 arithmetic (own generator, so the cases above
    # keep their values).  The last case spreads values wide enough that fp16 rounding of the
    # range matters.
    g16 = torch.Generator().manual_seed(7)
    for name, (n, k, sd) in {"f16_aligned": (8, 256, 0.02), "f16_ragged": (5, 100, 0.02),
                             "f16_wide": (6, 192, 300.0)}.items():
        w = (torch.randn(n, k, generator=g16) * sd).to(torch.float16)
        for key, val in codec_case(kv_cache, w).items():
            out[f"{name}.{key}"] = val

    # 3. constant groups take the scale-1 path and round-trip exactly.
    w = torch.full((4, 128), 0.375, dtype=torch.float32)
    w[2, 64:] = -1.25
    for key, val in codec_case(kv_cache, w).items():
        out[f"const.{key}"] = val

    # 4. the isolated-sweep format: uniform random bytes, scale U[0.005, 0.02], zero = -8*scale.
    n, k = 64, 512
    packed = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8,
                           generator=torch.Generator().manual_seed(10))
    scale = (0.005 + 0.015 * torch.rand(n, k // 64, generator=torch.Generator().manual_seed(11))
             ).to(torch.float16)
    zero = (-8.0 * scale.float()).to(torch.float16)
    qt = kv_cache.QuantizedTensor(packed=packed, scale=scale, zero=zero, axis=1, group=64,
                                  length=k, padding=0, shape=(n, k), dtype=torch.bfloat16)
    out["sweep.packed"] = bits(packed)
    out["sweep.scale"] = bits(scale)
    out["sweep.zero"] = bits(zero)
    out["sweep.deq_bf16"] = bits(qt.dequantize())
    qt.dtype = torch.float32
    out["sweep.deq_f32"] = bits(qt.dequantize())
    # The same weight through a bf16 F.linear, the reference's dequant-to-scratch matmul.
    x = torch.randn(3, k, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    out["sweep.x"] = bits(x)
    out["sweep.y_f32"] = bits(torch.nn.functional.linear(x.float(), qt.dequantize()))

    # 5. nibble order known answer: the reference packs [1, 2] into 0x21.
    out["pack.codes"] = np.array([[1, 2, 15, 0, 7]], dtype=np.uint8)
    out["pack.packed"] = bits(kv_cache._pack(torch.tensor([[1, 2, 15, 0, 7]], dtype=torch.uint8)))
    out["pack.unpacked"] = bits(kv_cache._unpack(torch.tensor([[0x21, 0xF0]], dtype=torch.uint8)))

    # 6. Mixtral router (transformers' own) and the reference's selection reader.
    from transformers import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralTopKRouter
    cfg = MixtralConfig(hidden_size=64, num_local_experts=8, num_experts_per_tok=2)
    rt = MixtralTopKRouter(cfg)
    with torch.no_grad():
        rt.weight.copy_(torch.randn(8, 64, generator=torch.Generator().manual_seed(20)) * 0.02)
        hidden = torch.randn(16, 64, generator=torch.Generator().manual_seed(21))
        logits, scores, indices = rt(hidden)
    sel = router.RouterSelection(8, 2)
    chosen = sel.observe((logits, scores, indices))
    out["router.weight"] = bits(rt.weight.detach())
    out["router.hidden"] = bits(hidden)
    out["router.probs"] = bits(logits)
    out["router.scores"] = bits(scores)
    out["router.indices"] = bits(indices)
    out["router.selection"] = np.array(chosen if chosen is not None else [], dtype=np.int64)

    path = os.path.join(HERE, "reference_codec.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ROCKETLLM_REFERENCE", "."))

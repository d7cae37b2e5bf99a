"""CPU restatement of the reference's decode path for an RW4 Llama.  TEST INFRASTRUCTURE ONLY.

Like ``rw4_oracle``, this checks the product and is never part of it: only ``tests/`` and the CPU
legs of ``bench.py`` import it (the reference's own code cannot travel to the GPU box, so this port
is what is timed there on the host cores, ``kind: "port"``).

The reference runs a packed checkpoint on the CPU as ``RocketModel(path, device="cpu",
dtype=torch.float32)`` (``rocketllm/base.py:203-461``): transformers' model in fp32, each layer's
RW4 triples expanded at the dequant-to-scratch seam (``QuantBackend.prepare_layer``,
``rocketllm/base.py:848-855``) by ``QuantizedTensor.dequantize`` (``rocketllm/quant/kv_cache.py:
249-257``) into an fp32 ``nn.Linear`` weight, then ``generate`` -> greedy decode with the KV cache
(``rocketllm/base.py:2014-2044``).  This restates the arithmetic of that path: the same fp32
weights (``rw4_oracle.dequantize``, pinned bit-exact to the reference codec) in transformers'
``LlamaForCausalLM`` on the CPU, greedy decode timed by a logits processor at every step (the
reference harness's decode-rate method, ``tests/bench_streaming.py:474-502``).  What it leaves out
is where the reference keeps weights between tokens (its per-layer shards, streaming hooks and
cache): that changes where a weight is, not what is computed, which is why its own CPU test requires
streamed and full loads to give identical tokens (``tests/test_cpu_generation.py:121-171``).
Pinned against the reference's own run on the same checkpoint by ``tests/test_tinyllama_cpu.py``
(``tests/golden/reference_tinyllama_2l.npz``).
"""
import json
import os
import time

import numpy as np
import torch

from . import rw4_oracle as o


def load_fp32_llama(path):
    """transformers ``LlamaForCausalLM`` in fp32 on the CPU over the RW4 checkpoint at ``path``
    (``config.json`` + ``model.safetensors``), every RW4 triple expanded by the oracle codec."""
    from safetensors.numpy import load_file
    from transformers import LlamaConfig, LlamaForCausalLM

    with open(os.path.join(path, "config.json")) as f:
        conf = json.load(f)
    conf.pop("quantization_config", None)
    config = LlamaConfig(**conf)
    with torch.device("meta"):
        model = LlamaForCausalLM(config)
    raw = load_file(os.path.join(path, "model.safetensors"))
    sd = {}
    for name, value in raw.items():
        if name.endswith("_packed"):
            base = name[:-len("_packed")]
            sd[base] = torch.from_numpy(o.dequantize(value, raw[base + "_scale"],
                                                     raw[base + "_zero_point"], out="f32"))
        elif not name.endswith(("_scale", "_zero_point")):
            sd[name] = torch.from_numpy(np.ascontiguousarray(value, dtype=np.float32))
    model.load_state_dict(sd, strict=True, assign=True)
    model.eval()
    # the rotary embedding's buffers were built on meta: build it again on the CPU
    model.model.rotary_emb = type(model.model.rotary_emb)(config)
    model.generation_config.eos_token_id = None
    model.generation_config.pad_token_id = None
    return model


def greedy_decode(model, prompt, new_tokens, threads=None):
    """Greedy decode with the KV cache.  Returns ``(tokens int64 [new_tokens], scores fp32
    [new_tokens, vocab], decode tok/s, prefill seconds, threads used)``: scores are recorded, and
    every step timestamped, by a logits processor -- transformers calls it once per generated
    token, the first time at the end of prefill."""
    from transformers import LogitsProcessor, LogitsProcessorList

    if threads:
        torch.set_num_threads(int(threads))

    class Marker(LogitsProcessor):
        def __init__(self):
            self.times, self.scores = [], []

        def __call__(self, input_ids, scores):
            self.times.append(time.perf_counter())
            self.scores.append(scores.detach().float().clone())
            return scores

    marker = Marker()
    t0 = time.perf_counter()
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=new_tokens, do_sample=False,
                             logits_processor=LogitsProcessorList([marker]), eos_token_id=None,
                             pad_token_id=0)
    seq = out if isinstance(out, torch.Tensor) else out.sequences
    tokens = seq[0, prompt.shape[1]:].numpy().astype(np.int64)
    scores = torch.stack(marker.scores)[:, 0].numpy()
    rate = ((len(marker.times) - 1) / (marker.times[-1] - marker.times[0])
            if len(marker.times) > 1 else None)
    return tokens, scores, rate, marker.times[0] - t0, torch.get_num_threads()


def dequantize_torch(packed, scale, zero):
    """The reference's ``QuantizedTensor.dequantize`` to fp32 (``rocketllm/quant/kv_cache.py:
    249-257``) for a ``[N, K/2]`` RW4 weight, in torch on the CPU: low nibble = even index
    (``_unpack``, ``:269-272``), ``code * scale + zero`` per group of 64 in fp32 (two roundings
    at most: the product is exact)."""
    p = torch.as_tensor(packed)
    codes = torch.stack([p & 0x0F, p >> 4], dim=-1).reshape(p.shape[0], -1).to(torch.float32)
    n, k = codes.shape
    grouped = codes.view(n, k // 64, 64)
    restored = grouped * torch.as_tensor(scale).float().unsqueeze(-1)
    restored = restored + torch.as_tensor(zero).float().unsqueeze(-1)
    return restored.view(n, k)


def dequant_linear(x, packed, scale, zero):
    """``F.linear(x, dequantize(W))`` in fp32: the reference's dequant-to-scratch path for one
    Linear (``rocketllm/base.py:848-855`` then ``nn.Linear``)."""
    return torch.nn.functional.linear(torch.as_tensor(x, dtype=torch.float32),
                                      dequantize_torch(packed, scale, zero))

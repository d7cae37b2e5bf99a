"""Golden greedy tokens and logits of the reference's own CPU decode path on the TinyLlama RW4
configuration.

Run here, where the reference's source tree is (it is not on the GPU box), from the repo root:

    python tests/golden/make_tinyllama_golden.py            # both fixtures, a few minutes

What it does, for the full configuration (22 layers, hidden 2048, MLP 5632, 32 / 4 heads,
vocab 32000) and for a 2-layer cut of it:

1. writes the checkpoint with ``rocketllm_b200.synthetic.write_rw4_llama`` -- weights N(0, 0.02)
   from CPU seed 0 -- encoding every Linear weight with the reference's own
   ``rocketllm.quant.kv_cache.quantize(W, 1, 64)``, and records a SHA-256 of every RW4 tensor so a
   checkpoint rebuilt elsewhere (the GPU test encodes with ``rw4_quantize``) can be shown
   byte-identical;
2. runs the reference's ``RocketModel(path, device="cpu", dtype=torch.float32)`` (per-layer shards
   on disk, its streaming hooks and cache, the RW4 triples expanded at its dequant-to-scratch seam
   by ``QuantizedTensor.dequantize``; see ``reference_harness.py``) on the prompt of 128 ids from
   CPU seed 1 and decodes greedily with the KV cache (32 tokens; 8 for the cut);
3. records every step's scores through a logits processor -- the top 64 (ids, values) per step,
   the full scores of the first and last step -- the greedy tokens, each step's top-1 margin, and
   the decode rate by logits-processor marks on this machine's threads;
4. for the full configuration, runs the same reference model again with ``dtype=torch.bfloat16``
   -- the reference's own bf16 path, weights ``dequantize().to(bfloat16)`` and bf16 activations --
   with the fp32 run's tokens fed back (teacher forcing), and records its scores at the fp32 run's
   top-64 ids, its first and last full scores and each step's argmax: how far a bf16 run of the
   reference itself lands from its fp32 run, the floor any bf16 implementation is measured
   against.

Outputs ``tests/golden/reference_tinyllama.npz`` and ``reference_tinyllama_2l.npz``.
"""
import hashlib
import os
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import reference_harness as rh  # noqa: E402
from rocketllm_b200.synthetic import TINYLLAMA, tinyllama_prompt, write_rw4_llama  # noqa: E402

TOPK = 64


def rw4_digest(sd):
    """SHA-256 over every RW4 tensor's bytes, in the checkpoint's tensor order."""
    h = hashlib.sha256()
    for name in sorted(sd):
        if name.endswith(("_packed", "_scale", "_zero_point")):
            h.update(name.encode())
            h.update(sd[name].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def reference_run(path, tokens, threads, dtype, force=None):
    model = rh.reference_cpu_model(path, threads=threads, dtype=dtype)
    prompt = tinyllama_prompt()
    marker = rh.phase_marker(force)
    t0 = time.perf_counter()
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=tokens, do_sample=False,
                             logits_processor=[marker])
    seq = out if isinstance(out, torch.Tensor) else out.sequences
    generated = seq[0, prompt.shape[1]:].numpy().astype(np.int64)
    scores = torch.stack(marker.scores)[:, 0].float()          # [steps, vocab]
    return prompt, generated, scores, marker.decode_tokens_per_second(), marker.times[0] - t0


def make(layers, tokens, out_name, threads, with_bf16):
    rocketllm = rh.import_reference()
    from rocketllm.quant.kv_cache import quantize

    def reference_quantize(w):
        q = quantize(w, 1, 64)
        return q.packed, q.scale, q.zero

    cfg = dict(TINYLLAMA, num_hidden_layers=layers)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "tinyllama_rw4")
        t0 = time.time()
        sd = write_rw4_llama(path, cfg, reference_quantize, seed=0, std=0.02)
        digest = rw4_digest(sd)
        del sd
        print(f"{out_name}: checkpoint written in {time.time() - t0:.1f} s", flush=True)
        prompt, generated, scores, rate, prefill = reference_run(path, tokens, threads,
                                                                 torch.float32)
        top = scores.topk(TOPK, dim=-1)
        top2 = scores.topk(2, dim=-1).values
        print(f"{out_name}: {tokens} tokens, prefill {prefill:.2f} s, decode {rate:.3f} tok/s on "
              f"{torch.get_num_threads()} threads", flush=True)
        extra = {}
        if with_bf16:
            # teacher-forced on the fp32 run's tokens, so every step's scores compare
            _, _, b_scores, b_rate, _ = reference_run(path, tokens, threads, torch.bfloat16,
                                                      force=generated)
            extra = dict(bf16_argmax=b_scores.argmax(-1).numpy().astype(np.int64),
                         bf16_top_values=b_scores.gather(1, top.indices).numpy().astype(np.float32),
                         bf16_first_scores=b_scores[0].numpy().astype(np.float32),
                         bf16_last_scores=b_scores[-1].numpy().astype(np.float32),
                         bf16_decode_tok_s=np.float64(b_rate))
            print(f"{out_name}: bf16 run decode {b_rate:.3f} tok/s", flush=True)
        np.savez_compressed(
            os.path.join(HERE, out_name),
            layers=np.int64(layers), prompt=prompt.numpy().astype(np.int64), tokens=generated,
            top_ids=top.indices.numpy().astype(np.int32),
            top_values=top.values.numpy().astype(np.float32),
            first_scores=scores[0].numpy().astype(np.float32),
            last_scores=scores[-1].numpy().astype(np.float32),
            margins=(top2[:, 0] - top2[:, 1]).numpy().astype(np.float32),
            rw4_sha256=np.array(digest), decode_tok_s=np.float64(rate),
            prefill_s=np.float64(prefill), threads=np.int64(torch.get_num_threads()),
            cpu_count=np.int64(os.cpu_count()), reference_torch=np.array(torch.__version__),
            **extra)


if __name__ == "__main__":
    threads = os.cpu_count()
    which = sys.argv[1:] or ["2l", "full"]
    if "2l" in which:
        make(2, 8, "reference_tinyllama_2l.npz", threads, False)
    if "full" in which:
        make(TINYLLAMA["num_hidden_layers"], 32, "reference_tinyllama.npz", threads, True)

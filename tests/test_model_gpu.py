"""Model-level parity on the GPU: a random-init model converted to RW4 and loaded through
transformers with the rw4 quantizer, against the reference's dequant-to-scratch path -- the same
transformers model in bf16 whose weights are QuantizedTensor.dequantize().to(bfloat16)
(rocketllm/quant/registry.py:529-535 + kv_cache.py:249-257; our dequant kernel is bit-exact with
it, tests/test_codec_gpu.py).  Bars: logits max-abs <= 2e-2, greedy tokens identical.
"""
import copy

import pytest
import torch

from rocketllm_b200 import kernels
from rocketllm_b200.quant import RW4Linear  # noqa: F401 - registers the rw4 quantizer
from rocketllm_b200.quant.convert import save_rw4_checkpoint

pytestmark = pytest.mark.gpu


def init_normal(model, seed=0):
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=gen) * 0.02)
    return model


def reference_model(dense, rw4):
    """The reference path: dense bf16 model whose quantized weights are the dequantized RW4 ones."""
    ref = copy.deepcopy(dense).to("cuda", torch.bfloat16)
    with torch.no_grad():
        for name, mod in rw4.named_modules():
            if isinstance(mod, RW4Linear):
                tgt = ref.get_submodule(name)
                tgt.weight.copy_(kernels.dequantize(mod.weight_packed, mod.weight_scale,
                                                    mod.weight_zero_point))
            elif getattr(mod, "rw4", False):
                tgt = ref.get_submodule(name)
                for wn in ("gate_up_proj", "down_proj"):
                    p, s, z = (getattr(mod, wn + sfx) for sfx in ("_packed", "_scale",
                                                                   "_zero_point"))
                    for e in range(p.shape[0]):
                        getattr(tgt, wn)[e].copy_(kernels.dequantize(p[e], s[e], z[e]))
    ref.config._experts_implementation = "eager"
    return ref


def run_pair(dense, tmp_path, steps=12, hooks=None):
    from transformers import AutoModelForCausalLM
    path = save_rw4_checkpoint(dense, str(tmp_path / "rw4"), device="cuda")
    rw4 = AutoModelForCausalLM.from_pretrained(path, dtype=torch.bfloat16).to("cuda")
    ref = reference_model(dense, rw4)
    if hooks is not None:
        handles = hooks(rw4, "rw4") + hooks(ref, "ref")
    ids = torch.randint(0, dense.config.vocab_size, (1, 24),
                        generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        lr = rw4(ids).logits.float()
        lf = ref(ids).logits.float()
    err = (lr - lf).abs().max().item()
    assert err <= 2e-2, f"logits max-abs {err}"
    if hooks is not None:
        for h in handles:
            h.remove()
    with torch.no_grad():
        gr = rw4.generate(ids, max_new_tokens=steps, do_sample=False, min_new_tokens=steps)
        gf = ref.generate(ids, max_new_tokens=steps, do_sample=False, min_new_tokens=steps)
    assert torch.equal(gr, gf), f"greedy tokens differ:\n{gr}\n{gf}"
    assert kernels.device_status() == 0
    return rw4


def test_llama_rw4_matches_reference_path(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                      max_position_embeddings=512, tie_word_embeddings=False, rope_theta=10000.0)
    dense = init_normal(LlamaForCausalLM(cfg), seed=0)
    rw4 = run_pair(dense, tmp_path)
    assert isinstance(rw4.lm_head, RW4Linear)


def test_mixtral_rw4_matches_reference_path(tmp_path):
    from transformers import MixtralConfig, MixtralForCausalLM
    cfg = MixtralConfig(hidden_size=512, intermediate_size=512, num_hidden_layers=2,
                        num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                        num_local_experts=8, num_experts_per_tok=2, max_position_embeddings=512,
                        tie_word_embeddings=False)
    dense = init_normal(MixtralForCausalLM(cfg), seed=3)
    # A decisive router (N(0, 0.2) instead of N(0, 0.02)): with near-uniform routing a top-2 vs
    # 3rd margin below the two paths' bf16 noise in the router probabilities (~1e-3) flips an
    # expert choice, which says nothing about the kernels.  Routing identity is asserted below.
    with torch.no_grad():
        for layer in dense.model.layers:
            layer.mlp.gate.weight.mul_(10.0)
    routes = {}

    def record(tag):
        def hook(mod, inp, out):
            routes.setdefault(tag, []).append(out[2].sort(-1).values.cpu())
        return hook

    rw4 = run_pair(dense, tmp_path, hooks=lambda m, tag: [
        layer.mlp.gate.register_forward_hook(record(tag)) for layer in m.model.layers])
    assert rw4.config._experts_implementation == "rw4"
    assert len(routes["rw4"]) == len(routes["ref"]) > 0
    for a, b in zip(routes["rw4"], routes["ref"]):
        assert torch.equal(a, b), "routing indices differ"

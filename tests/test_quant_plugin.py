"""The RW4 plugin surface on CPU: registry detection and sizing (the reference's
tests/test_quant_registry.py:273-417 checks, for the rw4 format), module replacement through the
transformers quantizer, and loading a pre-quantized checkpoint by name.  No kernel runs here."""
import json
import os

import pytest
import torch

from rocketllm_b200.quant import (QuantBackend, RW4Backend, RW4Linear, TensorSpec, convert_modules,
                                  decision_table, detect_backend)

N, K = 512, 1024


def rw4_shard(name="model.layers.0.mlp.down_proj", bias=True):
    shard = {
        f"{name}.weight_packed": torch.randint(0, 256, (N, K // 2), dtype=torch.uint8),
        f"{name}.weight_scale": torch.rand(N, K // 64).to(torch.float16),
        f"{name}.weight_zero_point": torch.rand(N, K // 64).to(torch.float16),
    }
    if bias:
        shard[f"{name}.bias"] = torch.zeros(N, dtype=torch.bfloat16)
    return shard


def test_detect_backend_from_the_declared_method():
    assert isinstance(detect_backend({"quant_method": "rw4", "bits": 4}), RW4Backend)
    assert isinstance(detect_backend({"quant_method": "RW4"}), RW4Backend)
    assert type(detect_backend(None)) is QuantBackend
    with pytest.raises(ValueError):
        detect_backend({"quant_method": "awq"})


def test_rw4_weight_groups_and_sizes():
    backend = detect_backend({"quant_method": "rw4", "bits": 4}, compute_dtype=torch.bfloat16)
    weights = backend.plan(rw4_shard())
    names = [w.name for w in weights]
    assert names == ["model.layers.0.mlp.down_proj.weight", "model.layers.0.mlp.down_proj.bias"]
    w = weights[0]
    assert w.tensor_names[0].endswith("weight_packed")  # payload first
    assert w.bits == 4
    assert w.logical_shape == (N, K)
    assert w.packed_bytes == N * K // 2 + 2 * N * (K // 64) * 2
    assert w.expanded_bytes == N * K * 2
    assert w.needs_scratch is False and w.scratch_bytes == 0
    bias = weights[1]
    assert bias.bits == 16 and bias.packed_bytes == N * 2
    # an fp32 compute dtype is what the expanded size expands into (the packed size is unchanged)
    wide = detect_backend({"quant_method": "rw4", "bits": 4}, compute_dtype=torch.float32)
    ww = wide.plan(rw4_shard())[0]
    assert ww.expanded_bytes == N * K * 4 and ww.packed_bytes == w.packed_bytes


def test_sizes_from_header_match_sizes_from_data():
    backend = detect_backend({"quant_method": "rw4"})
    shard = rw4_shard()
    specs = [TensorSpec.of(n, t) for n, t in shard.items()]
    a = backend.plan(shard)[0]
    b = backend.plan_from_specs(specs)[0]
    assert (a.packed_bytes, a.expanded_bytes) == (b.packed_bytes, b.expanded_bytes)
    with pytest.raises(ValueError, match="metadata"):
        b.materialize("cpu")


def test_packed_tensors_are_placed_verbatim():
    backend = detect_backend({"quant_method": "rw4"}, compute_dtype=torch.bfloat16)
    shard = rw4_shard()
    for name, value in shard.items():
        want = value.dtype if not name.endswith(".bias") else torch.bfloat16
        assert backend.target_dtype(name, value) == want
    assert backend.prepare_layer(shard) is shard  # no dequant-to-scratch


def test_decision_table_reports_the_fused_path():
    rows = {r["format"]: r for r in decision_table()}
    assert rows["rw4"]["path"] in ("fused_packed", "unavailable")
    assert rows["dense"]["path"] == "as_stored"


def tiny_llama_config():
    from transformers import LlamaConfig
    return LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, vocab_size=1000,
                       max_position_embeddings=256, tie_word_embeddings=False)


def test_quantizer_swaps_every_linear_on_meta():
    from transformers import LlamaForCausalLM
    with torch.device("meta"):
        model = LlamaForCausalLM(tiny_llama_config())
    names = convert_modules(model)
    assert "lm_head" in names and "model.layers.1.mlp.down_proj" in names
    assert not any(isinstance(m, torch.nn.Linear) for m in model.modules())
    lin = model.model.layers[0].self_attn.k_proj
    assert isinstance(lin, RW4Linear)
    assert lin.weight_packed.shape == (128, 256) and lin.weight_scale.shape == (128, 8)


def test_stacked_experts_get_rw4_triples():
    from transformers import MixtralConfig, MixtralForCausalLM
    cfg = MixtralConfig(hidden_size=512, intermediate_size=512, num_hidden_layers=1,
                        num_attention_heads=8, num_key_value_heads=2, vocab_size=1000,
                        num_local_experts=4, num_experts_per_tok=2)
    with torch.device("meta"):
        model = MixtralForCausalLM(cfg)
    convert_modules(model, modules_to_not_convert=["lm_head"])
    experts = model.model.layers[0].mlp.experts
    assert experts.gate_up_proj_packed.shape == (4, 1024, 256)
    assert experts.down_proj_scale.shape == (4, 512, 8)
    assert experts.gate_up_proj.numel() == 0 and "gate_up_proj" not in experts.state_dict()
    assert model.config._experts_implementation == "rw4"
    assert isinstance(model.model.layers[0].mlp.gate, torch.nn.Module)  # router left alone
    assert not isinstance(model.lm_head, RW4Linear)


def test_prequantized_checkpoint_loads_by_name_and_has_no_cpu_path(tmp_path):
    from safetensors.torch import save_file
    from transformers import AutoModelForCausalLM, LlamaForCausalLM
    cfg = tiny_llama_config()
    model = LlamaForCausalLM(cfg)
    sd = {}
    for name, mod in model.named_modules():
        if isinstance(mod, torch.nn.Linear):
            n, k = mod.weight.shape
            sd[f"{name}.weight_packed"] = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8)
            sd[f"{name}.weight_scale"] = torch.full((n, k // 64), 0.01, dtype=torch.float16)
            sd[f"{name}.weight_zero_point"] = torch.full((n, k // 64), -0.08, dtype=torch.float16)
    for name, p in model.state_dict().items():
        if not name.endswith(".weight") or "norm" in name or "embed" in name:
            if name not in sd and not any(name.startswith(k.rsplit(".", 1)[0] + ".weight")
                                          for k in sd):
                sd[name] = p
    sd["model.embed_tokens.weight"] = model.model.embed_tokens.weight.detach()
    for i in range(2):
        for nrm in ("input_layernorm", "post_attention_layernorm"):
            sd[f"model.layers.{i}.{nrm}.weight"] = torch.ones(512)
    sd["model.norm.weight"] = torch.ones(512)
    save_file(sd, os.path.join(tmp_path, "model.safetensors"), metadata={"format": "pt"})
    d = cfg.to_dict()
    d["quantization_config"] = {"quant_method": "rw4", "bits": 4, "group_size": 64}
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump(d, f)
    loaded = AutoModelForCausalLM.from_pretrained(str(tmp_path), dtype=torch.bfloat16)
    q = loaded.model.layers[1].mlp.up_proj
    assert isinstance(q, RW4Linear)
    assert torch.equal(q.weight_packed, sd["model.layers.1.mlp.up_proj.weight_packed"])
    with pytest.raises(ValueError, match="CUDA"):
        loaded(torch.tensor([[1, 2, 3]]))


def test_scales_keep_fp16_through_a_bf16_load(tmp_path):
    """A bf16 load must not cast the fp16 scale / zero companions (they are part of the format)."""
    test_prequantized_checkpoint_loads_by_name_and_has_no_cpu_path(tmp_path)
    from transformers import AutoModelForCausalLM
    loaded = AutoModelForCausalLM.from_pretrained(str(tmp_path), dtype=torch.bfloat16)
    lin = loaded.model.layers[0].self_attn.q_proj
    assert lin.weight_scale.dtype == torch.float16
    assert lin.weight_zero_point.dtype == torch.float16
    assert float(lin.weight_scale[0, 0]) == pytest.approx(0.01, rel=1e-3)
    assert loaded.model.norm.weight.dtype == torch.bfloat16

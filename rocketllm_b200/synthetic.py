"""Seeded synthetic RW4 inputs, shaped like the isolated dequant-matmul sweep.

Weights: uniform random code bytes, per-group scale ~ U[0.005, 0.02], zero = -8 * scale (so every
weight is (code - 8) * scale, centred on zero), group 64.  Activations: bf16 N(0, 1).
Generated on the target device with ``torch.Generator`` seeds so host and device agree bit for bit.
"""
import torch

# The isolated sweep's weight shapes (K, N) and batch sizes M.
SWEEP_SHAPES = ((4096, 4096), (4096, 14336), (14336, 4096), (8192, 28672), (16384, 53248))
SWEEP_M = (1, 4, 16, 64, 512, 2048)


def make_weight(n, k, device="cuda", seed=0, group=64):
    """``(packed u8 [n, k/2], scale f16 [n, k/group], zero f16 [n, k/group])``."""
    gen = torch.Generator(device=device).manual_seed(seed)
    packed = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    gen.manual_seed(seed + 1)
    scale = (0.005 + 0.015 * torch.rand((n, k // group), device=device, generator=gen)).to(
        torch.float16)
    zero = (-8.0 * scale.float()).to(torch.float16)
    return packed, scale, zero


def make_activation(m, k, device="cuda", seed=2):
    gen = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((m, k), device=device, generator=gen).to(torch.bfloat16)


@torch.no_grad()
def build_rw4_causal_lm(config, device="cuda", seed=0, std=0.02, layers=None, keep_embed=True,
                        keep_head=True):
    """A random-init RW4 ``*ForCausalLM`` built directly on ``device``: every Linear / stacked-expert
    weight drawn N(0, std) in bf16 and encoded with ``rw4_quantize`` (the reference codec), norms 1,
    other weights N(0, std).  No dense copy of the whole model ever exists.

    ``layers = (start, stop)`` materialises only those decoder layers (the others become
    ``nn.Identity``), ``keep_embed`` / ``keep_head`` the embedding and the final norm + lm_head: one
    pipeline stage of a model too large for one GPU.  Every tensor draws from its own generator
    seeded by ``seed`` and its name, so a stage holds exactly the values of the same layers of the
    whole model."""
    import zlib

    from transformers import AutoModelForCausalLM

    from . import kernels
    from .quant.hf import convert_modules
    from .quant.modules import RW4Linear

    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(config, dtype=torch.bfloat16)
    convert_modules(model)
    inner = model.model
    if layers is not None:
        for i in range(len(inner.layers)):
            if not layers[0] <= i < layers[1]:
                inner.layers[i] = torch.nn.Identity()
    if not keep_embed:
        inner.embed_tokens = None
    if not keep_head:
        model.lm_head = None
        inner.norm = None
    model.to_empty(device=device)

    def gen_for(name):
        return torch.Generator(device=device).manual_seed(
            (seed * 1000003 + zlib.crc32(name.encode())) % (1 << 62))

    def encode_into(name, packed, scale, zero, n, k):
        w = (torch.randn((n, k), device=device, generator=gen_for(name)) * std).to(torch.bfloat16)
        p, s, z, _ = kernels.quantize(w, 64)
        packed.copy_(p), scale.copy_(s), zero.copy_(z)
        del w, p, s, z

    for name, mod in model.named_modules():
        if isinstance(mod, RW4Linear):
            encode_into(name, mod.weight_packed, mod.weight_scale, mod.weight_zero_point,
                        mod.out_features, mod.in_features)
            if mod.bias is not None:
                mod.bias.zero_()
        elif getattr(mod, "rw4", False):
            for wn in ("gate_up_proj", "down_proj"):
                p, s, z = (getattr(mod, wn + sfx) for sfx in ("_packed", "_scale", "_zero_point"))
                for e in range(p.shape[0]):
                    encode_into(f"{name}.{wn}.{e}", p[e], s[e], z[e], p.shape[1],
                                p.shape[2] * 2)
    rw4_suffixes = ("_packed", "_scale", "_zero_point")
    for name, param in model.named_parameters():
        if name.endswith(rw4_suffixes) or name.endswith(".bias"):
            continue
        if "norm" in name:
            param.fill_(1.0)
        else:
            param.copy_((torch.randn(param.shape, device=device, generator=gen_for(name)) * std)
                        .to(param.dtype))
    # non-persistent buffers (rotary inverse frequencies) were left uninitialised by to_empty:
    # rebuild those modules' buffers on the device
    for mod in model.modules():
        if "inv_freq" in mod._buffers and hasattr(mod, "config"):
            fresh = type(mod)(mod.config, device=device)
            for bname, buf in fresh._buffers.items():
                mod._buffers[bname] = buf
            if hasattr(fresh, "attention_scaling"):
                mod.attention_scaling = fresh.attention_scaling
    return model.eval()


def algorithmic_bytes(m, k, n, group=64):
    """Bytes one ``y = x W^T`` call must move at least once: codes, scales, zeros, x and y."""
    return n * k // 2 + 2 * 2 * (k // group) * n + 2 * m * k + 2 * m * n


def flops(m, k, n):
    return 2 * m * n * k


# ---- seeded Llama checkpoints built on the CPU ---------------------------------------------------

# TinyLlama-1.1B architecture: the configuration the reference's CPU path is timed and compared on.
TINYLLAMA = dict(hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
                 num_attention_heads=32, num_key_value_heads=4, head_dim=64, vocab_size=32000,
                 rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048,
                 tie_word_embeddings=False, bos_token_id=None, eos_token_id=None,
                 pad_token_id=None)


def llama_tensor_plan(cfg):
    """``(name, shape, kind)`` of every tensor of a ``LlamaForCausalLM`` with config dict ``cfg`` in
    a fixed order; ``kind`` is ``"linear"`` (an ``nn.Linear`` weight), ``"norm"`` or ``"embed"``."""
    h, i, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    hd = cfg.get("head_dim") or h // cfg["num_attention_heads"]
    q, kv = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd
    plan = [("model.embed_tokens.weight", (v, h), "embed")]
    for layer in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        plan += [(p + "self_attn.q_proj.weight", (q, h), "linear"),
                 (p + "self_attn.k_proj.weight", (kv, h), "linear"),
                 (p + "self_attn.v_proj.weight", (kv, h), "linear"),
                 (p + "self_attn.o_proj.weight", (h, q), "linear"),
                 (p + "mlp.gate_proj.weight", (i, h), "linear"),
                 (p + "mlp.up_proj.weight", (i, h), "linear"),
                 (p + "mlp.down_proj.weight", (h, i), "linear"),
                 (p + "input_layernorm.weight", (h,), "norm"),
                 (p + "post_attention_layernorm.weight", (h,), "norm")]
    plan += [("model.norm.weight", (h,), "norm"), ("lm_head.weight", (v, h), "linear")]
    return plan


def seeded_llama_tensors(cfg, seed=0, std=0.02):
    """Yield ``(name, kind, tensor)``: every matrix ~ N(0, std) in fp32, drawn in plan order from
    one CPU ``torch.Generator(seed)`` (the same values on any machine with this torch), norms 1."""
    gen = torch.Generator().manual_seed(seed)
    for name, shape, kind in llama_tensor_plan(cfg):
        if kind == "norm":
            yield name, kind, torch.ones(shape, dtype=torch.float32)
        else:
            yield name, kind, torch.randn(shape, generator=gen, dtype=torch.float32) * std


def write_rw4_llama(path, cfg, quantize_fn, seed=0, std=0.02):
    """Write ``config.json`` + ``model.safetensors`` of a seeded Llama whose ``nn.Linear`` weights
    are RW4 (``X.weight_packed`` / ``X.weight_scale`` / ``X.weight_zero_point`` from
    ``quantize_fn(w fp32 [N, K]) -> (packed u8, scale f16, zero f16)``) and whose embedding and
    norms stay fp32.  Returns ``{name: tensor}`` of what was written (CPU tensors)."""
    import json
    import os

    from safetensors.torch import save_file
    from transformers import LlamaConfig

    os.makedirs(path, exist_ok=True)
    sd = {}
    for name, kind, t in seeded_llama_tensors(cfg, seed, std):
        if kind == "linear":
            packed, scale, zero = (a.contiguous().cpu() for a in quantize_fn(t))
            base = name  # X.weight -> X.weight_packed / _scale / _zero_point
            sd[base + "_packed"], sd[base + "_scale"], sd[base + "_zero_point"] = packed, scale, zero
        else:
            sd[name] = t
    save_file(sd, os.path.join(path, "model.safetensors"), metadata={"format": "pt"})
    conf = LlamaConfig(**cfg).to_dict()
    conf["architectures"] = ["LlamaForCausalLM"]
    conf["torch_dtype"] = "float32"
    conf["quantization_config"] = {"quant_method": "rw4", "bits": 4, "group_size": 64,
                                   "modules_to_not_convert": []}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(conf, f, indent=1)
    return sd


def tinyllama_prompt(length=128, seed=1, vocab=32000):
    """The reference configuration's prompt: ``length`` token ids uniform in [0, vocab) from
    ``seed`` (CPU generator)."""
    return torch.randint(0, vocab, (1, length), generator=torch.Generator().manual_seed(seed))

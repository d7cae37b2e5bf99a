"""The int4 KV cache's bookkeeping, device layout and attention plumbing, on CPU.

``RW4KVCache`` takes its codec and decode attention as injected operations; here they are the
oracle's numpy restatements (``CpuKVOps``), and ``attend`` decodes the device layout
(``include/rw4.h``) independently of the cache's own ``history``, so these tests pin the layout the
CUDA kernel reads.  The reference's own outputs come from ``tests/golden/reference_kv.npz``.
"""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import rw4_oracle as O
from rocketllm_b200.kv_cache import (ATTN_NAME, KVCacheConfig, RW4KVCache, enable_kv_attention,
                                     resolve_kv_cache)

KV = os.path.join(ROOT, "tests", "golden", "reference_kv.npz")


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class CpuKVOps:
    """The oracle codec and attention on CPU tensors (test infrastructure only)."""

    def __init__(self):
        self.attends = 0

    def quantize(self, x2d):
        p, s, z, _ = O.quantize(_bits(x2d), 64, "bf16")
        return torch.from_numpy(p), torch.from_numpy(s), torch.from_numpy(z)

    def dequantize(self, packed, scale, zero):
        return _bf16(O.dequantize(packed.numpy(), scale.numpy(), zero.numpy(), out="bf16"))

    def attend(self, query, layer, scaling):
        """Decode the device layout directly: K group g, channel c, byte i holds tokens
        64g+2i (low nibble) and 64g+2i+1; V token t, byte j holds channels 2j, 2j+1."""
        self.attends += 1
        b, kvh, d = layer.shape
        g = layer.groups
        kc = layer.k_codes[:, :, :g].numpy()
        codes = np.stack([kc & 15, kc >> 4], axis=-1).reshape(b, kvh, g, d, 64)
        ksz = layer.k_sz[:, :, :g].numpy().astype(np.float32)
        kq = codes * ksz[..., 0:1] + ksz[..., 1:2]                       # [b,kvh,g,d,64]
        kq = kq.transpose(0, 1, 2, 4, 3).reshape(b, kvh, g * 64, d)
        vc = layer.v_codes[:, :, :g * 64].numpy()
        vcodes = np.stack([vc & 15, vc >> 4], axis=-1).reshape(b, kvh, g * 64, d // 64, 64)
        vsz = layer.v_sz[:, :, :g * 64].numpy().astype(np.float32)
        vq = (vcodes * vsz[..., 0:1] + vsz[..., 1:2]).reshape(b, kvh, g * 64, d)
        kq = O.round_bf16(kq.astype(np.float32))
        vq = O.round_bf16(vq.astype(np.float32))
        kr = layer.k_res[:, :, :layer.rlen].float().numpy()
        vr = layer.v_res[:, :, :layer.rlen].float().numpy()
        k = np.concatenate([kq, kr], axis=2)
        v = np.concatenate([vq, vr], axis=2)
        out = O.attention_causal(query.float().numpy(), k, v, scaling)   # [b, h, q, d]
        return torch.from_numpy(out).to(torch.bfloat16).transpose(1, 2)


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(KV))


def _replay(gold, fused):
    b, kvh, h, d, prefill, steps = gold["shape"].tolist()
    cache = RW4KVCache(ops=CpuKVOps(), fused=fused)
    out = cache.update(_bf16(gold["k.0"]), _bf16(gold["v.0"]), 0)
    assert out[0].shape[2] == int(gold["hist_len.0"])
    for s in range(1, steps + 1):
        out = cache.update(_bf16(gold[f"k.{s}"]), _bf16(gold[f"v.{s}"]), 0)
    return cache, out


def test_history_matches_reference(gold):
    cache, (hk, hv) = _replay(gold, fused=False)
    np.testing.assert_array_equal(_bits(hk), gold["hist_k.last"])
    np.testing.assert_array_equal(_bits(hv), gold["hist_v.last"])
    assert cache.get_seq_length(0) == hk.shape[2]
    assert cache._kv[0].blocks == gold["blocks"].tolist()
    assert cache._kv[0].rlen == int(gold["residual"])


def test_quantized_layout_matches_reference_blocks(gold):
    cache, _ = _replay(gold, fused=False)
    kp, ks, kz, vp, vs, vz = cache.quantized(0)
    n = len(gold["blocks"])
    cat = {name: np.concatenate([gold[f"{name}{i}.{f}"] for i in range(n)],
                                axis=-1 if name == "kb" else 2)
           for name in ("kb", "vb") for f in ("packed",)}
    np.testing.assert_array_equal(kp.numpy(), cat["kb"])
    np.testing.assert_array_equal(vp.numpy(), cat["vb"])
    for mine, name, f, axis in ((ks, "kb", "scale", -1), (kz, "kb", "zero", -1),
                                (vs, "vb", "scale", 2), (vz, "vb", "zero", 2)):
        ref = np.concatenate([gold[f"{name}{i}.{f}"] for i in range(n)], axis=axis)
        np.testing.assert_array_equal(mine.numpy().view(np.uint16), ref.view(np.uint16))


def test_fused_step_returns_tagged_window_and_attends(gold):
    cache, (k, v) = _replay(gold, fused=True)
    assert getattr(k, "_rw4_kv", None) == (cache, 0)
    assert k.shape[2] == int(gold["residual"])          # the window only
    q = _bf16(gold["q"])
    d = q.shape[-1]
    out = cache.attend(0, q, d ** -0.5)                  # [b, 1, h, d]
    ref = O.bf16_bits_to_f32(gold["attn"])
    assert np.abs(out.float().numpy() - ref).max() <= 2e-2
    # the layout decoded independently equals the cache's own expanded history
    hk, hv = cache.history(0)
    np.testing.assert_array_equal(_bits(hk), gold["hist_k.last"])
    np.testing.assert_array_equal(_bits(hv), gold["hist_v.last"])


def test_crop_window_only(gold):
    cache, _ = _replay(gold, fused=False)
    n = cache.get_seq_length(0)
    quantized = cache._kv[0].groups * 64
    cache.crop(n - 5)
    assert cache.get_seq_length(0) == n - 5
    with pytest.raises(ValueError):
        cache.crop(quantized - 1)


def test_config_rejects_other_layouts():
    with pytest.raises(ValueError):
        KVCacheConfig(group_size=32)
    with pytest.raises(ValueError):
        KVCacheConfig(key_axis=3, value_axis=2)
    with pytest.raises(ValueError):
        KVCacheConfig(residual_length=32)


def test_resolve():
    assert resolve_kv_cache("int4")[0] == "int4"
    assert resolve_kv_cache("auto", 10, 100)[0] == "fp16"
    assert resolve_kv_cache("auto", 100, 100)[0] == "int4"
    with pytest.raises(ValueError):
        resolve_kv_cache("int8")


def _tiny_llama(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=512,
                      max_position_embeddings=1024)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


def test_model_decode_through_fused_attention():
    """A Llama decodes past two flushes with the fused attention (CPU ops); its logits follow the
    reference behaviour (expanded history + SDPA) step for step."""
    model = _tiny_llama()
    enable_kv_attention(model)
    assert model.config._attn_implementation == ATTN_NAME
    ops = CpuKVOps()
    fused = RW4KVCache(ops=ops, fused=True)
    plain = RW4KVCache(ops=CpuKVOps(), fused=False)
    ids = torch.randint(0, 512, (1, 150), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        a = model(ids, past_key_values=fused, use_cache=True).logits[:, -1]
        b = model(ids, past_key_values=plain, use_cache=True).logits[:, -1]
        assert (a - b).abs().max().item() == 0.0           # prefill: same path
        tok = a.argmax(-1, keepdim=True)
        worst = 0.0
        for _ in range(110):                               # 260 tokens: two groups flushed
            a = model(tok, past_key_values=fused, use_cache=True).logits[:, -1]
            b = model(tok, past_key_values=plain, use_cache=True).logits[:, -1]
            worst = max(worst, (a.float() - b.float()).abs().max().item())
            tok = b.argmax(-1, keepdim=True)
    assert ops.attends == 110 * 2                         # every decode step, every layer
    assert fused._kv[0].groups >= 2
    assert worst <= 2e-2


def test_chunked_queries_run_on_the_packed_history():
    """A ``causal_chunks`` cache hands 3-token chunks (a verify pass) to the packed attention too;
    the logits follow the reference behaviour (expanded history + masked SDPA) chunk by chunk,
    across flushes."""
    model = _tiny_llama()
    enable_kv_attention(model)
    ops = CpuKVOps()
    chunked = RW4KVCache(ops=ops, fused=True, causal_chunks=True)
    plain = RW4KVCache(ops=CpuKVOps(), fused=False)
    ids = torch.randint(0, 512, (1, 150), generator=torch.Generator().manual_seed(7))
    worst = 0.0
    with torch.no_grad():
        model(ids, past_key_values=chunked, use_cache=True)
        model(ids, past_key_values=plain, use_cache=True)
        g = torch.Generator().manual_seed(8)
        for _ in range(40):                       # 270 tokens: two groups flushed meanwhile
            chunk = torch.randint(0, 512, (1, 3), generator=g)
            a = model(chunk, past_key_values=chunked, use_cache=True).logits
            b = model(chunk, past_key_values=plain, use_cache=True).logits
            worst = max(worst, (a.float() - b.float()).abs().max().item())
    assert ops.attends == 40 * 2                  # every chunk, every layer, on the packed path
    assert chunked._kv[0].groups >= 2
    assert worst <= 2e-2

"""Layer streaming (pinned host blobs -> window device slots, prefetch in the pre-hook) produces
exactly the tokens and logits of the resident model -- the reference's own streaming gate
(tests/test_cpu_generation.py:121-171: streamed == full load) -- and moves every layer once per
token."""
import pytest
import torch

from rocketllm_b200.engine import AutoModel, RocketModel, footprint
from rocketllm_b200.quant.convert import save_rw4_checkpoint

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                      max_position_embeddings=512, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():
        for n, p in model.named_parameters():
            p.copy_(torch.ones_like(p) if "norm" in n else torch.randn_like(p) * 0.02)
    return save_rw4_checkpoint(model, str(tmp_path_factory.mktemp("rw4")), device="cuda")


@pytest.mark.parametrize("window", [1, 2, 3])
def test_streamed_equals_resident(checkpoint, window):
    ids = torch.randint(0, 2048, (1, 16), generator=torch.Generator().manual_seed(4)).cuda()
    resident = AutoModel.from_pretrained(checkpoint)
    assert resident.streamer is None
    streamed = RocketModel(checkpoint, vram_budget=1, window=window, kv_cache="fp16")  # forces streaming
    assert streamed.streamer is not None and streamed.streamer.window == 1
    streamed.close()
    rest, layers = footprint(resident.model)
    budget = rest + window * max(layers) + 1000  # room for exactly `window` layer slots
    streamed = RocketModel(checkpoint, vram_budget=budget, window=window, kv_cache="fp16")
    with torch.no_grad():
        assert torch.equal(resident(ids).logits, streamed(ids).logits)
        a = resident.generate(ids, max_new_tokens=8, do_sample=False, min_new_tokens=8)
        b = streamed.generate(ids, max_new_tokens=8, do_sample=False, min_new_tokens=8)
    assert torch.equal(a, b)
    st = streamed.stats()["streaming"]
    assert st["window"] == window
    assert st["fetches"] >= 4 * (1 + 8)          # every layer, every forward
    assert st["transfer"]["stalls"] == 0
    streamed.close()


def test_pinned_layers_within_budget(checkpoint):
    """Budget beyond the window slots keeps the last layers resident (the reference's pin
    placement); only the others stream, and the result is unchanged."""
    ids = torch.randint(0, 2048, (1, 16), generator=torch.Generator().manual_seed(6)).cuda()
    resident = AutoModel.from_pretrained(checkpoint)
    rest, layers = footprint(resident.model)
    budget = rest + 1 * max(layers) + 2 * max(layers) + 1000   # one slot + two pinned layers
    streamed = RocketModel(checkpoint, vram_budget=budget, window=1, kv_cache="fp16")
    st = streamed.stats()["streaming"]
    assert st["pinned"] == 2 and st["streamed"] == 2 and st["window"] == 1
    with torch.no_grad():
        assert torch.equal(resident(ids).logits, streamed(ids).logits)
        a = resident.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
        b = streamed.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
    assert torch.equal(a, b)
    st = streamed.stats()["streaming"]
    assert st["bytes"] <= 2 * max(layers) * (1 + 1 + 6)   # only the two streamed layers move
    streamed.close()


def test_kv_cache_int4_decodes_through_packed_attention(checkpoint, monkeypatch):
    """``kv_cache="int4"`` hands every generate an int4 cache whose one-token steps run the
    packed-history kernel; ``"auto"`` picks it exactly when the weights stream."""
    from rocketllm_b200.kv_cache import RW4KVCache
    calls = []
    original = RW4KVCache.attend

    def counting(self, layer_idx, query, scaling):
        calls.append(layer_idx)
        return original(self, layer_idx, query, scaling)

    monkeypatch.setattr(RW4KVCache, "attend", counting)
    # 190 prompt tokens stay in the exact window through the prefill (so the first token is the
    # fp16 cache's); the second decode step flushes the first group of 64
    ids = torch.randint(0, 2048, (1, 190), generator=torch.Generator().manual_seed(9)).cuda()
    exact = AutoModel.from_pretrained(checkpoint, kv_cache="fp16")
    assert exact.kv_cache_choice == "fp16"
    int4 = AutoModel.from_pretrained(checkpoint, kv_cache="int4")
    with torch.no_grad():
        a = exact.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
        b = int4.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
    assert len(calls) == 5 * 4                  # 5 one-token steps x 4 layers, all fused
    assert torch.equal(a[:, :191], b[:, :191])  # the prefill's token: same SDPA path
    assert int4.model.config._attn_implementation == "rw4_kv"
    auto_resident = AutoModel.from_pretrained(checkpoint)
    assert auto_resident.kv_cache_choice == "fp16"
    auto_streamed = RocketModel(checkpoint, vram_budget=1, window=1)
    assert auto_streamed.kv_cache_choice == "int4"
    auto_streamed.close()

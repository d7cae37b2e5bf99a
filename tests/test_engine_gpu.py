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
    streamed = RocketModel(checkpoint, vram_budget=1, window=window)  # forces streaming
    assert streamed.streamer is not None and streamed.streamer.window == 1
    streamed.close()
    rest, layers = footprint(resident.model)
    budget = rest + window * max(layers) + 1000  # room for exactly `window` layer slots
    streamed = RocketModel(checkpoint, vram_budget=budget, window=window)
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
    streamed = RocketModel(checkpoint, vram_budget=budget, window=1)
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

"""Per-expert streaming of routed experts (the reference's expert-row reads and residency,
rocketllm/base.py:1375-1464, moe/expert_cache.py:261-316): a Mixtral-architecture RW4 model whose
experts stream one by one through an expert cache produces exactly the resident model's logits and
greedy tokens, and only routed experts cross PCIe."""
import pytest
import torch

from rocketllm_b200.engine import AutoModel, RocketModel, footprint
from rocketllm_b200.expert_stream import expert_blob_bytes, is_rw4_experts
from rocketllm_b200.quant.convert import save_rw4_checkpoint

pytestmark = pytest.mark.gpu

E, LAYERS = 8, 3


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from transformers import MixtralConfig, MixtralForCausalLM
    cfg = MixtralConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=LAYERS,
                        num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                        num_local_experts=E, num_experts_per_tok=2, max_position_embeddings=512,
                        tie_word_embeddings=False)
    torch.manual_seed(0)
    model = MixtralForCausalLM(cfg)
    with torch.no_grad():
        for n, p in model.named_parameters():
            p.copy_(torch.ones_like(p) if "norm" in n else torch.randn_like(p) * 0.02)
        for layer in model.model.layers:   # decisive routing: no near-ties between the two runs
            layer.mlp.gate.weight.mul_(10.0)
    return save_rw4_checkpoint(model, str(tmp_path_factory.mktemp("rw4moe")), device="cuda")


def budget_for(model, slots, window=1):
    experts = [m for m in model.modules() if is_rw4_experts(m)]
    rest, dense = footprint(model, skip_experts=True)
    return rest + window * max(dense) + slots * expert_blob_bytes(experts[0]) + 1000


@pytest.mark.parametrize("slots", [E, 2 * E, 3 * E])
def test_streamed_experts_equal_resident(checkpoint, slots):
    ids = torch.randint(0, 2048, (1, 12), generator=torch.Generator().manual_seed(4)).cuda()
    resident = AutoModel.from_pretrained(checkpoint)
    assert resident.streamer is None
    budget = budget_for(resident.model, slots)
    streamed = RocketModel(checkpoint, vram_budget=budget, window=1, kv_cache="fp16")
    st = streamed.streamer
    assert st is not None and st.experts is not None
    # the budget beyond one layer's experts goes to pinning dense parts first, then expert slots
    assert E <= len(st.experts.slots) <= slots
    with torch.no_grad():
        assert torch.equal(resident(ids).logits, streamed(ids).logits)
        before = st.experts.stats()
        a = resident.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
        b = streamed.generate(ids, max_new_tokens=6, do_sample=False, min_new_tokens=6)
    assert torch.equal(a, b)
    after = st.experts.stats()
    eb = st.experts.slot_bytes
    # decode: at most top-2 experts per layer per token cross PCIe (the prefill of generate
    # routes 12 tokens, up to every expert)
    assert after["bytes"] - before["bytes"] <= (E + 5 * 2) * LAYERS * eb
    assert after["fetches"] > before["fetches"] or after["hits"] > before["hits"]
    if len(st.experts.slots) >= LAYERS * E:   # every expert fits: each crossed PCIe once
        assert after["fetches"] == after["resident"] <= LAYERS * E
    assert after["resident"] <= len(st.experts.slots)
    assert st.stats()["transfer"]["stalls"] == 0
    streamed.close()


def test_whole_layer_streaming_still_available(checkpoint):
    ids = torch.randint(0, 2048, (1, 8), generator=torch.Generator().manual_seed(5)).cuda()
    resident = AutoModel.from_pretrained(checkpoint)
    streamed = RocketModel(checkpoint, vram_budget=1, window=1, expert_streaming=False,
                           kv_cache="fp16")
    assert streamed.streamer.experts is None
    with torch.no_grad():
        assert torch.equal(resident(ids).logits, streamed(ids).logits)
    streamed.close()

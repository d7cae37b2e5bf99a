"""CUDA-graph greedy decode of an RW4 model replays exactly the eager static-cache decode, and the
synthetic on-device builder produces a working RW4 model."""
import pytest
import torch

from rocketllm_b200.decode import GraphedDecoder
from rocketllm_b200.synthetic import build_rw4_causal_lm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arch", ["llama", "mixtral"])
@pytest.mark.parametrize("batch", [1, 4])
def test_graph_decode_equals_eager(arch, batch):
    from transformers import LlamaConfig, MixtralConfig
    if arch == "llama":
        cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=2,
                          num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                          max_position_embeddings=256, tie_word_embeddings=False)
    else:
        cfg = MixtralConfig(hidden_size=512, intermediate_size=512, num_hidden_layers=2,
                            num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                            num_local_experts=8, num_experts_per_tok=2,
                            max_position_embeddings=256, tie_word_embeddings=False)
    model = build_rw4_causal_lm(cfg, device="cuda", seed=1)
    ids = torch.randint(0, 2048, (batch, 12), generator=torch.Generator().manual_seed(2)).cuda()
    eager = GraphedDecoder(model, batch, 64, use_graph=False).generate(ids, 10)
    graphed = GraphedDecoder(model, batch, 64, use_graph=True).generate(ids, 10)
    assert torch.equal(eager, graphed)
    with torch.no_grad():
        ref = model.generate(ids, max_new_tokens=10, min_new_tokens=10, do_sample=False)[:, 12:]
    assert torch.equal(eager, ref)


def test_full_static_cache_is_refused_on_the_host():
    from transformers import LlamaConfig
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=1,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                      max_position_embeddings=256, tie_word_embeddings=False)
    model = build_rw4_causal_lm(cfg, device="cuda", seed=1)
    dec = GraphedDecoder(model, 1, 8, use_graph=False)
    dec.prefill(torch.zeros(1, 6, dtype=torch.long, device="cuda"))
    dec.step()
    dec.step()
    with pytest.raises(ValueError, match="full"):
        dec.step()

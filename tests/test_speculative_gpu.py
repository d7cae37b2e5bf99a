"""Speculative decoding with an RW4 target on the B200: every verify pass runs the RW4 layers at
M = k+1 (the dequant-GEMV reads each weight once for all candidate positions), streamed or
resident, with the stock or the int4 KV cache.

Greedy speculation must reproduce the target's plain greedy decoding.  The RW4 GEMV gives a row the
same bits in a (k+1)-row verify pass as in a one-row step, but attention over a bf16 cache is a
library kernel whose rounding may depend on the query count (the reference documents the caveat,
``rocketllm/spec/draft.py:45-64``), so with the stock cache the sequences must agree up to the first
position where the plain run's top-1 margin is below 4e-2, and that position must exist only there.
With the int4 cache the two runs hold different caches from the first verify pass on: the pass
appends k+1 tokens at once and flushes a whole group as soon as the window passes its limit, where
one-token steps flush that group a few tokens later (the reference cache's rule, applied to the
same appends, ``rocketllm/quant/kv_cache.py:322-346``), so some queries attend over quantized keys
in one run and exact keys in the other; that case checks the first token and the pass statistics.
"""
import pytest
import torch

from rocketllm_b200.engine import AutoModel, RocketModel
from rocketllm_b200.quant.convert import save_rw4_checkpoint

pytestmark = pytest.mark.gpu

NEAR_TIE = 4e-2


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                      max_position_embeddings=1024, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():
        for n, p in model.named_parameters():
            p.copy_(torch.ones_like(p) if "norm" in n else torch.randn_like(p) * 0.02)
    return save_rw4_checkpoint(model, str(tmp_path_factory.mktemp("rw4")), device="cuda")


def _draft(checkpoint):
    """The same RW4 checkpoint, resident, as the draft: it proposes what the target would say."""
    from transformers import AutoModelForCausalLM
    return AutoModelForCausalLM.from_pretrained(checkpoint, dtype=torch.bfloat16).to("cuda")


def _agree_up_to_near_tie(spec, plain, prompt, near_tie=True):
    seq, logits = plain.sequences, plain.logits
    n = min(spec.shape[1], seq.shape[1])
    diff = (spec[0, :n] != seq[0, :n]).nonzero()
    if diff.numel() == 0:
        return n
    j = int(diff[0, 0])
    assert j > prompt  # the first token comes from the shared prefill
    if near_tie:
        top2 = logits[j - prompt][0].float().topk(2).values
        assert float(top2[0] - top2[1]) < NEAR_TIE, f"diverged at {j} with margin {top2}"
    return j


@pytest.mark.parametrize("kv", ["fp16", "int4"])
def test_streamed_speculation_matches_greedy(checkpoint, kv):
    ids = torch.randint(0, 2048, (1, 190), generator=torch.Generator().manual_seed(5)).cuda()
    n = 40
    plain = RocketModel(checkpoint, vram_budget=1, window=1, kv_cache=kv)
    plain.model.generation_config.eos_token_id = None      # exactly n tokens, nothing masked
    with torch.no_grad():
        ref = plain.generate(ids, max_new_tokens=n, do_sample=False,
                             return_dict_in_generate=True, output_logits=True)
    plain.close()
    # lookahead 3 with the int4 cache: 4 positions x 4 heads per kv head = 16 columns, so every
    # verify pass runs on the packed history (rw4_kv_attention); the fp16 cache takes 4
    spec = RocketModel(checkpoint, vram_budget=1, window=1, kv_cache=kv,
                       draft_model=_draft(checkpoint), speculative="auto",
                       lookahead=4 if kv == "fp16" else 3, max_lookahead=4 if kv == "fp16" else 3)
    spec.model.generation_config.eos_token_id = None
    assert spec.speculation_enabled()[0]          # streamed weights: "auto" speculates
    out = spec.generate(ids, max_new_tokens=n, do_sample=False)
    assert out.shape == (1, 190 + n)
    st = spec.speculation
    agree = _agree_up_to_near_tie(out, ref, 190, near_tie=kv == "fp16")
    if kv == "fp16":
        assert agree >= 190 + 8
    assert st.passes < n and st.tokens_per_pass > 2.0
    # the draft keeps exact keys while an int4 target attends over quantized ones, so near-ties
    # of this random-init model resolve differently more often
    assert st.acceptance_rate > (0.8 if kv == "fp16" else 0.5)
    spec.close()


def test_resident_auto_does_not_speculate(checkpoint):
    m = AutoModel.from_pretrained(checkpoint, draft_model=_draft(checkpoint))
    assert m.speculation_enabled() == (False, "the weights are resident; pass speculative='on' "
                                              "to force it")

"""Speculative decoding on CPU: the accept rule preserves the target distribution, greedy rules,
and greedy speculation equals plain greedy decoding at fp32 -- the reference's own three checks
(``rocketllm/spec/draft.py:26-43``: algebraic / empirical / end to end)."""
import pytest
import torch

from rocketllm_b200.speculative import (DraftIncompatible, DraftModel, SamplingParams,
                                        SpeculativeDecoder, check_compatible, resolve_speculation,
                                        verify)


def test_accept_rule_preserves_target_distribution():
    """A proposal drawn from q, accepted with min(1, p/q), else redrawn from (p - q)+: the first
    emitted token is distributed as p (Monte Carlo, 20k trials, 5-sigma bound)."""
    g = torch.Generator().manual_seed(0)
    p = torch.tensor([0.05, 0.40, 0.10, 0.30, 0.15])
    q = torch.tensor([0.30, 0.10, 0.25, 0.05, 0.30])
    spare = torch.tensor([0.2, 0.2, 0.2, 0.2, 0.2])
    n = 20000
    counts = torch.zeros(5)
    for _ in range(n):
        x = torch.multinomial(q, 1, generator=g)
        acc, tok = verify(x, q.view(1, -1), torch.stack([p, spare]), g)
        counts[int(x) if acc == 1 else tok] += 1
    freq = counts / n
    sigma = (p * (1 - p) / n).sqrt()
    assert ((freq - p).abs() <= 5 * sigma).all(), (freq, p)


def test_greedy_rules():
    v = 6
    one = lambda i: torch.nn.functional.one_hot(torch.tensor(i), v).float()  # noqa: E731
    props = torch.tensor([3, 1, 4])
    dq = torch.stack([one(3), one(1), one(4)])
    # target agrees on the first two, not the third (its argmax there is 5)
    tp = torch.stack([one(3), one(1), one(5), one(0)])
    assert verify(props, dq, tp) == (2, 5)
    # everything accepted: the bonus token comes from the spare distribution
    tp = torch.stack([one(3), one(1), one(4), one(2)])
    assert verify(props, dq, tp) == (3, 2)
    # nothing proposed: the pass still yields the target's token
    assert verify(torch.zeros(0, dtype=torch.int64), None, one(4).view(1, -1)) == (0, 4)


def _llama(layers, seed, vocab=512):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=vocab,
                      max_position_embeddings=512)
    return LlamaForCausalLM(cfg).eval()


@pytest.mark.parametrize("same_draft", [False, True])
def test_greedy_speculation_equals_greedy_fp32(same_draft):
    target = _llama(2, 0)
    draft = target if same_draft else _llama(1, 1)
    ids = torch.randint(0, 512, (1, 12), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        plain = target.generate(ids, max_new_tokens=40, min_new_tokens=40, do_sample=False)
    dec = SpeculativeDecoder(target, DraftModel(draft), lookahead=4, max_lookahead=8)
    out = dec.generate(ids, 40)
    assert torch.equal(out, plain)
    st = dec.stats
    assert st.emitted == 40
    if same_draft:   # a draft that is the target is always right: k + 1 tokens per pass
        assert st.acceptance_rate == 1.0 and st.tokens_per_pass > 4
    else:
        assert st.passes < 40 or st.acceptance_rate == 0.0


def test_end_of_sequence_truncates_like_generate():
    target = _llama(2, 0)
    ids = torch.randint(0, 512, (1, 12), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = target.generate(ids, max_new_tokens=30, min_new_tokens=30, do_sample=False)
    eos = int(ref[0, 12 + 9])          # the 10th generated token ends the run
    dec = SpeculativeDecoder(target, DraftModel(target), eos_token_id=eos)
    out = dec.generate(ids, 30)
    first = (ref[0, 12:] == eos).nonzero()[0, 0].item()
    assert torch.equal(out, ref[:, :12 + first + 1])
    dec = SpeculativeDecoder(target, DraftModel(target), eos_token_id=eos)
    assert dec.generate(ids, 30, min_new_tokens=30).shape[1] == 42   # not acted on before 30


def test_sampled_speculation_runs_and_counts():
    target = _llama(2, 0)
    draft = _llama(1, 1)
    ids = torch.randint(0, 512, (1, 8), generator=torch.Generator().manual_seed(4))
    dec = SpeculativeDecoder(target, DraftModel(draft), lookahead=3)
    out = dec.generate(ids, 25, SamplingParams(do_sample=True, temperature=0.8, top_k=50,
                                               top_p=0.9), torch.Generator().manual_seed(5))
    assert out.shape == (1, 33)
    st = dec.stats.to_dict()
    assert st["emitted"] == 25 and st["passes"] >= 1 and 0.0 <= st["acceptance_rate"] <= 1.0


def test_sampling_warp():
    s = SamplingParams(do_sample=True, temperature=1.0, top_k=2)
    probs = s.distribution(torch.tensor([[1.0, 3.0, 2.0, 0.0]]))
    assert probs[0, 0] == 0 and probs[0, 3] == 0 and torch.isclose(probs.sum(), torch.tensor(1.))
    s = SamplingParams(do_sample=True, top_p=0.5)
    probs = s.distribution(torch.tensor([[0.0, 5.0, 0.0, 0.0]]))
    assert probs[0, 1] == 1.0
    assert SamplingParams(do_sample=True, temperature=0.0).greedy


def test_compatibility_and_resolution():
    from transformers import LlamaConfig
    with pytest.raises(DraftIncompatible):
        check_compatible(LlamaConfig(vocab_size=100), None, LlamaConfig(vocab_size=101), None)
    assert check_compatible(LlamaConfig(vocab_size=100), None, LlamaConfig(vocab_size=100), None)
    assert resolve_speculation("auto", None, streamed=True)[0] is False
    assert resolve_speculation("auto", object(), streamed=True)[0] is True
    assert resolve_speculation("auto", object(), streamed=False)[0] is False
    assert resolve_speculation("on", object())[0] is True
    with pytest.raises(ValueError):
        resolve_speculation("maybe", object())


def test_speculation_over_int4_cache_crops_the_window():
    """Verify passes write k+1 positions into the int4 cache (crossing flushes) and rejected ones
    come back out of the exact window; the cache ends holding every token but the last."""
    from test_kv_cache_cpu import CpuKVOps

    from rocketllm_b200.kv_cache import RW4KVCache, enable_kv_attention
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=512,
                      max_position_embeddings=1024)
    target = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    draft = LlamaForCausalLM(LlamaConfig(**{**cfg.to_dict(), "num_hidden_layers": 1})) \
        .to(torch.bfloat16).eval()
    enable_kv_attention(target)
    caches = []

    def new_cache():
        caches.append(RW4KVCache(ops=CpuKVOps(), fused=True))
        return caches[-1]

    ids = torch.randint(0, 512, (1, 180), generator=torch.Generator().manual_seed(2))
    dec = SpeculativeDecoder(target, DraftModel(draft), lookahead=4, new_cache=new_cache)
    out = dec.generate(ids, 60)
    assert out.shape == (1, 240)
    cache = caches[0]
    assert cache.get_seq_length(0) == 239                 # every token but the last emitted
    assert cache._kv[0].groups >= 1 and cache.flushes >= 1
    assert dec.stats.passes <= 60 and dec.stats.emitted == 60


def test_warps_and_greedy_verdicts_match_the_reference():
    """Pinned to the reference's own ``SamplingParams.distribution`` and ``verify``
    (``tests/golden/reference_spec.npz``, written by ``tests/golden/make_spec_golden.py``)."""
    import os

    import numpy as np
    gold = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                     "reference_spec.npz")))
    logits = torch.from_numpy(gold["logits"])
    warps = {"greedy": dict(do_sample=False), "t07": dict(do_sample=True, temperature=0.7),
             "k5": dict(do_sample=True, temperature=1.3, top_k=5),
             "p08": dict(do_sample=True, temperature=0.9, top_p=0.8)}
    for name, kw in warps.items():
        got = SamplingParams(**kw).distribution(logits).numpy()
        np.testing.assert_allclose(got, gold[f"dist.{name}"], rtol=0, atol=1e-7, err_msg=name)
    greedy = SamplingParams()
    for c in gold["cases"].tolist():
        target = greedy.distribution(torch.from_numpy(gold[f"case{c}.target_logits"]))
        props = torch.from_numpy(gold[f"case{c}.proposals"])
        dq = torch.nn.functional.one_hot(props, target.shape[-1]).float()
        assert verify(props, dq, target) == tuple(gold[f"case{c}.result"].tolist()), c

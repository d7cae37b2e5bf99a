"""The packed-history decode attention kernel against the oracle (B200).

Each case fills an ``RW4KVCache`` on the device with seeded bf16 keys / values (a prefill and some
single-token steps, so groups have been flushed and the window is partly filled), then checks:

* the quantized storage equals the reference codec applied to the same tokens (bit-exact);
* the kernel's attention over packed history + window equals fp64 softmax attention over the
  reference's expanded history (the bf16 keys / values ``QuantizedKVCache.update`` returns), within
  2e-2 absolute on outputs of unit scale -- the tolerance of the logits bar; the kernel multiplies
  the exact codes (no bf16 rounding of the expanded keys) and rounds its operands to fp16 / bf16.
"""
import numpy as np
import pytest
import torch

from oracle import rw4_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _fill(cache, b, kvh, d, prefill, steps, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    chan = 1.0 + 4.0 * (torch.rand(d, generator=g) > 0.9).float()
    ks, vs = [], []

    def kv(t):
        k = (torch.randn(b, kvh, t, d, generator=g) * chan).to(torch.bfloat16)
        v = torch.randn(b, kvh, t, d, generator=g).to(torch.bfloat16)
        ks.append(k)
        vs.append(v)
        return k.to(dev), v.to(dev)

    if prefill:
        cache.update(*kv(prefill), 0)
    for _ in range(steps):
        cache.update(*kv(1), 0)
    return torch.cat(ks, dim=2), torch.cat(vs, dim=2)


CASES = [
    # b, heads, kv_heads, head_dim, prefill, steps
    (1, 32, 8, 128, 0, 1),        # one window token, no groups
    (1, 32, 8, 128, 150, 5),      # window only
    (1, 32, 8, 128, 191, 1),      # exactly one group flushed, window 128
    (1, 32, 8, 128, 700, 3),      # groups + window
    (2, 8, 8, 128, 330, 40),      # G = 1
    (3, 16, 2, 64, 500, 70),      # head_dim 64, G = 8, batch 3
    (1, 64, 4, 128, 900, 20),     # G = 16 (two head tiles)
    (1, 8, 2, 64, 2100, 2),       # many groups per warp
    (1, 8, 2, 128, 17000, 1),     # a cluster of 8 CTAs per head slot
]


@pytest.mark.parametrize("b,h,kvh,d,prefill,steps", CASES)
def test_kv_attention_matches_oracle(cuda, b, h, kvh, d, prefill, steps):
    from rocketllm_b200 import kernels
    from rocketllm_b200.kv_cache import RW4KVCache
    cache = RW4KVCache(fused=True)
    k_all, v_all = _fill(cache, b, kvh, d, prefill, steps, seed=b * 1000 + prefill + d, dev=cuda)
    layer = cache._kv[0]
    total = prefill + steps
    assert layer.groups * 64 + layer.rlen == total
    # the quantized storage is the reference codec of the flushed tokens, bit for bit
    if layer.groups:
        t = layer.groups * 64
        kp, ks, kz, vp, vs, vz = [x.cpu().numpy() for x in cache.quantized(0)]
        rk = O.kv_quantize(_bits(k_all[:, :, :t]), 2, 64)
        rv = O.kv_quantize(_bits(v_all[:, :, :t]), 3, 64)
        # the reference quantizes each flush as its own block; blocks are whole groups, so the
        # concatenation equals one quantize over all flushed tokens
        np.testing.assert_array_equal(kp, rk[0])
        np.testing.assert_array_equal(ks.view(np.uint16), rk[1].view(np.uint16))
        np.testing.assert_array_equal(kz.view(np.uint16), rk[2].view(np.uint16))
        np.testing.assert_array_equal(vp, rv[0])
        np.testing.assert_array_equal(vs.view(np.uint16), rv[1].view(np.uint16))
        np.testing.assert_array_equal(vz.view(np.uint16), rv[2].view(np.uint16))
    # expanded history (the reference's update output) from the device dequantize
    hk, hv = cache.history(0)
    q = torch.randn(b, h, 1, d, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    scaling = d ** -0.5
    out = cache.attend(0, q.to(cuda), scaling)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    ref = O.attention_decode(q[:, :, 0].float().numpy(), hk.float().cpu().numpy(),
                             hv.float().cpu().numpy(), scaling)
    got = out[:, 0].float().cpu().numpy()
    err = np.abs(got - ref).max()
    assert err <= ATOL, f"max abs error {err}"


def test_kv_attention_strided_query(cuda):
    """A query that is a transposed view ([b, 1, h, d] storage, as a projection's output after
    ``transpose(1, 2)``) is read through its strides."""
    from rocketllm_b200.kv_cache import RW4KVCache
    cache = RW4KVCache(fused=True)
    _fill(cache, 2, 4, 128, 260, 3, seed=5, dev=cuda)
    base = torch.randn(2, 1, 16, 128, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    q_view = base.to(cuda).transpose(1, 2)              # [2, 16, 1, 128], non-contiguous
    a = cache.attend(0, q_view, 128 ** -0.5)
    b = cache.attend(0, q_view.contiguous(), 128 ** -0.5)
    torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_kv_attention_rejects_bad_shapes(cuda):
    from rocketllm_b200 import _lib, kernels
    from rocketllm_b200.kv_cache import RW4KVCache
    cache = RW4KVCache(fused=True)
    _fill(cache, 1, 2, 128, 10, 0, seed=1, dev=cuda)
    layer = cache._kv[0]
    q = torch.zeros(1, 6, 1, 128, dtype=torch.bfloat16, device=cuda)   # 6 heads over 2 kv heads
    with pytest.raises(_lib.RW4Error):
        kernels.kv_attention_decode(q[:, :5], layer.k_codes, layer.k_sz, layer.v_codes,
                                    layer.v_sz, 0, layer.k_res, layer.v_res, layer.rlen, 1.0)
    with pytest.raises(_lib.RW4Error):   # more window tokens than the window holds
        kernels.kv_attention_decode(q, layer.k_codes, layer.k_sz, layer.v_codes, layer.v_sz, 0,
                                    layer.k_res, layer.v_res, layer.k_res.shape[2] + 1, 1.0)


def _llama(dev, head_dim, seed=0):
    """The model-parity tests' Llama (hidden 512, 3 layers, vocab 2048, N(0, 0.02) weights) with
    ``head_dim`` 64 (8 heads) or 128 (4 heads) over 2 kv heads."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=3,
                      num_attention_heads=512 // head_dim, num_key_value_heads=2,
                      vocab_size=2048, max_position_embeddings=2048, head_dim=head_dim)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).to(dev).eval()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_model_decode_fused_vs_reference_behaviour(cuda, head_dim):
    """A Llama decodes through the fused attention; at every step its logits stay within 2e-2 of
    the reference behaviour (the same cache expanding its history for SDPA), past three flushes,
    and its greedy token is the reference's wherever the reference's top-1 margin exceeds twice
    that bar (a smaller margin is a near-tie that rounding-level differences may legitimately
    flip; the random-init model has many)."""
    from rocketllm_b200.kv_cache import RW4KVCache, enable_kv_attention
    model = _llama(cuda, head_dim)
    enable_kv_attention(model)
    fused = RW4KVCache(fused=True)
    plain = RW4KVCache(fused=False)
    ids = torch.randint(0, 2048, (2, 200), generator=torch.Generator().manual_seed(2)).to(cuda)
    worst, checked = 0.0, 0
    with torch.no_grad():
        a = model(ids, past_key_values=fused, use_cache=True).logits[:, -1]
        b = model(ids, past_key_values=plain, use_cache=True).logits[:, -1]
        assert (a - b).abs().max().item() == 0.0
        tok = b.argmax(-1, keepdim=True)
        for step in range(150):
            a = model(tok, past_key_values=fused, use_cache=True).logits[:, -1]
            b = model(tok, past_key_values=plain, use_cache=True).logits[:, -1]
            worst = max(worst, (a.float() - b.float()).abs().max().item())
            top2 = b.float().topk(2, dim=-1).values
            decisive = (top2[:, 0] - top2[:, 1]) > 4e-2
            same = a.argmax(-1) == b.argmax(-1)
            assert bool((same | ~decisive).all()), f"greedy token differs at step {step}"
            checked += int(decisive.sum())
            tok = b.argmax(-1, keepdim=True)
    assert fused._kv[0].groups == plain._kv[0].groups >= 3
    assert worst <= 2e-2, worst
    assert checked >= 100        # most steps are decisive


CHUNK_CASES = [
    # b, heads, kv_heads, head_dim, prefill, q_len
    (1, 32, 8, 128, 189, 4),     # the chunk flushes a group; the window ends 1 token into a chunk
    (2, 8, 8, 128, 330, 8),      # one head per kv head, 8 positions
    (3, 16, 2, 64, 500, 2),      # 8 heads per kv head x 2 positions = 16 columns
    (1, 8, 2, 128, 17000, 3),    # a cluster of 8 CTAs per head slot
]


@pytest.mark.parametrize("b,h,kvh,d,prefill,q_len", CHUNK_CASES)
def test_kv_attention_chunk_matches_causal_oracle(cuda, b, h, kvh, d, prefill, q_len):
    """q_len query positions that are the window's last tokens attend causally over the packed
    history and the window (a speculative verify pass)."""
    from rocketllm_b200 import kernels
    from rocketllm_b200.kv_cache import RW4KVCache
    cache = RW4KVCache(fused=True, causal_chunks=True)
    _fill(cache, b, kvh, d, prefill, 0, seed=prefill + q_len, dev=cuda)
    g = torch.Generator().manual_seed(11)
    k = torch.randn(b, kvh, q_len, d, generator=g).to(torch.bfloat16)
    v = torch.randn(b, kvh, q_len, d, generator=g).to(torch.bfloat16)
    cache.update(k.to(cuda), v.to(cuda), 0)
    hk, hv = cache.history(0)
    q = torch.randn(b, h, q_len, d, generator=g).to(torch.bfloat16)
    out = cache.attend(0, q.to(cuda), d ** -0.5)          # [b, q_len, h, d]
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    ref = O.attention_causal(q.float().numpy(), hk.float().cpu().numpy(),
                             hv.float().cpu().numpy(), d ** -0.5)
    err = np.abs(out.transpose(1, 2).float().cpu().numpy() - ref).max()
    assert err <= ATOL, f"max abs error {err}"


def test_kv_attention_chunk_column_limit(cuda):
    from rocketllm_b200 import _lib, kernels
    from rocketllm_b200.kv_cache import RW4KVCache
    cache = RW4KVCache(fused=True, causal_chunks=True)
    _fill(cache, 1, 2, 128, 20, 0, seed=2, dev=cuda)
    layer = cache._kv[0]
    q = torch.zeros(1, 8, 5, 128, dtype=torch.bfloat16, device=cuda)   # 5 x 4 = 20 columns
    with pytest.raises(_lib.RW4Error):
        kernels.kv_attention_decode(q, layer.k_codes, layer.k_sz, layer.v_codes, layer.v_sz,
                                    layer.groups, layer.k_res, layer.v_res, layer.rlen, 1.0)

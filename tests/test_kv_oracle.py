"""The oracle's int4 KV cache against the reference's own ``QuantizedKVCache`` (CPU, no GPU).

``tests/golden/reference_kv.npz`` holds what the reference cache returned for a seeded prefill of
260 tokens followed by 60 single-token decode steps (``make_kv_golden.py``), and transformers' SDPA
attention of one query over the final history.  Everything here is bit-exact except the attention
(fp64 oracle vs the reference's fp32 / bf16 SDPA), which is held to a stated tolerance.
"""
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import rw4_oracle as O

KV = os.path.join(ROOT, "tests", "golden", "reference_kv.npz")


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(KV))


@pytest.fixture(scope="module")
def replay(gold):
    b, kvh, h, d, prefill, steps = gold["shape"].tolist()
    cache = O.KiviCache(group=64, residual=128)
    hk, hv = cache.update(gold["k.0"], gold["v.0"])
    first_len = hk.shape[2]
    for s in range(1, steps + 1):
        hk, hv = cache.update(gold[f"k.{s}"], gold[f"v.{s}"])
    return cache, hk, hv, first_len


def test_prefill_history_length(gold, replay):
    assert replay[3] == int(gold["hist_len.0"])


def test_history_bit_exact(gold, replay):
    _, hk, hv, _ = replay
    np.testing.assert_array_equal(hk, gold["hist_k.last"])
    np.testing.assert_array_equal(hv, gold["hist_v.last"])


def test_blocks_bit_exact(gold, replay):
    cache = replay[0]
    assert [t for _, _, t in cache.blocks] == gold["blocks"].tolist()
    assert cache.k.shape[2] == int(gold["residual"])
    for i, (kb, vb, _) in enumerate(cache.blocks):
        for name, blk in (("kb", kb), ("vb", vb)):
            np.testing.assert_array_equal(blk[0], gold[f"{name}{i}.packed"])
            np.testing.assert_array_equal(blk[1].view(np.uint16),
                                          gold[f"{name}{i}.scale"].view(np.uint16))
            np.testing.assert_array_equal(blk[2].view(np.uint16),
                                          gold[f"{name}{i}.zero"].view(np.uint16))


def test_attention_matches_sdpa(gold, replay):
    _, hk, hv, _ = replay
    d = hk.shape[-1]
    q = O.bf16_bits_to_f32(gold["q"])[:, :, 0, :]
    out = O.attention_decode(q, O.bf16_bits_to_f32(hk), O.bf16_bits_to_f32(hv), d ** -0.5)
    ref32 = gold["attn_f32"][:, 0]                      # [b, h, d] fp32 SDPA
    np.testing.assert_allclose(out, ref32, rtol=0, atol=2e-6)
    ref16 = O.bf16_bits_to_f32(gold["attn"])[:, 0]      # the bf16 model's SDPA output
    assert np.abs(out - ref16).max() <= 2e-2


def test_window_never_flushes_a_partial_group():
    # 128 + 63 tokens stay exact; the 192nd moves exactly one group of 64
    rng = np.random.default_rng(0)
    cache = O.KiviCache(group=64, residual=128)
    for t in range(191):
        x = O.f32_to_bf16_bits(rng.standard_normal((1, 1, 1, 64)).astype(np.float32))
        cache.update(x, x)
    assert cache.quantized_tokens() == 0 and cache.k.shape[2] == 191
    x = O.f32_to_bf16_bits(rng.standard_normal((1, 1, 1, 64)).astype(np.float32))
    hk, _ = cache.update(x, x)
    assert cache.quantized_tokens() == 64 and cache.k.shape[2] == 128 and hk.shape[2] == 192


def test_causal_attention_matches_sdpa_with_a_cache_mask():
    """``attention_causal``: Q query positions that are the last Q of T keys, each seeing keys up to
    its own position -- torch SDPA with the bottom-right aligned causal mask, in fp64."""
    import torch
    rng = np.random.default_rng(3)
    b, h, kvh, q_len, t, d = 2, 8, 2, 4, 37, 64
    q = rng.standard_normal((b, h, q_len, d)).astype(np.float32)
    k = rng.standard_normal((b, kvh, t, d)).astype(np.float32)
    v = rng.standard_normal((b, kvh, t, d)).astype(np.float32)
    out = O.attention_causal(q, k, v, d ** -0.5)
    mask = torch.arange(t)[None, :] <= (t - q_len + torch.arange(q_len))[:, None]
    kk = torch.from_numpy(k).double().repeat_interleave(h // kvh, dim=1)
    vv = torch.from_numpy(v).double().repeat_interleave(h // kvh, dim=1)
    ref = torch.nn.functional.scaled_dot_product_attention(
        torch.from_numpy(q).double(), kk, vv, attn_mask=mask, scale=d ** -0.5)
    np.testing.assert_allclose(out, ref.numpy(), rtol=0, atol=1e-6)
    np.testing.assert_allclose(O.attention_causal(q[:, :, -1:], k, v, d ** -0.5)[:, :, 0],
                               O.attention_decode(q[:, :, -1], k, v, d ** -0.5), atol=1e-7)


# -- codec properties the reference's own suite asserts (tests/test_kv_cache.py:38-138), stated
#    here for the oracle codec on bf16 keys / values --------------------------------------------

def _kv_bits(shape, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return O.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def _round_trip(bits, axis):
    length = bits.shape[axis]
    p, s, z, _ = O.kv_quantize(bits, axis, 64)
    return O.kv_dequantize(p, s, z, axis, length, out="f32")


@pytest.mark.parametrize("axis", [2, 3])
def test_round_trip_within_half_a_step(axis):
    """Every value comes back within half its group's step ((max - min) / 15), plus a little for
    the scale and zero being stored in fp16."""
    bits = _kv_bits((1, 2, 256, 128), seed=axis)
    x = O.bf16_bits_to_f32(bits)
    back = _round_trip(bits, axis)
    moved = np.moveaxis(x, axis, -1)
    grouped = moved.reshape(moved.shape[:-1] + (-1, 64))
    spread = grouped.max(-1) - grouped.min(-1)
    err = np.abs(np.moveaxis(back, axis, -1).reshape(grouped.shape) - grouped).max(-1)
    assert np.all(err <= spread / 30 + spread * 1e-3 + 1e-4)


def test_constant_and_ragged_groups_are_exact():
    const = O.f32_to_bf16_bits(np.full((1, 1, 64, 64), 0.375, np.float32))
    assert np.array_equal(_round_trip(const, 2), O.bf16_bits_to_f32(const))
    # 100 tokens: the last group is padded by repeating its last value, which cannot widen it
    ragged = O.f32_to_bf16_bits(np.full((1, 1, 100, 8), 5.0, np.float32))
    assert np.array_equal(_round_trip(ragged, 2), O.bf16_bits_to_f32(ragged))


def test_an_axis_shorter_than_a_group():
    bits = _kv_bits((1, 2, 8, 16), seed=4)
    p, s, z, pad = O.kv_quantize(bits, 3, 64)
    assert s.shape[-1] == 1 and pad == 0              # one group of 16
    back = O.kv_dequantize(p, s, z, 3, 16, out="f32")
    assert back.shape == bits.shape
    assert np.abs(back - O.bf16_bits_to_f32(bits)).max() < 1.0


def test_four_bits_per_value():
    bits = _kv_bits((1, 2, 1024, 64), seed=5)
    p, s, z, _ = O.kv_quantize(bits, 2, 64)
    assert p.dtype == np.uint8 and p.nbytes + s.nbytes + z.nbytes < bits.size * 2 / 3


def test_keys_need_per_channel_groups():
    """With one outlier channel, grouping keys along tokens (a scale per channel) keeps the other
    channels accurate; grouping along channels (the value layout) would not."""
    x = np.random.default_rng(3).standard_normal((1, 2, 256, 64)).astype(np.float32)
    x[..., 7] *= 30.0
    bits = O.f32_to_bf16_bits(x)
    xf = O.bf16_bits_to_f32(bits)
    others = [c for c in range(64) if c != 7]
    good = np.abs(_round_trip(bits, 2)[..., others] - xf[..., others]).mean()
    bad = np.abs(_round_trip(bits, 3)[..., others] - xf[..., others]).mean()
    assert good * 3 < bad

"""The oracle against the reference's own outputs (golden fixtures made by make_golden.py).

Pins the CPU restatement in oracle/rw4_oracle.py bit for bit to RocketLLM's int4 codec
(rocketllm/quant/kv_cache.py:190-272) and to transformers' Mixtral router, which the GPU parity
tests then compare against.  Also restates the reference's own known-answer tests for the codec
(tests/test_kv_cache.py:39-111): half-step round-trip bound, constant groups exact, ragged tails.
"""
import numpy as np
import pytest

from oracle import rw4_oracle as o

CODEC_CASES = ["f32_aligned", "f32_ragged", "bf16_aligned", "bf16_ragged", "f16_aligned",
               "f16_ragged", "f16_wide", "const"]


def _dtype(w):
    """The reference tensor's dtype from its stored form (bf16 is kept as its uint16 bits)."""
    return {np.dtype(np.uint16): "bf16", np.dtype(np.float16): "f16"}.get(w.dtype, "f32")


def _u(a):
    a = np.asarray(a)
    return a.view({2: np.uint16, 4: np.uint32, 1: np.uint8}[a.dtype.itemsize])


@pytest.mark.parametrize("case", CODEC_CASES)
def test_quantize_matches_reference(golden, case):
    w = golden[f"{case}.w"]
    packed, scale, zero, padding = o.quantize(w, 64, _dtype(w))
    assert np.array_equal(packed, golden[f"{case}.packed"])
    assert np.array_equal(_u(scale), _u(golden[f"{case}.scale"]))
    assert np.array_equal(_u(zero), _u(golden[f"{case}.zero"]))
    assert padding == int(golden[f"{case}.padding"])


@pytest.mark.parametrize("case", CODEC_CASES)
def test_dequantize_matches_reference(golden, case):
    w = golden[f"{case}.w"]
    deq = o.dequantize(golden[f"{case}.packed"], golden[f"{case}.scale"], golden[f"{case}.zero"],
                       k=w.shape[1], out=_dtype(w))
    assert np.array_equal(_u(deq), _u(golden[f"{case}.deq"]))


def test_sweep_format_dequant_and_linear(golden):
    p, s, z = golden["sweep.packed"], golden["sweep.scale"], golden["sweep.zero"]
    assert np.array_equal(o.dequantize(p, s, z, out="bf16"), golden["sweep.deq_bf16"])
    assert np.array_equal(_u(o.dequantize(p, s, z, out="f32")), _u(golden["sweep.deq_f32"]))
    y = o.linear(golden["sweep.x"], p, s, z)
    ref = golden["sweep.y_f32"]
    assert np.abs(y - ref).max() <= 1e-5 * (1 + np.abs(ref).max())


def test_torch_port_dequant_matches_reference(golden):
    """The torch restatement the CPU baseline times (oracle/cpu_decode.py) gives the reference's
    fp32 dequantization bit for bit."""
    import torch

    from oracle import cpu_decode
    p, s, z = golden["sweep.packed"], golden["sweep.scale"], golden["sweep.zero"]
    got = cpu_decode.dequantize_torch(torch.from_numpy(p), torch.from_numpy(s),
                                      torch.from_numpy(z)).numpy()
    assert np.array_equal(_u(got), _u(golden["sweep.deq_f32"]))


def test_nibble_order_known_answer(golden):
    assert np.array_equal(o.pack(golden["pack.codes"]), golden["pack.packed"])
    assert o.pack(np.array([[1, 2]], np.uint8))[0, 0] == 0x21
    assert np.array_equal(o.unpack(np.array([[0x21, 0xF0]], np.uint8)), golden["pack.unpacked"])


def test_router_topk_and_selection(golden):
    idx, w = o.router_topk(golden["router.hidden"], golden["router.weight"], 2)
    assert np.array_equal(idx, golden["router.indices"])
    assert np.abs(w - golden["router.scores"]).max() < 1e-6
    assert o.router_selection(idx) == tuple(golden["router.selection"].tolist())


def test_round_trip_within_half_a_step():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((32, 256)).astype(np.float32)
    p, s, z, _ = o.quantize(w)
    back = o.dequantize(p, s, z)
    g = w.reshape(32, 4, 64)
    spread = g.max(-1) - g.min(-1)
    err = np.abs(back.reshape(32, 4, 64) - g).max(-1)
    assert np.all(err <= spread / 15 / 2 + spread * 1e-3 + 1e-4)


def test_constant_and_ragged_groups_are_exact():
    w = np.full((2, 100), 5.0, np.float32)
    p, s, z, pad = o.quantize(w)
    assert pad == 28
    assert np.array_equal(o.dequantize(p, s, z, k=100), w)


def test_moe_permute_and_combine_invert():
    rng = np.random.default_rng(5)
    T, k, E, H = 9, 2, 4, 8
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int64)
    perm, off = o.moe_permute(idx, E)
    assert off[0] == 0 and off[-1] == T * k
    flat = idx.reshape(-1)
    for e in range(E):
        rows = perm[off[e]:off[e + 1]]
        assert np.all(flat[rows] == e) and np.all(np.diff(rows) > 0)
    y_tok = rng.standard_normal((T, H)).astype(np.float32)
    y_perm = y_tok[perm // k]
    wts = np.full((T, k), 0.5, np.float32)
    assert np.allclose(o.moe_combine(y_perm, perm, wts, T, k), y_tok, atol=1e-6)

"""GPU parity of the codec kernels with the reference codec: bit-exact, through the C ABI."""
import numpy as np
import pytest
import torch

from oracle import rw4_oracle as o
from rocketllm_b200 import kernels

pytestmark = pytest.mark.gpu

CODEC_CASES = ["f32_aligned", "f32_ragged", "bf16_aligned", "bf16_ragged", "f16_aligned",
               "f16_ragged", "f16_wide", "const"]


def to_dev(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(a).to(dev)


def bits(t):
    t = t.cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    return t.numpy()


@pytest.mark.parametrize("case", CODEC_CASES)
def test_quantize_bit_exact_with_reference(golden, cuda, case):
    w = golden[f"{case}.w"]
    packed, scale, zero, pad = kernels.quantize(to_dev(w, cuda), 64)
    assert np.array_equal(bits(packed), golden[f"{case}.packed"])
    assert np.array_equal(bits(scale), golden[f"{case}.scale"].view(np.uint16))
    assert np.array_equal(bits(zero), golden[f"{case}.zero"].view(np.uint16))
    assert pad == int(golden[f"{case}.padding"])


@pytest.mark.parametrize("case", CODEC_CASES)
def test_dequantize_bit_exact_with_reference(golden, cuda, case):
    w = golden[f"{case}.w"]
    # the reference dequantizes to the weight's own dtype (bf16 is stored as its uint16 bits)
    dtype = {np.dtype(np.uint16): torch.bfloat16, np.dtype(np.float16): torch.float16}.get(
        w.dtype, torch.float32)
    out = kernels.dequantize(to_dev(golden[f"{case}.packed"], cuda),
                             to_dev(golden[f"{case}.scale"], cuda),
                             to_dev(golden[f"{case}.zero"], cuda), k=w.shape[1], dtype=dtype)
    ref = golden[f"{case}.deq"]
    assert np.array_equal(bits(out), ref.view({2: np.uint16, 4: np.uint32}[ref.dtype.itemsize]))


def test_sweep_format_dequant_bit_exact(golden, cuda):
    args = [to_dev(golden[f"sweep.{n}"], cuda) for n in ("packed", "scale", "zero")]
    assert np.array_equal(bits(kernels.dequantize(*args)), golden["sweep.deq_bf16"])
    assert np.array_equal(bits(kernels.dequantize(*args, dtype=torch.float32)),
                          golden["sweep.deq_f32"].view(np.uint32))


@pytest.mark.parametrize("n,k", [(33, 4096), (7, 320), (128, 14336), (3, 96)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_dequantize_matches_oracle_random(cuda, n, k, dtype):
    gen = torch.Generator().manual_seed(n * k)
    w = torch.randn(n, k, generator=gen) * 0.02
    p, s, z, _ = o.quantize(w.numpy(), 64, "f32")
    out = kernels.dequantize(to_dev(p, cuda), to_dev(s, cuda), to_dev(z, cuda), k=k, dtype=dtype)
    ref = o.dequantize(p, s, z, k=k, out={torch.bfloat16: "bf16", torch.float32: "f32",
                                           torch.float16: "f16"}[dtype])
    assert np.array_equal(bits(out), ref.view({2: np.uint16, 4: np.uint32}[ref.dtype.itemsize]))


@pytest.mark.parametrize("n,k", [(257, 4096), (64, 200), (1, 64)])
def test_quantize_matches_oracle_random(cuda, n, k):
    gen = torch.Generator().manual_seed(n + k)
    for dtype, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        w = (torch.randn(n, k, generator=gen) * 0.05).to(dtype)
        packed, scale, zero, pad = kernels.quantize(w.to(cuda), 64)
        wnp = bits(w) if dtype == torch.bfloat16 else w.numpy()
        p, s, z, pd = o.quantize(wnp, 64, tag)
        assert np.array_equal(bits(packed), p)
        assert np.array_equal(bits(scale), s.view(np.uint16))
        assert np.array_equal(bits(zero), z.view(np.uint16))
        assert pad == pd


def test_quantize_dequantize_round_trip_full_size(cuda):
    """Size-independent property at a full sweep shape: encoding any weight and decoding it again
    lands every value within half a quantization step of its group (the reference's own bound,
    tests/test_kv_cache.py:39-70), and re-encoding a decoded weight is a fixed point of decode."""
    gen = torch.Generator(device=cuda).manual_seed(9)
    w = torch.randn(14336, 4096, device=cuda, generator=gen) * 0.02
    p, s, z, _ = kernels.quantize(w, 64)
    back = kernels.dequantize(p, s, z, dtype=torch.float32)
    g = w.view(14336, 64, 64)
    spread = g.amax(-1) - g.amin(-1)
    err = (back.view(14336, 64, 64) - g).abs().amax(-1)
    assert bool(torch.all(err <= spread / 30 + spread * 1e-3 + 1e-4))
    # decode(encode(decode(q))) == decode(q) up to the fp16 rounding of the new scale
    p2, s2, z2, _ = kernels.quantize(back, 64)
    again = kernels.dequantize(p2, s2, z2, dtype=torch.float32)
    assert bool(torch.all((again - back).abs() <= s.float().repeat_interleave(64, 1) * 0.51))

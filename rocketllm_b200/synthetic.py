"""Seeded synthetic RW4 inputs, shaped like the isolated dequant-matmul sweep.

Weights: uniform random code bytes, per-group scale ~ U[0.005, 0.02], zero = -8 * scale (so every
weight is (code - 8) * scale, centred on zero), group 64.  Activations: bf16 N(0, 1).
Generated on the target device with ``torch.Generator`` seeds so host and device agree bit for bit.
"""
import torch

# The isolated sweep's weight shapes (K, N) and batch sizes M.
SWEEP_SHAPES = ((4096, 4096), (4096, 14336), (14336, 4096), (8192, 28672), (16384, 53248))
SWEEP_M = (1, 4, 16, 64, 512, 2048)


def make_weight(n, k, device="cuda", seed=0, group=64):
    """``(packed u8 [n, k/2], scale f16 [n, k/group], zero f16 [n, k/group])``."""
    gen = torch.Generator(device=device).manual_seed(seed)
    packed = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=device, generator=gen)
    gen.manual_seed(seed + 1)
    scale = (0.005 + 0.015 * torch.rand((n, k // group), device=device, generator=gen)).to(
        torch.float16)
    zero = (-8.0 * scale.float()).to(torch.float16)
    return packed, scale, zero


def make_activation(m, k, device="cuda", seed=2):
    gen = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((m, k), device=device, generator=gen).to(torch.bfloat16)


def algorithmic_bytes(m, k, n, group=64):
    """Bytes one ``y = x W^T`` call must move at least once: codes, scales, zeros, x and y."""
    return n * k // 2 + 2 * 2 * (k // group) * n + 2 * m * k + 2 * m * n


def flops(m, k, n):
    return 2 * m * n * k

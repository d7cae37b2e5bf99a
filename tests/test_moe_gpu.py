"""GPU parity of the routed-expert kernels with the oracle and with transformers' own experts.

Permutation and combine are integer / fixed-order work and must match exactly; the grouped RW4 GEMV
matches the oracle within the bf16 tolerance of tests/test_linear_gpu.py.
"""
import numpy as np
import pytest
import torch

from oracle import rw4_oracle as o
from rocketllm_b200 import kernels
from rocketllm_b200.synthetic import make_weight

pytestmark = pytest.mark.gpu


def bits(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def close(y, ref, rel=1 / 128):
    """|y - ref| <= rel * |ref| + 2e-3 * rms(ref).  rel = 1/128 is one bf16 rounding; the SwiGLU
    output passes through three bf16 roundings (gate, up, activation) before the final one, so a
    one-ulp difference in the gate can move it by up to four ulps: rel = 1/32 there."""
    y = y.float().cpu().numpy()
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-12
    err = np.abs(y - ref)
    bound = np.abs(ref) * rel + 2e-3 * rms
    assert np.all(err <= bound), f"max err {err.max():.4g}, worst excess {(err - bound).max():.4g}"


def routing(t, k, e, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)]).to(torch.int64)


@pytest.mark.parametrize("t,k,e", [(1, 2, 8), (5, 2, 8), (37, 2, 8), (64, 4, 16), (3, 1, 1)])
def test_permute_matches_oracle(cuda, t, k, e):
    idx = routing(t, k, e, t * 7 + e)
    perm, inv, offsets = kernels.moe_permute(idx.to(cuda), e)
    p_ref, off_ref = o.moe_permute(idx.numpy(), e)
    assert np.array_equal(perm.cpu().numpy(), p_ref)
    assert np.array_equal(offsets.cpu().numpy(), off_ref)
    inv_ref = np.empty_like(p_ref)
    inv_ref[p_ref] = np.arange(p_ref.size)
    assert np.array_equal(inv.cpu().numpy(), inv_ref)


def test_permute_drops_out_of_range_ids(cuda):
    idx = torch.tensor([[0, 3], [9, 1], [-1, 3]], dtype=torch.int64)
    perm, inv, offsets = kernels.moe_permute(idx.to(cuda), 4)
    assert offsets.cpu().tolist() == [0, 1, 2, 2, 4]
    assert inv.cpu().tolist() == [0, 2, -1, 1, -1, 3]
    assert perm.cpu().tolist() == [0, 3, 1, 5, -1, -1]


def test_gather(cuda):
    x = torch.randn(6, 64, device=cuda).to(torch.bfloat16)
    idx = routing(6, 2, 4, 1).to(cuda)
    perm, inv, offsets = kernels.moe_permute(idx, 4)
    xp = kernels.moe_gather(x, perm, 2)
    assert torch.equal(xp, x[(perm.long() // 2)])


def expert_weights(e, n, k, device, seed):
    return [make_weight(n, k, device=device, seed=seed + 3 * i) for i in range(e)]


def oracle_grouped(x_perm, offsets, weights, act, inter=None):
    xb = bits(x_perm)
    off = offsets.cpu().numpy()
    outs = []
    for e, w in enumerate(weights):
        rows = slice(off[e], off[e + 1])
        if off[e + 1] == off[e]:
            continue
        p, s, z = (a.cpu().numpy() for a in w)
        h = o.linear(xb[rows], p, s, z)
        if act == 1:
            h = o.round_bf16(o.silu(o.round_bf16(h[:, :inter]))) * o.round_bf16(h[:, inter:])
        outs.append((rows, h))
    return outs


@pytest.mark.parametrize("t,act", [(1, 0), (5, 0), (40, 0), (1, 1), (12, 1), (40, 1)])
def test_grouped_matches_oracle(cuda, t, act):
    e, k_top, hid, inter = 8, 2, 1024, 512
    n = 2 * inter if act == 1 else hid
    weights = expert_weights(e, n, hid, cuda, seed=11 + act)
    idx = routing(t, k_top, e, 100 + t).to(cuda)
    x = torch.randn(t, hid, device=cuda).to(torch.bfloat16)
    perm, inv, offsets = kernels.moe_permute(idx, e)
    xp = kernels.moe_gather(x, perm, k_top)
    y = kernels.moe_grouped(xp, offsets, weights, act=act, max_rows=t * k_top)
    torch.cuda.synchronize()
    for rows, ref in oracle_grouped(xp, offsets, weights, act, inter):
        close(y[rows], ref, rel=1 / 32 if act == 1 else 1 / 128)


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("hid", [1024, 4096])
@pytest.mark.parametrize("sigma", [1e-3, 1.0])
def test_grouped_one_token(cuda, act, hid, sigma):
    """One token (each routed expert gets one row, max_rows=1), small and unit activations."""
    e, k_top, inter = 8, 2, 512
    n = 2 * inter if act == 1 else hid
    weights = expert_weights(e, n, hid, cuda, seed=21 + act)
    idx = routing(1, k_top, e, 7).to(cuda)
    x = (torch.randn(1, hid, device=cuda) * sigma).to(torch.bfloat16)
    perm, inv, offsets = kernels.moe_permute(idx, e)
    xp = kernels.moe_gather(x, perm, k_top)
    y = kernels.moe_grouped(xp, offsets, weights, act=act, max_rows=1)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    for rows, ref in oracle_grouped(xp, offsets, weights, act, inter):
        close(y[rows], ref, rel=1 / 32 if act == 1 else 1 / 128)


@pytest.mark.parametrize("act", [0, 1])
def test_grouped_token_independent_of_batch(cuda, act):
    """A token's expert outputs have the same bits alone (a one-token step) and among 24 tokens."""
    e, k_top, hid, inter = 8, 2, 1024, 512
    n = 2 * inter if act == 1 else hid
    weights = expert_weights(e, n, hid, cuda, seed=31 + act)
    idx = routing(24, k_top, e, 9).to(cuda)
    x = torch.randn(24, hid, device=cuda).to(torch.bfloat16)

    def run(xt, it):
        perm, inv, offsets = kernels.moe_permute(it, e)
        y = kernels.moe_grouped(kernels.moe_gather(xt, perm, k_top), offsets, weights, act=act,
                                max_rows=xt.shape[0] * k_top)
        return y[inv.long()].view(xt.shape[0], k_top, -1)   # per (token, slot)

    together = run(x, idx)
    for t in (0, 5, 23):
        assert torch.equal(run(x[t:t + 1], idx[t:t + 1])[0], together[t]), f"token {t}"


def test_grouped_flags_rows_beyond_max_rows(cuda):
    """An expert with more rows than max_rows covers is reported in the device status word."""
    e, hid = 4, 1024
    weights = expert_weights(e, hid, hid, cuda, seed=3)
    idx = torch.tensor([[0], [0], [1]], dtype=torch.int64, device=cuda)   # expert 0: two rows
    x = torch.randn(3, hid, device=cuda).to(torch.bfloat16)
    perm, inv, offsets = kernels.moe_permute(idx, e)
    xp = kernels.moe_gather(x, perm, 1)
    kernels.moe_grouped(xp, offsets, weights, act=0, max_rows=1)
    torch.cuda.synchronize()
    assert kernels.device_status() & 4


def test_combine_reproduces_reference_rounding_order(cuda):
    t, k, e, h = 9, 2, 4, 64
    idx = routing(t, k, e, 5)
    w = torch.rand(t, k, generator=torch.Generator().manual_seed(6))
    y_perm = torch.randn(t * k, h, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    perm, inv, offsets = kernels.moe_permute(idx.to(cuda), e)
    out = kernels.moe_combine(y_perm.to(cuda), inv, idx.to(cuda), w.to(cuda))
    # the reference: for expert in ascending order, final.index_add_(bf16(y * w)) on a bf16 tensor
    inv_c = inv.cpu()
    ref = torch.zeros(t, h, dtype=torch.bfloat16)
    for ex in range(e):
        for tok in range(t):
            for j in range(k):
                if idx[tok, j] == ex:
                    contrib = (y_perm[inv_c[tok * k + j]].float() * w[tok, j]).to(torch.bfloat16)
                    ref[tok] = (ref[tok].float() + contrib.float()).to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref)


def test_full_moe_layer_against_transformers_experts(cuda):
    """Routed experts end to end vs transformers' MixtralExperts on the dequantized weights."""
    from transformers import MixtralConfig
    from transformers.models.mixtral.modeling_mixtral import MixtralExperts
    e, k_top, hid, inter, t = 8, 2, 1024, 512, 6
    gate_up = expert_weights(e, 2 * inter, hid, cuda, seed=40)
    down = expert_weights(e, hid, inter, cuda, seed=80)
    cfg = MixtralConfig(hidden_size=hid, intermediate_size=inter, num_local_experts=e,
                        num_experts_per_tok=k_top)
    cfg._experts_implementation = "eager"
    ref_mod = MixtralExperts(cfg).to(cuda, torch.bfloat16)
    with torch.no_grad():
        for i in range(e):
            ref_mod.gate_up_proj[i].copy_(kernels.dequantize(*gate_up[i]))
            ref_mod.down_proj[i].copy_(kernels.dequantize(*down[i]))
    x = torch.randn(t, hid, device=cuda).to(torch.bfloat16)
    idx = routing(t, k_top, e, 9).to(cuda)
    w = torch.softmax(torch.randn(t, k_top, device=cuda), -1)
    with torch.no_grad():
        ref = ref_mod(x, idx, w).float().cpu().numpy()
    perm, inv, offsets = kernels.moe_permute(idx, e)
    xp = kernels.moe_gather(x, perm, k_top)
    act = kernels.moe_grouped(xp, offsets, gate_up, act=1, max_rows=t * k_top)
    yp = kernels.moe_grouped(act, offsets, down, act=0, max_rows=t * k_top)
    out = kernels.moe_combine(yp, inv, idx, w)
    y = out.float().cpu().numpy()
    rms = float(np.sqrt(np.mean(ref ** 2)))
    assert np.abs(y - ref).max() <= 0.05 * rms + np.abs(ref).max() / 64

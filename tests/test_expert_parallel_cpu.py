"""Expert parallelism over two gloo ranks on the CPU: the count / row / id exchange and the return
trip reproduce the single-process routed-experts result exactly.  The local operations are a CPU
implementation of the same four steps (the oracle's permutation, a dense SwiGLU expert), injected
in place of the CUDA kernels; what is tested is the partitioning and the collectives."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import rw4_oracle as o

E, K_TOP, H, I = 8, 2, 32, 16


class CpuOps:
    def __init__(self, weights):
        self.w = weights  # {global expert: (w_gate_up [2I, H], w_down [H, I])}

    def permute(self, idx, num_experts):
        # the CUDA kernel's contract: slots whose id is outside [0, E) are dropped (perm -1 at
        # the end, inv -1); the rest are the oracle's stable sort
        flat = idx.numpy().reshape(-1)
        ok = (flat >= 0) & (flat < num_experts)
        sub, off = o.moe_permute(flat[ok].reshape(-1, 1), num_experts)
        perm = np.full(flat.shape, -1, np.int32)
        perm[:sub.size] = np.nonzero(ok)[0][sub].astype(np.int32)
        inv = np.full(perm.shape, -1, np.int32)
        valid = perm >= 0
        inv[perm[valid]] = np.arange(perm.size, dtype=np.int32)[valid]
        return torch.from_numpy(perm), torch.from_numpy(inv), torch.from_numpy(off)

    def gather(self, x, perm, k):
        out = torch.zeros((perm.numel(), x.shape[1]), dtype=x.dtype)
        ok = perm >= 0
        out[ok] = x[perm[ok].long() // k]
        return out

    def experts(self, rows, offsets, gate_up, down, max_rows):
        out = torch.zeros_like(rows)
        for e in range(offsets.numel() - 1):
            a, b = int(offsets[e]), int(offsets[e + 1])
            if b > a:
                wgu, wd = gate_up[e], down[e]
                hgu = rows[a:b] @ wgu.T
                out[a:b] = (torch.nn.functional.silu(hgu[:, :I]) * hgu[:, I:]) @ wd.T
        return out

    def combine(self, y_rows, inv, idx, w):
        t, k = w.shape
        out = torch.zeros((t, y_rows.shape[1]), dtype=y_rows.dtype)
        for tok in range(t):
            for j in sorted(range(k), key=lambda j: int(idx[tok, j])):
                r = int(inv[tok * k + j])
                if r >= 0:
                    out[tok] += w[tok, j] * y_rows[r]
        return out


def make_problem(seed):
    g = torch.Generator().manual_seed(seed)
    weights = [(torch.randn(2 * I, H, generator=g) * 0.1, torch.randn(H, I, generator=g) * 0.1)
               for _ in range(E)]
    return weights


def tokens(rank, t):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(t, H, generator=g)
    idx = (torch.stack([torch.randperm(E, generator=g)[:K_TOP] for _ in range(t)]) if t
           else torch.empty(0, K_TOP, dtype=torch.long))
    w = torch.softmax(torch.randn(t, K_TOP, generator=g), -1)
    return x, idx, w


def single_process(x, idx, w, weights):
    ops = CpuOps(None)
    perm, inv, off = ops.permute(idx, E)
    rows = ops.gather(x, perm, K_TOP)
    y = ops.experts(rows, off, [a for a, _ in weights], [b for _, b in weights], rows.shape[0])
    return ops.combine(y, inv, idx, w)


def _worker(rank, world, port, t_per_rank, out, fixed=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from rocketllm_b200.expert_parallel import ExpertParallelMoE
    weights = make_problem(0)
    per = E // world
    mine = weights[rank * per:(rank + 1) * per]
    moe = ExpertParallelMoE(E, [a for a, _ in mine], [b for _, b in mine], ops=CpuOps(None),
                            fixed_capacity=fixed)
    x, idx, w = tokens(rank, t_per_rank[rank])
    y = moe(x, idx, w)
    ref = single_process(x, idx, w, weights)
    out[rank] = float((y - ref).abs().max()) if y.numel() else 0.0
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("t_per_rank", [(5, 7), (1, 0), (16, 16)])
def test_expert_parallel_matches_single_process(t_per_rank):
    world = 2
    port = 29500 + sum(t_per_rank) * 7 % 300
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(world, port, t_per_rank, out), nprocs=world, join=True)
        # fp32 matmuls batch rows differently on each side: equal to rounding
        assert all(out[r] <= 1e-6 for r in range(world)), dict(out)


@pytest.mark.parametrize("world,t", [(2, 5), (2, 1), (4, 3)])
def test_fixed_capacity_exchange_matches_single_process(world, t):
    """Zero-padded fixed-size buffers (no host round trip): the same result (equal token counts
    on every rank, as the mode requires)."""
    port = 29900 + world * 10 + t
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(world, port, (t,) * world, out, True), nprocs=world, join=True)
        assert all(out[r] <= 1e-6 for r in range(world)), dict(out)

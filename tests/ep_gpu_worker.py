"""Worker for tests/test_expert_parallel_gpu.py: run under torchrun, one rank per GPU (NCCL).

Every rank builds the same RW4 Mixtral-style experts (seeded), keeps its own tokens, and checks the
expert-parallel layer against the single-GPU routed-experts path on its tokens: bitwise equal."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    from rocketllm_b200 import kernels
    from rocketllm_b200.expert_parallel import ExpertParallelMoE, shard_experts
    from rocketllm_b200.quant.modules import rw4_experts_forward
    from rocketllm_b200.synthetic import make_weight
    import datetime
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    E, H, I, K_TOP = 8, 1024, 512, 2

    class Experts(torch.nn.Module):
        pass
    ex = Experts()
    for name, (n, k) in (("gate_up_proj", (2 * I, H)), ("down_proj", (H, I))):
        trip = [make_weight(n, k, device=dev, seed=31 * e + (n == H)) for e in range(E)]
        for j, sfx in enumerate(("_packed", "_scale", "_zero_point")):
            ex.register_parameter(name + sfx, torch.nn.Parameter(
                torch.stack([t[j] for t in trip]), requires_grad=False))
    ex.num_experts = E
    failures = 0
    for t in (1, 5, 32):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + t)
        x = torch.randn(t, H, device=dev, generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(E, device=dev, generator=g)[:K_TOP] for _ in range(t)])
        w = torch.softmax(torch.randn(t, K_TOP, device=dev, generator=g), -1)
        # the single-GPU routed experts on the same kernels (max_rows = t*k: the bf16 grouped
        # GEMV, as the exchange's receiving side uses; a one-token step on one GPU would take the
        # fp16 one-row kernel, equal within rounding but not bit for bit)
        trip = {n: [(getattr(ex, n + "_packed")[e], getattr(ex, n + "_scale")[e],
                     getattr(ex, n + "_zero_point")[e]) for e in range(E)]
                for n in ("gate_up_proj", "down_proj")}
        perm, inv, off = kernels.moe_permute(idx, E)
        xp = kernels.moe_gather(x, perm, K_TOP)
        act = kernels.moe_grouped(xp, off, trip["gate_up_proj"], act=1, max_rows=t * K_TOP)
        yp = kernels.moe_grouped(act, off, trip["down_proj"], act=0, max_rows=t * K_TOP)
        ref = kernels.moe_combine(yp, inv, idx, w)
        if t > 1:
            assert torch.equal(ref, rw4_experts_forward(ex, x, idx, w))
        gu, dn = shard_experts(ex, rank, world)
        for fixed in (False, True):
            y = ExpertParallelMoE(E, gu, dn, fixed_capacity=fixed)(x, idx, w)
            torch.cuda.synchronize()
            if not torch.equal(y, ref):
                failures += 1
                print(f"rank {rank} t={t} fixed={fixed}: max diff "
                      f"{(y.float() - ref.float()).abs().max().item()}", flush=True)
    assert kernels.device_status() == 0
    f = torch.tensor([failures], device=dev)
    dist.all_reduce(f)
    dist.destroy_process_group()
    if rank == 0:
        print("EP_OK" if int(f) == 0 else f"EP_FAIL {int(f)}", flush=True)
    sys.exit(0 if int(f) == 0 else 1)


if __name__ == "__main__":
    main()

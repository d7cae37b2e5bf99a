"""Expert-parallel routed experts over NCCL (one process per GPU).

The reference runs every expert on one device (``rocketllm/base.py:1083-1464``); this partitions a
stacked-experts layer's ``E`` experts over ``G`` ranks (rank ``r`` owns experts ``[r E/G,
(r+1) E/G)``) while every rank keeps its own tokens (data parallel).  One MoE layer on every rank:

1. ``permute`` the local (token, slot) pairs by expert id -- rows bound for each rank are then
   contiguous, because each rank owns a contiguous expert range;
2. exchange per-destination row counts (a small all-to-all), then the rows themselves and their
   expert ids (``all_to_all_single`` with those split sizes);
3. on the receiving rank, permute the received rows by local expert, run the grouped RW4 GEMV
   (gate/up with the fused SwiGLU, then down) over the local experts only, and restore the
   received order;
4. send the rows back (the inverse all-to-all) and ``combine`` them into each token in ascending
   expert order -- the same order and rounding as the single-GPU path, so the result is identical.

The kernels are injected (``ops``): the default runs the RW4 CUDA kernels; the CPU tests run the
exchange logic over gloo with a CPU implementation of the same four operations.  Collectives run on
the default process group; every rank takes the same collective steps in the same order.
"""
import torch
import torch.distributed as dist


class CudaExpertOps:
    """The four local operations on the RW4 CUDA kernels."""

    def __init__(self):
        from . import kernels
        self.k = kernels

    def permute(self, idx, num_experts):
        return self.k.moe_permute(idx, num_experts)

    def gather(self, x, perm, k):
        return self.k.moe_gather(x, perm, k)

    def experts(self, x_rows, offsets, gate_up, down, max_rows):
        act = self.k.moe_grouped(x_rows, offsets, gate_up, act=1, max_rows=max_rows)
        return self.k.moe_grouped(act, offsets, down, act=0, max_rows=max_rows)

    def combine(self, y_rows, inv, idx, w):
        return self.k.moe_combine(y_rows, inv, idx, w)


class ExpertParallelMoE:
    """The routed experts of one layer, partitioned over the ranks of ``group``.

    ``gate_up`` / ``down`` are this rank's experts as lists of ``(packed, scale, zero)`` (global
    expert ``first_expert + i`` at index ``i``).
    """

    def __init__(self, num_experts, gate_up, down, group=None, ops=None, fixed_capacity=False):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.num_experts = num_experts
        self.per_rank = num_experts // self.world
        self.first_expert = self.rank * self.per_rank
        if len(gate_up) != self.per_rank or len(down) != self.per_rank:
            raise ValueError("this rank must hold exactly num_experts / world experts")
        self.gate_up = gate_up
        self.down = down
        self.ops = ops if ops is not None else CudaExpertOps()
        # fixed_capacity: every rank sends every peer a buffer of T*k rows (zero-padded, the
        # worst case of one token's k slots) -- equal split sizes, no host round trip, so a step
        # can be captured in a CUDA graph; all ranks must then call with the same token count T
        self.fixed_capacity = fixed_capacity

    def _exchange_counts(self, send_counts):
        recv = torch.empty_like(send_counts)
        dist.all_to_all_single(recv, send_counts, group=self.group)
        return recv

    def forward(self, hidden, top_k_index, top_k_weights):
        if self.fixed_capacity:
            return self._forward_fixed(hidden, top_k_index, top_k_weights)
        t, h = hidden.shape
        k = top_k_index.shape[1]
        idx = top_k_index.to(torch.int64).contiguous()
        ops = self.ops
        # 1. local permutation by global expert id
        perm, inv, offsets = ops.permute(idx, self.num_experts)
        x_sorted = ops.gather(hidden.contiguous(), perm, k)
        ids_sorted = idx.reshape(-1)[perm.long().clamp(min=0)]
        bounds = offsets[::self.per_rank].to(torch.int64)      # [world + 1]
        send_counts = (bounds[1:] - bounds[:-1]).contiguous()
        # 2. counts, then rows and their expert ids
        recv_counts = self._exchange_counts(send_counts)
        send_split = send_counts.cpu().tolist()
        recv_split = recv_counts.cpu().tolist()
        n_recv = int(sum(recv_split))
        x_recv = hidden.new_empty((n_recv, h))
        ids_recv = ids_sorted.new_empty((n_recv,))
        dist.all_to_all_single(x_recv, x_sorted[: sum(send_split)].contiguous(), recv_split,
                               send_split, group=self.group)
        dist.all_to_all_single(ids_recv, ids_sorted[: sum(send_split)].contiguous(), recv_split,
                               send_split, group=self.group)
        # 3. local experts
        if n_recv:
            local_ids = (ids_recv - self.first_expert).reshape(-1, 1).contiguous()
            perm2, inv2, off2 = ops.permute(local_ids, self.per_rank)
            rows = ops.gather(x_recv, perm2, 1)
            y_rows = ops.experts(rows, off2, self.gate_up, self.down, n_recv)
            y_recv = ops.gather(y_rows, inv2, 1)   # back to the received order
        else:
            y_recv = hidden.new_empty((0, h))
        # 4. rows home, then combine in ascending expert order
        y_back = hidden.new_empty((int(sum(send_split)), h))
        dist.all_to_all_single(y_back, y_recv.contiguous(), send_split, recv_split,
                               group=self.group)
        if y_back.shape[0] < t * k:  # slots with out-of-range ids were dropped by permute
            pad = hidden.new_zeros((t * k - y_back.shape[0], h))
            y_back = torch.cat([y_back, pad])
        return ops.combine(y_back, inv, idx, top_k_weights.contiguous())

    def _forward_fixed(self, hidden, top_k_index, top_k_weights):
        """The same exchange with fixed, zero-padded per-peer buffers (device-side only)."""
        t, h = hidden.shape
        k = top_k_index.shape[1]
        cap = max(1, t * k)
        world, dev = self.world, hidden.device
        idx = top_k_index.to(torch.int64).contiguous()
        ops = self.ops
        perm, inv, offsets = ops.permute(idx, self.num_experts)
        x_sorted = ops.gather(hidden.contiguous(), perm, k)
        ids_sorted = idx.reshape(-1)[perm.long().clamp(min=0)] if t else \
            torch.zeros(0, dtype=torch.int64, device=dev)
        bounds = offsets[::self.per_rank].to(torch.int64)                 # [world + 1]
        counts = bounds[1:] - bounds[:-1]
        j = torch.arange(cap, device=dev)
        valid = j[None, :] < counts[:, None]                              # [world, cap]
        src = (bounds[:-1, None] + j[None, :]).clamp(0, max(t * k - 1, 0))
        if t:
            send_x = torch.where(valid[..., None], x_sorted[src], torch.zeros((), dtype=hidden.dtype,
                                                                               device=dev))
            send_ids = torch.where(valid, ids_sorted[src], torch.full((), -1, dtype=torch.int64,
                                                                        device=dev))
        else:
            send_x = torch.zeros((world, cap, h), dtype=hidden.dtype, device=dev)
            send_ids = torch.full((world, cap), -1, dtype=torch.int64, device=dev)
        recv_x = torch.empty_like(send_x)
        recv_ids = torch.empty_like(send_ids)
        dist.all_to_all_single(recv_x.view(world * cap, h), send_x.view(world * cap, h),
                               group=self.group)
        dist.all_to_all_single(recv_ids.view(-1), send_ids.reshape(-1), group=self.group)
        # local experts; padding rows carry id -1 and fall outside [0, per_rank): dropped
        local = torch.where(recv_ids >= 0, recv_ids - self.first_expert,
                            torch.full((), self.per_rank, dtype=torch.int64, device=dev))
        perm2, inv2, off2 = ops.permute(local.reshape(-1, 1).contiguous(), self.per_rank)
        rows = ops.gather(recv_x.view(world * cap, h), perm2, 1)
        y_rows = ops.experts(rows, off2, self.gate_up, self.down, world * cap)
        y_recv = ops.gather(y_rows, inv2, 1)                              # padding rows: zeros
        y_back = torch.empty_like(y_recv)
        dist.all_to_all_single(y_back, y_recv, group=self.group)
        y_back = y_back.view(world, cap, h)
        # back to this rank's expert-sorted order: position p went to rank r at slot p - bounds[r]
        p = torch.arange(t * k, device=dev)
        r = (p[:, None] >= bounds[None, 1:]).sum(1)                       # world = dropped slot
        rc = r.clamp(max=world - 1)
        y_sorted = y_back[rc, (p - bounds[rc]).clamp(0, cap - 1)]
        y_sorted = torch.where((r < world)[:, None], y_sorted,
                               torch.zeros((), dtype=y_sorted.dtype, device=dev))
        return ops.combine(y_sorted, inv, idx, top_k_weights.contiguous())

    __call__ = forward


def shard_experts(experts_module, rank, world):
    """This rank's ``(gate_up, down)`` lists from an RW4 stacked-experts module (views, no copy)."""
    e = experts_module.gate_up_proj_packed.shape[0]
    per = e // world
    sl = range(rank * per, (rank + 1) * per)

    def triples(name):
        p = getattr(experts_module, name + "_packed")
        s = getattr(experts_module, name + "_scale")
        z = getattr(experts_module, name + "_zero_point")
        return [(p[i], s[i], z[i]) for i in sl]

    return triples("gate_up_proj"), triples("down_proj")


def enable_expert_parallel(model, group=None, ops=None, drop_remote=True, fixed_capacity=False):
    """Partition every RW4 stacked-experts module of ``model`` over ``group``: keep this rank's
    experts (views of the stacked tensors; the other experts' memory is released when
    ``drop_remote``) and bind a forward that runs :class:`ExpertParallelMoE`.  Attention and the
    router stay replicated and each rank feeds its own tokens.  Returns the number of layers."""
    import types
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    n = 0
    for module in model.modules():
        if not getattr(module, "rw4", False):
            continue
        e = module.gate_up_proj_packed.shape[0]
        per = e // world
        if drop_remote:
            for name in ("gate_up_proj", "down_proj"):
                for sfx in ("_packed", "_scale", "_zero_point"):
                    full = getattr(module, name + sfx)
                    keep = full[rank * per:(rank + 1) * per].clone()
                    module._parameters[name + sfx] = torch.nn.Parameter(keep,
                                                                        requires_grad=False)
            triples = {name: [(getattr(module, name + "_packed")[i],
                               getattr(module, name + "_scale")[i],
                               getattr(module, name + "_zero_point")[i]) for i in range(per)]
                       for name in ("gate_up_proj", "down_proj")}
            moe = ExpertParallelMoE(e, triples["gate_up_proj"], triples["down_proj"], group, ops,
                                    fixed_capacity)
        else:
            gu, dn = shard_experts(module, rank, world)
            moe = ExpertParallelMoE(e, gu, dn, group, ops, fixed_capacity)
        module.expert_parallel = moe
        module.forward = types.MethodType(
            lambda self, hidden, idx, w: self.expert_parallel(hidden, idx, w), module)
        n += 1
    return n

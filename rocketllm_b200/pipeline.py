"""Pipeline-parallel greedy decode over NCCL (one process per GPU).

The reference runs every layer on one device (``rocketllm/base.py:336``).  For models whose RW4
weights do not fit one GPU (the 405B architecture is ~227 GB), rank ``r`` of ``G`` keeps the
contiguous decoder layers ``[r L/G, (r+1) L/G)``, rank 0 the embedding, the last rank the final
norm and ``lm_head``.  One forward (prefill or one decode step): rank 0 embeds, every rank runs its
layers on the hidden states it received from the previous rank (``dist.recv``) and sends the
result on (``dist.send``; NCCL point-to-point over NVLink), the last rank computes the logits and
the greedy token, and the token is broadcast to every rank for the next step.  Each rank keeps the
KV cache of its own layers.  ``PipelineDecoder`` runs the layers as transformers' modules
(RW4Linear inside); ``GraphedPipelineDecoder`` runs a decode step of resident RW4 Llama layers
through the fused decode ops over the rank's own layer range
(:class:`~rocketllm_b200.fused_decode.FusedLayerRange`), the prefill through the modules.
"""
import torch
import torch.distributed as dist


def layer_range(num_layers, rank, world):
    """Contiguous, balanced ``[start, stop)`` of the layers rank ``rank`` owns."""
    base, extra = divmod(num_layers, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class PipelineDecoder:
    """Greedy decode of a ``*ForCausalLM`` whose decoder layers are split over ``group``.

    ``model`` is this rank's copy; layers outside the rank's range (and the embedding / head on
    ranks that do not use them) are dropped to free their memory.  ``cache`` is the key/value cache
    of this rank's layers (default: transformers' ``DynamicCache``; an
    :class:`~rocketllm_b200.kv_cache.RW4KVCache` keeps them in int4).
    """

    def __init__(self, model, group=None, device="cuda", drop_remote=True, local=False,
                 cache=None):
        from transformers import DynamicCache
        self.group = group
        self.local = local or not dist.is_initialized()   # one rank, no communication
        self.world = 1 if self.local else dist.get_world_size(group)
        self.rank = 0 if self.local else dist.get_rank(group)
        self.device = torch.device(device)
        self.model = model
        inner = model.model
        self.layers = inner.layers
        self.start, self.stop = layer_range(len(self.layers), self.rank, self.world)
        self.first = self.rank == 0
        self.last = self.rank == self.world - 1
        if drop_remote:
            for i in range(len(self.layers)):
                if not self.start <= i < self.stop:
                    self.layers[i] = torch.nn.Identity()
            if not self.first:
                inner.embed_tokens = None
            if not self.last:
                model.lm_head = None
                inner.norm = None
        self.rotary = inner.rotary_emb
        self.embed = inner.embed_tokens
        self.cache = cache if cache is not None else DynamicCache(config=model.config)
        self.hidden_size = model.config.hidden_size
        self.dtype = next(p.dtype for p in model.parameters() if p.is_floating_point()
                          and p.dtype != torch.float16)
        self.seen = 0

    def _peer(self, delta):
        ranks = dist.get_process_group_ranks(self.group) if self.group is not None else None
        r = self.rank + delta
        return ranks[r] if ranks is not None else r

    @torch.no_grad()
    def _forward(self, ids, b, t):
        """One pipeline pass over ``t`` new positions; returns the greedy token [b, 1] (all ranks)."""
        pos = torch.arange(self.seen, self.seen + t, device=self.device)
        if self.first:
            h = self.embed(ids.to(self.device))
        else:
            h = torch.empty((b, t, self.hidden_size), dtype=self.dtype, device=self.device)
            # (the first rank's embedding output has this dtype; `dtype` follows the model)
            dist.recv(h, src=self._peer(-1), group=self.group)
        position_ids = pos.unsqueeze(0).expand(b, -1)
        cos_sin = self.rotary(h, position_ids)
        for i in range(self.start, self.stop):
            h = self.layers[i](h, attention_mask=None, position_ids=position_ids,
                               past_key_values=self.cache, use_cache=True, cache_position=pos,
                               position_embeddings=cos_sin)
            if isinstance(h, tuple):
                h = h[0]
        tok = torch.empty((b, 1), dtype=torch.long, device=self.device)
        if not self.last:
            dist.send(h.contiguous(), dst=self._peer(1), group=self.group)
        else:
            logits = self.model.lm_head(self.model.model.norm(h[:, -1:, :]))
            tok.copy_(logits[:, -1].argmax(-1, keepdim=True))
        if not self.local:
            last = dist.get_process_group_ranks(self.group)[-1] if self.group is not None else \
                self.world - 1
            dist.broadcast(tok, src=last, group=self.group)
        self.seen += t
        return tok

    def generate(self, input_ids, new_tokens):
        """Greedy tokens ``[B, new_tokens]``; every rank returns them."""
        b, t = input_ids.shape
        toks = [self._forward(input_ids, b, t)]
        for _ in range(new_tokens - 1):
            toks.append(self._forward(toks[-1], b, 1))
        return torch.cat(toks, dim=1)


class GraphedPipelineDecoder(PipelineDecoder):
    """:class:`PipelineDecoder` with a static KV cache and each rank's per-token stage captured in a
    CUDA graph: the hand-off (``recv`` before, ``send`` after) and the token broadcast stay outside
    the graph, everything a stage computes (embedding on the first rank, its decoder layers, the
    norm / lm_head / argmax on the last) replays from it.  ``batch`` sequences, at most
    ``max_len`` positions.

    The prefill runs the prompt through an empty cache with causal attention (no mask: queries
    never reach the unwritten cache slots); decode steps attend over the whole static cache under a
    mask of the positions written so far.  ``fused`` (default: where it applies, i.e. resident RW4
    Llama layers on a CUDA device) runs each decode step through the fused decode ops over this
    rank's layers instead of the modules; ``fused=True`` where it does not apply raises
    ``ValueError``."""

    def __init__(self, model, batch, max_len, group=None, device="cuda", drop_remote=True,
                 local=False, use_graph=True, fused=None):
        super().__init__(model, group, device, drop_remote, local)
        from transformers import StaticCache

        from .fused_decode import FusedLayerRange, fusable_layers
        self.cache = StaticCache(config=model.config, max_cache_len=max_len)
        # The stage's decode step: the fused decode ops over its layers (resident RW4 Llama
        # layers; default where they apply) or the transformers modules.
        own = range(self.start, self.stop)
        can_fuse = self.device.type == "cuda" and fusable_layers(model, own, self.last)
        if fused is None:
            fused = can_fuse
        elif fused and not can_fuse:
            raise ValueError("the fused stage covers resident RW4 Llama layers on a CUDA device")
        self.fl = (FusedLayerRange(model, batch, own, max_len, self.last, device=self.device)
                   if fused else None)
        self._counters = None
        self.batch, self.max_len = batch, max_len
        h = self.hidden_size
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.h_in = torch.zeros(batch, 1, h, dtype=self.dtype, device=self.device)
        self.h_out = torch.zeros(batch, 1, h, dtype=self.dtype, device=self.device)
        self.key_pos = torch.arange(max_len, device=self.device)
        self.use_graph = use_graph
        self.graph = None
        self.host_pos = 0

    def _run_layers(self, h, pos, masked):
        b = h.shape[0]
        position_ids = pos.unsqueeze(0).expand(b, -1)
        cos_sin = self.rotary(h, position_ids)
        mask = None
        if masked:   # [b, 1, q, max_len]: key j visible to the query at position p iff j <= p
            mask = (self.key_pos[None, :] <= pos[:, None])[None, None].expand(b, 1, -1, -1)
        for i in range(self.start, self.stop):
            h = self.layers[i](h, attention_mask=mask, position_ids=position_ids,
                               past_key_values=self.cache, use_cache=True, cache_position=pos,
                               position_embeddings=cos_sin)
            if isinstance(h, tuple):
                h = h[0]
        return h

    def _last_rank(self):
        if self.local:
            return 0
        return dist.get_process_group_ranks(self.group)[-1] if self.group is not None else \
            self.world - 1

    @torch.no_grad()
    def prefill(self, input_ids):
        b, t = input_ids.shape
        if b != self.batch or t + 1 > self.max_len:
            raise ValueError(f"prompt [{b}, {t}] does not fit batch {self.batch} / "
                             f"{self.max_len} positions")
        pos = torch.arange(t, device=self.device)
        if self.first:
            h = self.embed(input_ids.to(self.device))
        else:
            h = torch.empty((b, t, self.hidden_size), dtype=self.dtype, device=self.device)
            dist.recv(h, src=self._peer(-1), group=self.group)
        h = self._run_layers(h, pos, masked=False)
        if not self.last:
            dist.send(h.contiguous(), dst=self._peer(1), group=self.group)
        else:
            logits = self.model.lm_head(self.model.model.norm(h[:, -1:, :]))
            self.ids.copy_(logits[:, -1].argmax(-1, keepdim=True))
        if not self.local:
            dist.broadcast(self.ids, src=self._last_rank(), group=self.group)
        self.pos.fill_(t)
        self.host_pos = t
        # the static cache's write counters of this stage's layers, advanced by the fused step
        counters = (getattr(self.cache.layers[i], "cumulative_length", None)
                    for i in range(self.start, self.stop))
        self._counters = [c for c in counters if torch.is_tensor(c)]
        return self.ids.clone()

    def _fused_stage(self):
        """The stage's decode step through the fused ops (``FusedLayerRange``): embedding on the
        first rank, the rank's layers, then the final norm + lm_head and the greedy choice on the
        last rank -- the launches :class:`~rocketllm_b200.fused_decode.FusedDecoder` makes for
        the same layers."""
        fl, b = self.fl, self.batch
        stream = torch.cuda.current_stream(self.device).cuda_stream
        h = self.embed(self.ids) if self.first else self.h_in
        cur = fl.h[0]
        cur.copy_(h.view(b, self.hidden_size))
        cos, sin = fl._rotary(self.rotary, cur, self.pos)
        cur = fl.run(cur, self.pos, cos, sin, fl._step_mask(self.pos), self.cache, stream)
        if self._counters:
            torch._foreach_add_(self._counters, 1)
        if self.last:
            from . import kernels
            kernels.argmax_rows(fl.head_logits(cur), out=self.ids)
        else:
            self.h_out.view(b, self.hidden_size).copy_(cur)
        self.pos.add_(1)

    def _stage(self):
        if self.fl is not None:
            return self._fused_stage()
        h = self.embed(self.ids) if self.first else self.h_in
        h = self._run_layers(h, self.pos, masked=True)
        if self.last:
            logits = self.model.lm_head(self.model.model.norm(h))
            self.ids.copy_(logits[:, -1].argmax(-1, keepdim=True))
        else:
            self.h_out.copy_(h)
        self.pos.add_(1)

    def _state(self):
        state = [self.ids, self.pos]
        for layer in getattr(self.cache, "layers", []):
            c = getattr(layer, "cumulative_length", None)
            if torch.is_tensor(c) and c.is_cuda:
                state.append(c)
        return state

    @torch.no_grad()
    def capture(self):
        """Warm up on a side stream and capture the stage (no communication inside); the state a
        step advances is restored afterwards, so the first replay starts where the prefill
        ended."""
        state = self._state()
        saved = [t.clone() for t in state]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._stage()
            for t, v in zip(state, saved):
                t.copy_(v)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._stage()
        for t, v in zip(state, saved):
            t.copy_(v)
        torch.cuda.synchronize(self.device)

    @torch.no_grad()
    def step(self):
        """One greedy token for every sequence; returns ``ids`` [batch, 1] (all ranks)."""
        if self.host_pos + 1 > self.max_len:
            raise ValueError(f"static KV cache full ({self.max_len} positions)")
        if self.use_graph and self.graph is None:
            self.capture()
        if not self.first:
            dist.recv(self.h_in, src=self._peer(-1), group=self.group)
        if self.use_graph:
            self.graph.replay()
        else:
            self._stage()
        if not self.last:
            dist.send(self.h_out, dst=self._peer(1), group=self.group)
        if not self.local:
            dist.broadcast(self.ids, src=self._last_rank(), group=self.group)
        self.host_pos += 1
        return self.ids

    @torch.no_grad()
    def generate(self, input_ids, new_tokens):
        toks = [self.prefill(input_ids)]
        for _ in range(new_tokens - 1):
            toks.append(self.step().clone())
        return torch.cat(toks, dim=1)

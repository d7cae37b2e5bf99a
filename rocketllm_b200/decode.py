"""CUDA-graph greedy decode for RW4 models (the B200 replacement for a tracing compiler).

A decode step of a transformers model issues a few hundred small launches from Python; at batch 1
on B200 the RW4 GEMVs of a whole 8B-parameter model take well under a millisecond, so the host
would be the bottleneck.  ``GraphedDecoder`` runs the step once eagerly (to allocate the static KV
cache and set every kernel's launch attributes), captures it in a CUDA graph with the token and
position living in device tensors, and then replays the graph once per token: the argmax, the next
token's feedback and the position increment are inside the graph, so a replay needs no host sync.
The RW4 kernels launch on the capturing stream through the C ABI, so they are captured like any
other kernel; their TMA descriptors are kernel parameters fixed at capture (the weights do not
move).
"""
import torch


class GraphedDecoder:
    """Greedy decode of ``model`` (an RW4 ``*ForCausalLM`` on one GPU) with a static KV cache."""

    def __init__(self, model, batch, max_len, device="cuda", use_graph=True):
        from transformers import StaticCache
        self.model = model
        self.device = torch.device(device)
        self.batch = batch
        self.max_len = max_len
        self.cache = StaticCache(config=model.config, max_cache_len=max_len)
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.use_graph = use_graph
        self.graph = None
        self.out = None
        self.host_pos = 0   # host copy of the next write position (bounds check before launch)

    @torch.no_grad()
    def prefill(self, input_ids):
        t = input_ids.shape[1]
        if t + 1 > self.max_len:
            raise ValueError("prompt longer than the static cache")
        self.host_pos = t
        pos = torch.arange(t, device=self.device)
        logits = self.model(input_ids.to(self.device), past_key_values=self.cache,
                            cache_position=pos, use_cache=True).logits[:, -1]
        nxt = logits.argmax(-1, keepdim=True)
        self.ids.copy_(nxt)
        self.pos.fill_(t)
        return nxt

    @torch.no_grad()
    def _step(self):
        logits = self.model(self.ids, past_key_values=self.cache, cache_position=self.pos,
                            use_cache=True).logits[:, -1]
        self.logits = logits   # the step's scores (a static tensor once captured)
        nxt = logits.argmax(-1, keepdim=True)
        self.ids.copy_(nxt)
        self.pos.add_(1)
        return nxt

    @torch.no_grad()
    def capture(self):
        """Warm up on a side stream, then capture one step.  Call after ``prefill``; the warm-up
        step's cache writes land at the current position and are overwritten by the first
        replay, since the position is restored."""
        if self.host_pos + 1 > self.max_len:
            raise ValueError(f"static KV cache full ({self.max_len} positions)")
        state = self._state()
        saved = [t.clone() for t in state]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._step()
            for t, v in zip(state, saved):
                t.copy_(v)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._step()
        # capture does not execute: restore the state the first replay starts from
        for t, v in zip(state, saved):
            t.copy_(v)
        torch.cuda.synchronize(self.device)

    def _state(self):
        """Device tensors a step advances: the token, the position and the static cache's own
        write counters (transformers' StaticLayer writes at ``cumulative_length``)."""
        state = [self.ids, self.pos]
        for layer in getattr(self.cache, "layers", []):
            c = getattr(layer, "cumulative_length", None)
            if torch.is_tensor(c):
                state.append(c)
        return state

    @torch.no_grad()
    def step(self):
        if self.host_pos + 1 > self.max_len:
            raise ValueError(f"static KV cache full ({self.max_len} positions)")
        self.host_pos += 1
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
            return self.out
        return self._step()

    @torch.no_grad()
    def generate(self, input_ids, new_tokens):
        """Greedy tokens ``[B, new_tokens]`` (the first comes from the prefill)."""
        toks = [self.prefill(input_ids).clone()]
        for _ in range(new_tokens - 1):
            toks.append(self.step().clone())
        return torch.cat(toks, dim=1)

"""Fused decode step for resident RW4 Llama- and Mixtral-architecture models (the decode-step op
stream around the RW4 GEMVs, B200-first).

Through the transformers modules one decode step of a Llama layer is about fifty small launches:
RMSNorm as six elementwise kernels, q / k / v as three GEMVs, the rotary embedding as cat / neg /
mul / add kernels, ``index_copy_`` into the static cache, the grouped-query key / value copies
(``repeat_kv``), attention, o_proj, the residual add, RMSNorm again, gate, up, SiLU, the product,
down, the residual add (transformers ``models/llama/modeling_llama.py``).  The step here is about
six launches per layer at batch 1 (attention included; from two rows on each GEMV adds its
activation-conversion pass), each reproducing the modules' bf16 rounding sequence:

    rw4_linear_rmsnorm_ws             input_layernorm, then q_proj, k_proj, v_proj as one GEMV
                                      over the concatenated weight (the norm runs inside the
                                      GEMV's activation conversion)
    rw4_rope_kv                       apply_rotary_pos_emb + StaticCache.update (device position)
    rw4_decode_attention              attention over the static cache up to the device-side
                                      position, grouped-query heads, no key / value copies (SDPA
                                      with enable_gqa and a mask for shapes it does not cover)
    rw4_linear_residual_ws            o_proj + residual add in the GEMV epilogue
    rw4_linear_rmsnorm_swiglu_ws      post_attention_layernorm, then gate_proj, up_proj as one
                                      GEMV over the concatenated weight, act_fn(gate) * up in
                                      its epilogue
    rw4_linear_residual_ws            down_proj + residual add

The q/k/v and gate/up weights are concatenated once at set-up and the original modules'
parameters become views of the concatenated tensors, so nothing is duplicated and the
transformers forward (prefill, or any other use) runs on the same bytes.  The prefill itself
runs through the modules; only decode steps take the fused path, captured in a CUDA graph by
:class:`~rocketllm_b200.decode.GraphedDecoder`'s machinery.

Mixtral-architecture models (transformers ``models/mixtral/modeling_mixtral.py``: the same
attention and norms, a sparse-MoE block in place of the MLP) take the same attention half; the
MoE half is the model's own block -- its top-k router, then its routed-experts module, which is
the RW4 grouped path (``rw4_experts_forward``) or, after ``enable_expert_parallel``, the
expert-parallel exchange -- followed by the residual add:

    rw4_rmsnorm                       post_attention_layernorm
    mlp (router + routed experts)     MixtralSparseMoeBlock, unchanged
    residual add                      ``residual + hidden_states``
"""
import ctypes
import os

import torch

from . import _lib, kernels
from .decode import GraphedDecoder
from .quant.modules import RW4Linear


def _rw4(mods):
    return all(isinstance(x, RW4Linear) and x.bias is None for x in mods)


def fusable(model):
    """Whether ``model`` is a resident RW4 ``*ForCausalLM`` the fused step covers: a Llama
    architecture whose projections are all ``RW4Linear`` without bias, or a Mixtral architecture
    whose attention projections are and whose routed experts are RW4 (or expert-parallel over
    them); no sliding window, no streaming hooks, all on one CUDA device."""
    cfg = model.config
    kind = getattr(cfg, "model_type", None)
    if kind not in ("llama", "mixtral") or getattr(cfg, "sliding_window", None):
        return False
    inner = getattr(model, "model", None)
    if inner is None or not isinstance(getattr(model, "lm_head", None), RW4Linear):
        return False
    for layer in inner.layers:
        a, m = layer.self_attn, layer.mlp
        if not _rw4((a.q_proj, a.k_proj, a.v_proj, a.o_proj)):
            return False
        if layer._forward_pre_hooks or layer._forward_hooks:
            return False
        if kind == "llama":
            if not _rw4((m.gate_proj, m.up_proj, m.down_proj)):
                return False
            if getattr(m, "act_fn", None) is None or cfg.hidden_act not in ("silu", "swish"):
                return False
        else:
            experts = getattr(m, "experts", None)
            if getattr(m, "gate", None) is None or not getattr(experts, "rw4", False):
                return False
            if m._forward_pre_hooks or m._forward_hooks or experts._forward_pre_hooks:
                return False
    return all(p.is_cuda for p in model.parameters())


def _concat_rows(mods):
    """One RW4 weight whose rows are the given modules' rows in order; each module's parameters
    become views of it (the originals are released).  Done once: a later call finds the modules
    already views of the same tensors and returns those."""
    done = getattr(mods[0], "_rw4_rows_fused", None)
    if done is not None and done[1] == tuple(id(m) for m in mods) and all(
            getattr(m, leaf).data_ptr() == base.data_ptr() + off * base.stride(0) *
            base.element_size()
            for leaf, base in zip(("weight_packed", "weight_scale", "weight_zero_point"), done[0])
            for m, off in zip(mods, done[2])):
        return done[0]
    parts = {}
    for leaf in ("weight_packed", "weight_scale", "weight_zero_point"):
        tensors = [getattr(m, leaf) for m in mods]
        fused = torch.cat([t.detach() for t in tensors], dim=0).contiguous()
        parts[leaf] = fused
        off = 0
        offsets = []
        for m, t in zip(mods, tensors):
            n = t.shape[0]
            m._parameters[leaf] = torch.nn.Parameter(fused[off:off + n], requires_grad=False)
            offsets.append(off)
            off += n
    out = (parts["weight_packed"], parts["weight_scale"], parts["weight_zero_point"])
    mods[0]._rw4_rows_fused = (out, tuple(id(m) for m in mods), tuple(offsets))
    return out


class _LayerWeights:
    __slots__ = ("ln1", "ln2", "qkv", "o", "gate_up", "down", "eps1", "eps2", "moe")


class _FusedOps:
    """The fused per-layer decode ops over a list of decoder layers of a resident RW4 Llama or
    Mixtral model: their weights (q|k|v and gate|up concatenated), the step's static buffers and
    workspace, and the layer loop.  :class:`FusedDecoder` runs it over every layer; a pipeline
    stage (:class:`~rocketllm_b200.pipeline.GraphedPipelineDecoder`) over the layers it owns.
    The user sets ``device`` and ``batch`` before calling ``_setup``."""

    def _setup(self, model, batch, layer_ids, max_len, with_head, attention):
        cfg = model.config
        self.hq = cfg.num_attention_heads
        self.hk = cfg.num_key_value_heads
        self.hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.hq
        self.hidden = cfg.hidden_size
        self.inter = cfg.intermediate_size
        moe = cfg.model_type == "mixtral"
        self.layer_ids = list(layer_ids)
        self.layers = []
        for i in self.layer_ids:
            layer = model.model.layers[i]
            a, m = layer.self_attn, layer.mlp
            w = _LayerWeights()
            w.ln1, w.eps1 = layer.input_layernorm.weight, layer.input_layernorm.variance_epsilon
            w.ln2 = layer.post_attention_layernorm.weight
            w.eps2 = layer.post_attention_layernorm.variance_epsilon
            w.qkv = _concat_rows([a.q_proj, a.k_proj, a.v_proj])
            w.o = (a.o_proj.weight_packed, a.o_proj.weight_scale, a.o_proj.weight_zero_point)
            w.moe = m if moe else None
            if not moe:
                w.gate_up = _concat_rows([m.gate_proj, m.up_proj])
                w.down = (m.down_proj.weight_packed, m.down_proj.weight_scale,
                          m.down_proj.weight_zero_point)
            self.layers.append(w)
        self.head = None
        if with_head:
            norm = model.model.norm
            self.final_norm, self.final_eps = norm.weight, norm.variance_epsilon
            head = model.lm_head
            self.head = (head.weight_packed, head.weight_scale, head.weight_zero_point)
        dev, b = self.device, batch
        bf = dict(dtype=torch.bfloat16, device=dev)
        nqkv = (self.hq + 2 * self.hk) * self.hd
        # static buffers of the step (a captured graph reads and writes these addresses)
        self.h = [torch.empty(b, self.hidden, **bf) for _ in range(2)]
        self.xn = torch.empty(b, self.hidden, **bf)
        self.qkv_out = torch.empty(b, nqkv, **bf)
        self.q_rot = torch.empty(b, self.hq, 1, self.hd, **bf)
        # attention: rw4_decode_attention (device-side length, programmatic launch) where it
        # covers the shape, else SDPA over the whole static cache with a mask.  A Mixtral keeps
        # SDPA, the module path's own kernel: its top-k routing is discontinuous, and attention
        # that differs within bf16 rounding flips near-tied expert choices, so the fused step
        # keeps the modules' attention bits there.
        if attention is None:   # RW4_FUSED_ATTENTION=sdpa selects SDPA (for measurements)
            attention = os.environ.get("RW4_FUSED_ATTENTION", "rw4")
        if attention not in ("rw4", "sdpa"):
            raise ValueError(f"attention must be 'rw4' or 'sdpa', not {attention!r}")
        self.own_attention = (attention == "rw4" and not moe and self.hq % self.hk == 0
                              and self.hq // self.hk <= 8 and self.hd in (64, 128))
        self.attn_out = torch.empty(b, self.hq, 1, self.hd, **bf)
        shapes = [(self.hidden, nqkv), (self.hq * self.hd, self.hidden)]
        if with_head:
            shapes.append((self.hidden, self.head[0].shape[0]))
        if not moe:
            self.act = torch.empty(b, self.inter, **bf)
            shapes += [(self.hidden, 2 * self.inter), (self.inter, self.hidden)]
        self.positions = torch.arange(max_len, device=dev)
        self.logits_buf = torch.empty(b, self.head[0].shape[0], **bf) if with_head else None
        self._counters = None
        wsb = max(kernels.linear_workspace_bytes(b, k, n) for k, n in shapes)
        for k, n in shapes:   # the projections that follow a norm take it in their conversion
            nb = ctypes.c_size_t(0)
            _lib.call("rw4_linear_rmsnorm_workspace_size", b, k, n, ctypes.byref(nb))
            wsb = max(wsb, nb.value)
            if not moe and n == 2 * self.inter:   # gate|up with the SwiGLU epilogue
                _lib.call("rw4_linear_rmsnorm_swiglu_workspace_size", b, k, n, ctypes.byref(nb))
                wsb = max(wsb, nb.value)
        self.ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)

    def _lin(self, x, w, out, residual=None):
        m, k = x.shape
        n = w[0].shape[0]
        ws, wsb = self.ws.data_ptr(), self.ws.numel()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if residual is None:
            _lib.call("rw4_linear_ws", x.data_ptr(), m, k, w[0].data_ptr(), w[1].data_ptr(),
                      w[2].data_ptr(), n, 64, out.data_ptr(), 0, ws, wsb, stream)
        else:
            _lib.call("rw4_linear_residual_ws", x.data_ptr(), m, k, w[0].data_ptr(),
                      w[1].data_ptr(), w[2].data_ptr(), n, 64, residual.data_ptr(),
                      out.data_ptr(), ws, wsb, stream)
        return out

    def _lin_norm(self, x, weight, eps, w, out, swiglu=False):
        """``out = rmsnorm(x) . W^T``: the norm runs inside the projection's activation
        conversion (the one-row GEMV's prologue, or the x-prep pass of a batch): one launch.
        ``swiglu``: W is [gate; up] and ``out = act_fn(gate) * up``, in the same launch."""
        m, k = x.shape
        fn = "rw4_linear_rmsnorm_swiglu_ws" if swiglu else "rw4_linear_rmsnorm_ws"
        _lib.call(fn, x.data_ptr(), m, k, weight.data_ptr(), float(eps),
                  w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(), w[0].shape[0], 64,
                  out.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                  torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def _norm(self, x, weight, eps, out):
        _lib.call("rw4_rmsnorm", x.data_ptr(), weight.data_ptr(), x.shape[0], x.shape[1],
                  float(eps), out.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def _run_layers(self, cur, pos, cos, sin, mask, cache, stream):
        """The fused ops of every layer in ``layer_ids`` on the residual stream ``cur`` (one of
        ``self.h``; the other is the step's second buffer), the layers' keys and values in
        ``cache.layers[i]``; returns the buffer holding the result."""
        b = self.batch
        nq, nk = self.hq * self.hd, self.hk * self.hd
        qkv = self.qkv_out
        other = self.h[1] if cur is self.h[0] else self.h[0]
        for i, w in zip(self.layer_ids, self.layers):
            layer = cache.layers[i]
            self._lin_norm(cur, w.ln1, w.eps1, w.qkv, qkv)
            _lib.call("rw4_rope_kv", qkv.data_ptr(), qkv[:, nq:].data_ptr(),
                      qkv[:, nq + nk:].data_ptr(), qkv.shape[1], b, self.hq, self.hk, self.hd,
                      cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), layer.keys.shape[2],
                      self.q_rot.data_ptr(), layer.keys.data_ptr(), layer.values.data_ptr(),
                      stream)
            if self.own_attention:
                attn = self.attn_out
                _lib.call("rw4_decode_attention", self.q_rot.data_ptr(), b, self.hq, self.hk,
                          self.hd, layer.keys.data_ptr(), layer.values.data_ptr(),
                          layer.keys.shape[2], pos.data_ptr(), self.hd ** -0.5,
                          attn.data_ptr(), stream)
            else:
                attn = torch.nn.functional.scaled_dot_product_attention(
                    self.q_rot, layer.keys, layer.values, attn_mask=mask,
                    scale=self.hd ** -0.5, enable_gqa=True)
            # residual stream: each add writes the other buffer (no in-place update)
            self._lin(attn.reshape(b, nq), w.o, other, residual=cur)
            cur, other = other, cur
            if w.moe is not None:
                # the model's own sparse-MoE block (router + routed experts), then the residual
                xn = self._norm(cur, w.ln2, w.eps2, self.xn)
                y = w.moe(xn.view(b, 1, self.hidden)).view(b, self.hidden)
                torch.add(cur, y, out=other)
            else:
                self._lin_norm(cur, w.ln2, w.eps2, w.gate_up, self.act, swiglu=True)
                self._lin(self.act, w.down, other, residual=cur)
            cur, other = other, cur
        return cur

    def _rotary(self, rotary_emb, h, pos):
        """bf16 cos / sin [batch, head_dim] of the step's position (the model's rotary module)."""
        b = self.batch
        cos, sin = rotary_emb(h.view(b, 1, self.hidden), pos.view(1, 1).expand(b, 1))
        return (cos.reshape(b, self.hd).to(torch.bfloat16).contiguous(),
                sin.reshape(b, self.hd).to(torch.bfloat16).contiguous())

    def _step_mask(self, pos):
        """The additive mask SDPA needs (0 up to the position, -inf after), or None."""
        if self.own_attention:
            return None
        mask = torch.where(self.positions <= pos, 0.0, float("-inf")).to(torch.bfloat16)
        return mask.view(1, 1, 1, -1)


class FusedDecoder(_FusedOps, GraphedDecoder):
    """Greedy decode of a resident RW4 Llama or Mixtral model with the fused step (see the module
    docstring); same interface as :class:`~rocketllm_b200.decode.GraphedDecoder` (``prefill``,
    ``step``, ``generate``, ``capture``).  Raises ``ValueError`` for a model :func:`fusable`
    rejects.  ``attention``: ``"rw4"`` (default: ``rw4_decode_attention`` where it covers the
    shape) or ``"sdpa"`` (torch's SDPA over the static cache with a mask)."""

    def __init__(self, model, batch, max_len, device="cuda", use_graph=True, attention=None):
        if not fusable(model):
            raise ValueError("the fused decode step covers resident RW4 Llama- and "
                             "Mixtral-architecture models")
        GraphedDecoder.__init__(self, model, batch, max_len, device=device, use_graph=use_graph)
        self._setup(model, batch, range(len(model.model.layers)), max_len, True, attention)

    @torch.no_grad()
    def prefill(self, input_ids):
        nxt = super().prefill(input_ids)
        self._counters = [layer.cumulative_length for layer in self.cache.layers]
        return nxt

    @torch.no_grad()
    def _step(self):
        model, b = self.model, self.batch
        stream = torch.cuda.current_stream(self.device).cuda_stream
        inner = model.model
        h = inner.embed_tokens(self.ids).view(b, self.hidden)
        if h.dtype != torch.bfloat16:
            h = h.to(torch.bfloat16)
        cur = self.h[0]
        cur.copy_(h)
        pos = self.pos
        cos, sin = self._rotary(inner.rotary_emb, cur, pos)
        mask = self._step_mask(pos)
        cur = self._run_layers(cur, pos, cos, sin, mask, self.cache, stream)
        # the static cache's own write counters, kept in step for transformers (one launch)
        torch._foreach_add_(self._counters, 1)
        logits = self._lin_norm(cur, self.final_norm, self.final_eps, self.head, self.logits_buf)
        self.logits = logits
        # the greedy choice straight into the next step's token (logits.argmax's bits)
        kernels.argmax_rows(logits, out=self.ids)
        self.pos.add_(1)
        return self.ids


class FusedLayerRange(_FusedOps):
    """The fused decode ops of the decoder layers ``layer_ids`` of a resident RW4 Llama model (the
    layers a pipeline stage owns): ``run(cur, pos, cos, sin, mask, cache, stream)`` on one token
    per sequence, ``head(cur)`` for the stage that holds the final norm and ``lm_head``."""

    def __init__(self, model, batch, layer_ids, max_len, with_head, device="cuda",
                 attention=None):
        self.device = torch.device(device)
        self.batch = batch
        self._setup(model, batch, layer_ids, max_len, with_head, attention)

    def run(self, cur, pos, cos, sin, mask, cache, stream):
        return self._run_layers(cur, pos, cos, sin, mask, cache, stream)

    def head_logits(self, cur):
        return self._lin_norm(cur, self.final_norm, self.final_eps, self.head, self.logits_buf)


def fusable_layers(model, layer_ids, with_head):
    """Whether :class:`FusedLayerRange` covers these layers of ``model``: a Llama architecture,
    the layers' projections (and ``lm_head`` when ``with_head``) ``RW4Linear`` without bias, no
    hooks, SiLU, all on a CUDA device."""
    cfg = model.config
    if getattr(cfg, "model_type", None) != "llama" or getattr(cfg, "sliding_window", None):
        return False
    if cfg.hidden_act not in ("silu", "swish"):
        return False
    inner = getattr(model, "model", None)
    if inner is None:
        return False
    if with_head and (not isinstance(getattr(model, "lm_head", None), RW4Linear)
                      or getattr(inner, "norm", None) is None):
        return False
    for i in layer_ids:
        layer = inner.layers[i]
        a, m = getattr(layer, "self_attn", None), getattr(layer, "mlp", None)
        if a is None or m is None:
            return False
        if not _rw4((a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj,
                     m.down_proj)):
            return False
        if layer._forward_pre_hooks or layer._forward_hooks:
            return False
        if not all(p.is_cuda for p in layer.parameters()):
            return False
    return True

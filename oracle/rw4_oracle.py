"""CPU oracle for the RW4 4-bit hot path.  TEST INFRASTRUCTURE ONLY.

This module checks the product and is never part of it.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The shipped package
(``rocketllm_b200``) never imports anything under ``oracle/`` and raises when its CUDA library is
missing instead of falling back here.

It restates, in numpy, the reference algorithm of RocketLLM's int4 codec and of the ops the hot
path runs over its output.  Every function cites the reference lines it follows (paths are relative
to the RocketLLM project root):

* ``rocketllm/quant/kv_cache.py:160-187``  ``_pad_to_group``  (ragged tail repeats the last value)
* ``rocketllm/quant/kv_cache.py:190-221``  ``quantize``       (asymmetric int4, group along an axis)
* ``rocketllm/quant/kv_cache.py:249-257``  ``QuantizedTensor.dequantize``
* ``rocketllm/quant/kv_cache.py:260-272``  ``_pack`` / ``_unpack`` (even index = low nibble)
* transformers ``models/mixtral/modeling_mixtral.py:101-116`` ``MixtralTopKRouter`` (softmax fp32,
  top-k, renormalise) and ``:62-98`` ``MixtralExperts.forward`` (gate/up, SiLU, down, weighted sum)
* ``rocketllm/moe/router.py:70-94`` ``RouterSelection.observe`` (sorted unique expert ids)
* ``rocketllm/quant/kv_cache.py:277-352`` ``QuantizedKVCache.update`` / ``_flush`` (window of exact
  tokens, whole groups moved into quantized blocks) and the attention a decode step runs over the
  expanded history (transformers ``integrations/sdpa_attention.py``)

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against fixtures in
``tests/golden/`` that ``tests/golden/make_golden.py`` produced by running the reference's own
``kv_cache`` codec and transformers' own Mixtral router on the same seeded inputs, and
``tests/test_kv_oracle.py`` checks the KV-cache functions against ``tests/golden/reference_kv.npz``,
which ``tests/golden/make_kv_golden.py`` produced by running the reference's ``QuantizedKVCache``
and transformers' SDPA attention.

bf16 has no numpy dtype, so bf16 tensors travel as their raw ``uint16`` bit patterns; conversion
to and from fp32 uses round-to-nearest-even on the bit pattern, the rounding torch's ``.to()``
applies.
"""
import numpy as np

LEVELS = 15          # int4 -> sixteen levels (kv_cache.py:140)
BITS = 4             # two codes per byte (kv_cache.py:141)


# ----------------------------------------------------------------------------------------------
# bf16 helpers (bit patterns in uint16)
# ----------------------------------------------------------------------------------------------

def f32_to_bf16_bits(a):
    """fp32 -> bf16 bit pattern, round to nearest even (NaN kept quiet)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)
    return rounded


def bf16_bits_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a):
    """Round an fp32 array to bf16 precision and return it as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# ----------------------------------------------------------------------------------------------
# the codec
# ----------------------------------------------------------------------------------------------

def pack(codes):
    """Two 4-bit codes per byte along the last axis: ``low | high << 4``.

    Follows ``kv_cache.py:260-265``: an odd length is padded with one zero code; element ``2i``
    lands in the low nibble of byte ``i`` and ``2i+1`` in the high nibble.
    """
    codes = np.asarray(codes, dtype=np.uint8)
    if codes.shape[-1] % 2:
        codes = np.concatenate([codes, np.zeros(codes.shape[:-1] + (1,), np.uint8)], axis=-1)
    low = codes[..., 0::2]
    high = codes[..., 1::2]
    return (low | (high << BITS)).astype(np.uint8)


def unpack(packed):
    """Inverse of :func:`pack` (``kv_cache.py:268-272``)."""
    packed = np.asarray(packed, dtype=np.uint8)
    low = packed & LEVELS
    high = (packed >> BITS) & LEVELS
    return np.stack([low, high], axis=-1).reshape(packed.shape[:-1] + (packed.shape[-1] * 2,))


def _pad_rows_to_group(w, group):
    """Ragged last group padded by repeating the last column (``kv_cache.py:160-187``)."""
    k = w.shape[-1]
    rem = (-k) % group
    if not rem:
        return w, 0
    tail = np.repeat(w[..., -1:], rem, axis=-1)
    return np.concatenate([w, tail], axis=-1), rem


def quantize(w, group=64, dtype="f32"):
    """Quantize a 2-D weight ``[N, K]`` along its last axis, as the reference ``quantize(W, 1, g)``.

    ``dtype`` is the dtype the reference tensor has: ``"f32"`` (``w`` is float32), ``"bf16"``
    (``w`` is the uint16 bit pattern of a bf16 tensor) or ``"f16"`` (``w`` is float16).  It
    matters because the reference computes ``(hi - lo) / 15`` in the tensor's own dtype
    (``kv_cache.py:208``), each op rounded to that dtype, and only then widens to fp32 for the code
    computation (``:213``).

    Returns ``(packed u8 [N, Kp/2], scale f16 [N, Kp/g], zero f16 [N, Kp/g], padding)`` where
    ``Kp`` is ``K`` rounded up to the group.
    """
    if dtype == "bf16":
        wf = bf16_bits_to_f32(w)
    elif dtype == "f32":
        wf = np.asarray(w, dtype=np.float32)
    elif dtype == "f16":
        wf = np.asarray(w, dtype=np.float16).astype(np.float32)
    else:
        raise ValueError(dtype)
    n, k = wf.shape
    g = min(group, k) if k else group
    padded, padding = _pad_rows_to_group(wf, g)
    kp = padded.shape[1]
    grouped = padded.reshape(n, kp // g, g)
    lo = grouped.min(axis=-1, keepdims=True)
    hi = grouped.max(axis=-1, keepdims=True)
    if dtype == "bf16":
        diff = round_bf16(hi - lo)
        scale = round_bf16(diff / np.float32(LEVELS))
    elif dtype == "f16":
        diff = (hi - lo).astype(np.float16).astype(np.float32)
        scale = (diff / np.float32(LEVELS)).astype(np.float16).astype(np.float32)
    else:
        scale = (hi - lo) / np.float32(LEVELS)
    scale = scale.astype(np.float32)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    codes = np.clip(np.rint((grouped - lo) / scale), 0, LEVELS).astype(np.uint8)
    packed = pack(codes.reshape(n, kp))
    return (packed, scale[..., 0].astype(np.float16), lo[..., 0].astype(np.float16), padding)


def dequantize(packed, scale, zero, k=None, out="f32"):
    """``codes * scale + zero`` in fp32, narrowed to ``k`` columns, then cast (``kv_cache.py:249-257``).

    ``out`` is ``"f32"`` (returns float32), ``"bf16"`` (returns uint16 bf16 bit patterns) or
    ``"f16"`` (returns float16).
    The fp32 product is exact (a 4-bit code times an fp16 scale needs at most 15 significant
    bits), so a fused multiply-add on the device gives the same fp32 value before the cast.
    """
    codes = unpack(packed).astype(np.float32)
    n, kp = codes.shape
    g = kp // scale.shape[1]
    grouped = codes.reshape(n, kp // g, g)
    restored = grouped * scale.astype(np.float32)[..., None]
    restored = restored + zero.astype(np.float32)[..., None]
    flat = restored.reshape(n, kp)
    if k is not None:
        flat = flat[:, :k]
    flat = np.ascontiguousarray(flat, dtype=np.float32)
    if out == "f32":
        return flat
    if out == "bf16":
        return f32_to_bf16_bits(flat)
    if out == "f16":
        return flat.astype(np.float16)
    raise ValueError(out)


def linear(x_bf16_bits, packed, scale, zero, k=None, bf16_weight=False):
    """``y = x . W^T`` in fp32 over the dequantized weight (the reference's dequant-to-scratch
    ``F.linear``; ``rocketllm/quant/registry.py:529-535`` then transformers ``nn.Linear``).

    ``bf16_weight=True`` rounds the dequantized weight to bf16 first -- exactly the weight the
    reference's bf16 model multiplies by (``dequantize().to(bfloat16)``); the default keeps the
    exact fp32 weight (the fp32 CPU model's weight).
    Returns fp32 ``[M, N]``; the device returns bf16 and is compared within a tolerance.
    """
    w = dequantize(packed, scale, zero, k=k)
    if bf16_weight:
        w = round_bf16(w)
    x = bf16_bits_to_f32(x_bf16_bits)
    return (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def synthetic_weight(n, k, group=64, seed=0):
    """The isolated-sweep weight: uniform random bytes, scale ~ U[0.005, 0.02], zero = -8 * scale.

    Mirrors ``make_weight`` in ``rocketllm_b200.quant.synthetic`` with numpy's generator so the CPU
    side can build the same kind of input without torch; bit-identical inputs come from torch when
    a test needs the exact device tensors.
    """
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scale = (0.005 + 0.015 * rng.random((n, k // group), dtype=np.float32)).astype(np.float16)
    zero = (np.float32(-8.0) * scale.astype(np.float32)).astype(np.float16)
    return packed, scale, zero


# ----------------------------------------------------------------------------------------------
# MoE: router, permutation, expert MLP, combine
# ----------------------------------------------------------------------------------------------

def softmax_f32(logits):
    z = logits.astype(np.float32)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def router_topk(hidden, router_w, top_k):
    """``MixtralTopKRouter``: logits = h . Wr^T, softmax in fp32, top-k, renormalise.

    Follows transformers ``models/mixtral/modeling_mixtral.py:101-116``.  Returns
    ``(indices int64 [T, k], weights f32 [T, k])``, indices in descending-score order.
    """
    logits = hidden.astype(np.float32) @ router_w.astype(np.float32).T
    probs = softmax_f32(logits)
    order = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k]
    weights = np.take_along_axis(probs, order, axis=-1)
    weights = weights / weights.sum(axis=-1, keepdims=True)
    return order.astype(np.int64), weights.astype(np.float32)


def router_selection(indices):
    """``RouterSelection.observe``: the sorted set of experts any token chose (``router.py:88-93``)."""
    return tuple(sorted(set(np.asarray(indices).reshape(-1).tolist())))


def moe_permute(topk_idx, num_experts):
    """Stable counting sort of the ``T*k`` (token, slot) pairs by expert.

    Returns ``(perm int32 [T*k], offsets int32 [E+1])``: ``perm[p]`` is the flat slot index
    ``t*k + j`` placed at row ``p`` of the expert-sorted order; rows of expert ``e`` are
    ``offsets[e]:offsets[e+1]``, in increasing flat-slot order.  The reference's per-expert loop
    (transformers ``modeling_mixtral.py:74-98``) visits each expert's (slot, token) pairs slot-major;
    the order inside an expert only decides which row a result sits in, never its value, because
    every row is computed independently and :func:`moe_combine` gathers by slot.
    """
    flat = np.asarray(topk_idx, dtype=np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=num_experts).astype(np.int64)
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    perm = np.argsort(flat, kind="stable").astype(np.int32)
    return perm, offsets.astype(np.int32)


def moe_combine(y_perm, perm, topk_w, num_tokens, top_k):
    """``out[t] = sum_j w[t, j] * y[row of (t, j)]`` in slot order ``j = 0..k-1``, fp32."""
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.shape[0], dtype=perm.dtype)
    y = y_perm.astype(np.float32)
    out = np.zeros((num_tokens, y.shape[1]), dtype=np.float32)
    for j in range(top_k):
        rows = inv[np.arange(num_tokens) * top_k + j]
        out += topk_w[:, j:j + 1].astype(np.float32) * y[rows]
    return out


def silu(a):
    a = a.astype(np.float32)
    return a / (np.float32(1.0) + np.exp(-a))


def expert_mlp(x_bf16_bits, gate_up, down, inter):
    """One expert's SwiGLU MLP over dequantized weights, fp32 (``modeling_mixtral.py:84-91``).

    ``gate_up`` and ``down`` are ``(packed, scale, zero)`` triples; ``gate_up`` stacks the gate rows
    ``[0, I)`` over the up rows ``[I, 2I)``.  The intermediate activation is rounded to bf16, as the
    bf16 model's own ``F.linear`` output would be.
    """
    h = linear(x_bf16_bits, *gate_up)
    act = round_bf16(silu(round_bf16(h[:, :inter])) * round_bf16(h[:, inter:]))
    return linear(f32_to_bf16_bits(act), *down)


# ----------------------------------------------------------------------------------------------
# int4 KV cache (KIVI layout): K grouped along tokens, V along channels, recent tokens exact
# ----------------------------------------------------------------------------------------------

def kv_quantize(x, axis, group=64, dtype="bf16"):
    """The reference ``quantize(tensor, axis, group_size)`` on an N-d tensor (``kv_cache.py:190-221``).

    The grouped axis is moved last and every leading index is one row of :func:`quantize`.
    Returns ``(packed u8 [..., Lp/2], scale f16 [..., Lp/g], zero f16 [..., Lp/g], padding)``
    in the moved layout, exactly the fields of the reference's ``QuantizedTensor``.
    """
    x = np.asarray(x)
    moved = np.moveaxis(x, axis, -1)
    lead = moved.shape[:-1]
    packed, scale, zero, padding = quantize(moved.reshape(-1, moved.shape[-1]), group, dtype)
    return (packed.reshape(lead + packed.shape[1:]), scale.reshape(lead + scale.shape[1:]),
            zero.reshape(lead + zero.shape[1:]), padding)


def kv_dequantize(packed, scale, zero, axis, length, out="bf16"):
    """``QuantizedTensor.dequantize`` (``kv_cache.py:249-257``): rows of the moved layout expanded,
    narrowed to ``length`` along the grouped axis, the axis moved back, cast to ``out``."""
    lead = packed.shape[:-1]
    flat = dequantize(packed.reshape(-1, packed.shape[-1]), scale.reshape(-1, scale.shape[-1]),
                      zero.reshape(-1, zero.shape[-1]), k=length, out=out)
    return np.moveaxis(flat.reshape(lead + (length,)), -1, axis)


class KiviCache:
    """The reference ``QuantizedKVCache`` restated for one layer (``kv_cache.py:277-352``).

    ``update(k, v)`` takes bf16 bit patterns ``[b, kvh, t, d]``, appends them to the exact window,
    moves whole groups of the oldest tokens past ``residual`` into append-only quantized blocks
    (K along tokens, V along channels) and returns the whole history in bf16 bits: the expanded
    blocks, oldest first, then the window.
    """

    def __init__(self, group=64, residual=128):
        self.group, self.residual = group, residual
        self.k = self.v = None
        self.blocks = []          # (k_block, v_block): kv_quantize outputs of each flush

    def update(self, k, v):
        k = np.asarray(k, dtype=np.uint16)
        v = np.asarray(v, dtype=np.uint16)
        self.k = k if self.k is None else np.concatenate([self.k, k], axis=2)
        self.v = v if self.v is None else np.concatenate([self.v, v], axis=2)
        excess = self.k.shape[2] - self.residual
        take = (excess // self.group) * self.group if excess > 0 else 0
        if take > 0:
            self.blocks.append((kv_quantize(self.k[:, :, :take], 2, self.group),
                                kv_quantize(self.v[:, :, :take], 3, self.group), take))
            self.k = self.k[:, :, take:]
            self.v = self.v[:, :, take:]
        return self.history()

    def quantized_tokens(self):
        return sum(t for _, _, t in self.blocks)

    def history(self):
        ks = [kv_dequantize(*kb[:3], axis=2, length=t) for kb, _, t in self.blocks]
        vs = [kv_dequantize(*vb[:3], axis=3, length=self.k.shape[3]) for _, vb, t in self.blocks]
        return (np.concatenate(ks + [self.k], axis=2), np.concatenate(vs + [self.v], axis=2))


def attention_decode(q, k, v, scaling):
    """One query token's softmax attention over ``k``/``v`` ``[b, kvh, T, d]`` (fp32 inputs),
    query ``[b, h, d]``; query head ``h`` reads kv head ``h // (h_total / kvh)`` (transformers
    ``repeat_kv``).  fp64 arithmetic, fp32 result ``[b, h, d]``."""
    b, h, d = q.shape
    kvh = k.shape[1]
    rep = h // kvh
    kk = np.repeat(k.astype(np.float64), rep, axis=1)
    vv = np.repeat(v.astype(np.float64), rep, axis=1)
    logits = np.einsum("bhd,bhtd->bht", q.astype(np.float64), kk) * scaling
    logits -= logits.max(axis=-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bht,bhtd->bhd", p, vv).astype(np.float32)


def attention_causal(q, k, v, scaling):
    """``Q`` query positions ``[b, h, Q, d]`` that are the last ``Q`` of the ``T`` keys / values
    ``[b, kvh, T, d]``: position ``i`` attends to keys ``0 .. T - Q + i`` (transformers' causal
    SDPA over a cache).  fp64 arithmetic, fp32 result ``[b, h, Q, d]``."""
    b, h, nq, d = q.shape
    t = k.shape[2]
    out = np.empty((b, h, nq, d), dtype=np.float32)
    for i in range(nq):
        n = t - nq + i + 1
        out[:, :, i] = attention_decode(q[:, :, i], k[:, :, :n], v[:, :, :n], scaling)
    return out

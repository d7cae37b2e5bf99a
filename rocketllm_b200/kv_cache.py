"""int4 KV cache (KIVI layout) whose decode attention reads the packed history directly.

Counterpart of the reference's ``QuantizedKVCache`` (``rocketllm/quant/kv_cache.py:146-445``):
K is quantized per channel over groups of 64 tokens, V per token over groups of 64 channels, the
newest tokens stay exact in a window of ``residual_length`` (+ up to one group), and whole groups
past the window move into append-only quantized storage.  The codes, scales and zeros are the
reference codec's output bit for bit (the RW4 quantize kernel is that codec).

The difference is what a decode step does with them.  The reference expands every quantized block
back to the compute dtype on every step and hands the model's attention the whole history
(``kv_cache.py:308-316``).  Here the storage is laid out for the device (``include/rw4.h``,
``rw4_kv_attention_decode``) and, once :func:`enable_kv_attention` has installed the ``"rw4_kv"``
attention implementation, a one-token step returns only the window from ``update`` -- tagged with
its cache and layer -- and the attention function runs the CUDA kernel over packed history +
window; so does a short multi-token chunk (a speculative verify pass) of a cache created with
``causal_chunks``, causally masked inside the window.  Anything else (a prefill, a masked query, a
cache used without the attention implementation) gets the reference's behaviour: the expanded
history, then SDPA.

The codec and attention operations are injected (``ops``): the default runs the RW4 CUDA kernels;
the CPU tests drive the same bookkeeping with a numpy implementation of the three operations.
"""
import dataclasses

import torch
from transformers.cache_utils import Cache

ATTN_NAME = "rw4_kv"

KV_AUTO = "auto"
KV_FP16 = "fp16"
KV_INT4 = "int4"
KV_HQQ = "hqq"
KV_QUANTO = "quanto"
KV_CHOICES = (KV_AUTO, KV_FP16, KV_INT4, KV_HQQ, KV_QUANTO)


@dataclasses.dataclass(frozen=True)
class KVCacheConfig:
    """Layout of the cache (``kv_cache.py:146-170``).  The device layout fixes a group of 64 and the
    recipe's axes (K along tokens, V along channels); other values are rejected, not emulated."""

    group_size: int = 64
    residual_length: int = 128
    compute_dtype: object = torch.bfloat16
    key_axis: int = 2
    value_axis: int = 3

    def __post_init__(self):
        if self.group_size < 2:
            raise ValueError(f"group_size must be at least 2, not {self.group_size}")
        if self.residual_length < self.group_size:
            raise ValueError(f"residual_length {self.residual_length} is below group_size "
                             f"{self.group_size}; the window could never complete a group")
        if self.group_size != 64 or self.key_axis != 2 or self.value_axis != 3:
            raise ValueError("the int4 KV layout is group 64, K along tokens (axis 2), V along "
                             "channels (axis 3)")


class CudaKVOps:
    """The codec and the decode attention on the RW4 CUDA kernels."""

    def __init__(self):
        from . import kernels
        self.k = kernels

    def quantize(self, x2d):
        packed, scale, zero, _ = self.k.quantize(x2d, 64)
        return packed, scale, zero

    def dequantize(self, packed, scale, zero):
        return self.k.dequantize(packed, scale, zero)

    def attend(self, query, layer, scaling):
        return self.k.kv_attention_decode(query, layer.k_codes, layer.k_sz, layer.v_codes,
                                          layer.v_sz, layer.groups, layer.k_res, layer.v_res,
                                          layer.rlen, scaling)


class _KVLayer:
    """One layer's storage: quantized groups (capacity ``gcap``) and the exact window."""

    def __init__(self, like, rcap):
        b, kvh, _, d = like.shape
        if d % 64:
            raise ValueError(f"head_dim {d} is not a multiple of 64")
        dev = like.device
        self.shape = (b, kvh, d)
        self.dtype = like.dtype
        self.k_codes = torch.empty((b, kvh, 0, d, 32), dtype=torch.uint8, device=dev)
        self.k_sz = torch.empty((b, kvh, 0, d, 2), dtype=torch.float16, device=dev)
        self.v_codes = torch.empty((b, kvh, 0, d // 2), dtype=torch.uint8, device=dev)
        self.v_sz = torch.empty((b, kvh, 0, d // 64, 2), dtype=torch.float16, device=dev)
        self.groups = 0
        self.blocks = []   # tokens moved by each flush, oldest first (the reference's blocks)
        self.k_res = torch.zeros((b, kvh, rcap, d), dtype=like.dtype, device=dev)
        self.v_res = torch.zeros((b, kvh, rcap, d), dtype=like.dtype, device=dev)
        self.rlen = 0

    @property
    def gcap(self):
        return self.k_codes.shape[2]

    def grow_groups(self, need):
        if need <= self.gcap:
            return
        cap = max(need, 2 * self.gcap, 4)
        b, kvh, d = self.shape
        g = self.groups
        kc = torch.empty((b, kvh, cap, d, 32), dtype=torch.uint8, device=self.k_codes.device)
        ks = torch.empty((b, kvh, cap, d, 2), dtype=torch.float16, device=self.k_codes.device)
        vc = torch.empty((b, kvh, cap * 64, d // 2), dtype=torch.uint8, device=self.k_codes.device)
        vs = torch.empty((b, kvh, cap * 64, d // 64, 2), dtype=torch.float16,
                         device=self.k_codes.device)
        if g:
            kc[:, :, :g].copy_(self.k_codes[:, :, :g])
            ks[:, :, :g].copy_(self.k_sz[:, :, :g])
            vc[:, :, :g * 64].copy_(self.v_codes[:, :, :g * 64])
            vs[:, :, :g * 64].copy_(self.v_sz[:, :, :g * 64])
        self.k_codes, self.k_sz, self.v_codes, self.v_sz = kc, ks, vc, vs

    def grow_window(self, need):
        if need <= self.k_res.shape[2]:
            return
        cap = (need + 63) // 64 * 64
        for name in ("k_res", "v_res"):
            old = getattr(self, name)
            new = torch.zeros(old.shape[:2] + (cap, old.shape[3]), dtype=old.dtype,
                              device=old.device)
            new[:, :, :self.rlen].copy_(old[:, :, :self.rlen])
            setattr(self, name, new)

    def nbytes(self):
        t = self.groups * 64
        b, kvh, d = self.shape
        quant = b * kvh * (self.groups * d * (32 + 4) + t * (d // 2 + (d // 64) * 4))
        return quant + 2 * b * kvh * self.rlen * d * self.k_res.element_size()


class RW4KVCache(Cache):
    """int4 KV cache with an exact window, in the shape transformers expects.

    ``fused``: a one-token ``update`` returns the window only, tagged for the ``"rw4_kv"``
    attention implementation (see :func:`enable_kv_attention`, which must be active on the model);
    otherwise ``update`` returns the expanded history as the reference does.

    ``causal_chunks``: the caller promises that every multi-token update (up to 16 tokens) is the
    causal continuation of one unpadded sequence per batch row -- a speculative verify pass -- so
    those queries too can run on the packed history (causally masked inside the window) whatever
    mask transformers builds for them.
    """

    is_compileable = False

    def __init__(self, config=None, ops=None, fused=False, causal_chunks=False):
        try:
            Cache.__init__(self, layers=[])
        except (TypeError, ValueError):
            Cache.__init__(self)
        self.config = config if config is not None else KVCacheConfig()
        self.ops = ops if ops is not None else CudaKVOps()
        self.fused = fused
        self.causal_chunks = causal_chunks
        self._kv = []
        self._seen_tokens = 0
        self.flushes = 0

    # -- transformers Cache surface ------------------------------------------------------------

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        if key_states.dtype != torch.bfloat16:
            raise TypeError(f"the int4 KV cache takes bf16 keys / values, not {key_states.dtype}")
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]
        layer = self._ensure(layer_idx, key_states)
        t = key_states.shape[-2]
        layer.grow_window(layer.rlen + t)
        layer.k_res[:, :, layer.rlen:layer.rlen + t].copy_(key_states)
        layer.v_res[:, :, layer.rlen:layer.rlen + t].copy_(value_states)
        layer.rlen += t
        self._flush(layer)
        if self.fused and (t == 1 or (self.causal_chunks and t <= 16)):
            k = layer.k_res[:, :, :layer.rlen]
            v = layer.v_res[:, :, :layer.rlen]
            k._rw4_kv = (self, layer_idx)
            return k, v
        return self.history(layer_idx)

    def _ensure(self, layer_idx, like):
        while len(self._kv) <= layer_idx:
            rcap = self.config.residual_length + self.config.group_size
            self._kv.append(_KVLayer(like, max(rcap, 64)))
        return self._kv[layer_idx]

    def _flush(self, layer):
        """Whole groups of the oldest window tokens past ``residual_length`` move into the
        quantized storage (``kv_cache.py:328-352``)."""
        cfg = self.config
        excess = layer.rlen - cfg.residual_length
        if excess <= 0:
            return
        take = (excess // cfg.group_size) * cfg.group_size
        if take <= 0:
            return
        b, kvh, d = layer.shape
        ng = take // 64
        g0 = layer.groups
        layer.grow_groups(g0 + ng)
        k = layer.k_res[:, :, :take]
        v = layer.v_res[:, :, :take]
        # K: rows (b, kvh, channel) grouped along tokens
        kp, ks, kz = self.ops.quantize(k.transpose(2, 3).reshape(b * kvh * d, take).contiguous())
        layer.k_codes[:, :, g0:g0 + ng].copy_(kp.view(b, kvh, d, ng, 32).permute(0, 1, 3, 2, 4))
        layer.k_sz[:, :, g0:g0 + ng, :, 0].copy_(ks.view(b, kvh, d, ng).permute(0, 1, 3, 2))
        layer.k_sz[:, :, g0:g0 + ng, :, 1].copy_(kz.view(b, kvh, d, ng).permute(0, 1, 3, 2))
        # V: rows (b, kvh, token) grouped along channels
        vp, vs, vz = self.ops.quantize(v.reshape(b * kvh * take, d).contiguous())
        t0 = g0 * 64
        layer.v_codes[:, :, t0:t0 + take].copy_(vp.view(b, kvh, take, d // 2))
        layer.v_sz[:, :, t0:t0 + take, :, 0].copy_(vs.view(b, kvh, take, d // 64))
        layer.v_sz[:, :, t0:t0 + take, :, 1].copy_(vz.view(b, kvh, take, d // 64))
        layer.groups += ng
        layer.blocks.append(take)
        rest = layer.rlen - take
        for buf in (layer.k_res, layer.v_res):
            buf[:, :, :rest].copy_(buf[:, :, take:take + rest].clone())
        layer.rlen = rest
        self.flushes += 1

    def history(self, layer_idx):
        """The whole history ``(K, V)`` ``[b, kvh, T, d]`` in the compute dtype: the expanded
        quantized groups, oldest first, then the window (what the reference's ``update``
        returns)."""
        layer = self._kv[layer_idx]
        kr = layer.k_res[:, :, :layer.rlen]
        vr = layer.v_res[:, :, :layer.rlen]
        if not layer.groups:
            return kr, vr
        b, kvh, d = layer.shape
        g = layer.groups
        t = g * 64
        kp = layer.k_codes[:, :, :g].permute(0, 1, 3, 2, 4).reshape(b * kvh * d, g * 32)
        ks = layer.k_sz[:, :, :g, :, 0].permute(0, 1, 3, 2).reshape(b * kvh * d, g)
        kz = layer.k_sz[:, :, :g, :, 1].permute(0, 1, 3, 2).reshape(b * kvh * d, g)
        kq = self.ops.dequantize(kp.contiguous(), ks.contiguous(), kz.contiguous())
        kq = kq.view(b, kvh, d, t).transpose(2, 3).to(layer.dtype)
        vp = layer.v_codes[:, :, :t].reshape(b * kvh * t, d // 2)
        vs = layer.v_sz[:, :, :t, :, 0].reshape(b * kvh * t, d // 64)
        vz = layer.v_sz[:, :, :t, :, 1].reshape(b * kvh * t, d // 64)
        vq = self.ops.dequantize(vp.contiguous(), vs.contiguous(), vz.contiguous())
        vq = vq.view(b, kvh, t, d).to(layer.dtype)
        return torch.cat([kq, kr], dim=2), torch.cat([vq, vr], dim=2)

    def attend(self, layer_idx, query, scaling):
        """Queries ``[b, h, q, d]`` -- the window's last ``q`` tokens, attending causally -- over
        the layer's packed history and window; returns ``[b, q, h, d]`` in the compute dtype."""
        return self.ops.attend(query, self._kv[layer_idx], scaling)

    def quantized(self, layer_idx):
        """The quantized history in the reference's block layout, blocks concatenated along the
        token axis: ``(k_packed [b,kvh,d,T/2], k_scale [b,kvh,d,T/64], k_zero, v_packed
        [b,kvh,T,d/2], v_scale [b,kvh,T,d/64], v_zero)``."""
        layer = self._kv[layer_idx]
        b, kvh, d = layer.shape
        g = layer.groups
        t = g * 64
        kp = layer.k_codes[:, :, :g].permute(0, 1, 3, 2, 4).reshape(b, kvh, d, g * 32)
        ks = layer.k_sz[:, :, :g, :, 0].permute(0, 1, 3, 2)
        kz = layer.k_sz[:, :, :g, :, 1].permute(0, 1, 3, 2)
        return (kp, ks, kz, layer.v_codes[:, :, :t], layer.v_sz[:, :, :t, :, 0],
                layer.v_sz[:, :, :t, :, 1])

    def crop(self, max_length):
        """Drop everything past ``max_length`` tokens -- from the exact window only; cutting into a
        quantized group raises (``kv_cache.py:354-385``)."""
        for i, layer in enumerate(self._kv):
            length = self.get_seq_length(i)
            if max_length < 0:
                max_length = length - abs(max_length)
            if length <= max_length:
                continue
            quantized = layer.groups * 64
            keep = max_length - quantized
            if keep < 0:
                raise ValueError(
                    f"cannot crop this cache to {max_length} tokens: {quantized} of them are "
                    f"already quantized into whole groups and only the {length - quantized} most "
                    f"recent are still exact; raise residual_length above the speculative "
                    f"lookahead if a deeper rollback is needed")
            layer.rlen = keep
        self._seen_tokens = min(self._seen_tokens, max(0, int(max_length)))

    def get_seq_length(self, layer_idx=0):
        if layer_idx >= len(self._kv):
            return 0
        layer = self._kv[layer_idx]
        return layer.groups * 64 + layer.rlen

    def get_mask_sizes(self, query_length, layer_idx=0):
        if torch.is_tensor(query_length):   # older call sites pass cache_position
            query_length = query_length.shape[0]
        return self.get_seq_length(layer_idx) + query_length, 0

    def get_max_cache_shape(self, layer_idx=0):
        return -1

    def get_usable_length(self, new_seq_length, layer_idx=0):
        return self.get_seq_length(layer_idx)

    @property
    def is_sliding(self):
        return [False] * len(self._kv)

    @property
    def is_initialized(self):
        return len(self._kv) > 0

    def reorder_cache(self, beam_idx):
        for layer in self._kv:
            for name in ("k_codes", "k_sz", "v_codes", "v_sz", "k_res", "v_res"):
                t = getattr(layer, name)
                if t.numel():
                    setattr(layer, name, t.index_select(0, beam_idx.to(t.device)))

    @property
    def seen_tokens(self):
        return self._seen_tokens

    def __len__(self):
        return len(self._kv)

    def nbytes(self):
        """Bytes of the valid history: codes, scales and zeros plus the exact window."""
        return sum(layer.nbytes() for layer in self._kv)

    def report(self):
        n = len(self._kv)
        return {
            "kind": "int4", "layers": n, "tokens": self.get_seq_length(0),
            "quantized_tokens": self._kv[0].groups * 64 if n else 0,
            "residual_tokens": sum(layer.rlen for layer in self._kv) // max(1, n),
            "group_size": self.config.group_size,
            "residual_length": self.config.residual_length, "flushes": self.flushes,
            "bytes": self.nbytes(), "fused": self.fused,
        }


# -- the attention implementation ---------------------------------------------------------------

def rw4_kv_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                     is_causal=None, **kwargs):
    """transformers attention interface ``"rw4_kv"``: the packed-history kernel for a one-token
    query whose keys came from a fused :class:`RW4KVCache` (or a chunk of up to 16 / (heads per kv
    head) positions of a ``causal_chunks`` cache), SDPA over the expanded history for every other
    case."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    tag = getattr(key, "_rw4_kv", None)
    if tag is not None:
        cache, layer_idx = tag
        if scaling is None:
            scaling = query.shape[-1] ** -0.5
        drop = dropout if getattr(module, "training", False) else 0.0
        q_len = query.shape[2]
        cols = q_len * (query.shape[1] // key.shape[1])
        if not drop and ((q_len == 1 and attention_mask is None) or
                         (1 < q_len and cache.causal_chunks and cols <= 16)):
            return cache.attend(layer_idx, query, scaling), None
        key, value = cache.history(layer_idx)
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                  scaling=scaling, is_causal=is_causal, **kwargs)


_REGISTERED = False


def register_kv_attention():
    """Register ``"rw4_kv"`` with transformers' attention and mask interfaces (idempotent); the
    masks are SDPA's."""
    global _REGISTERED
    if _REGISTERED:
        return
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(ATTN_NAME, rw4_kv_attention)
    AttentionMaskInterface.register(ATTN_NAME, sdpa_mask)
    _REGISTERED = True


def enable_kv_attention(model):
    """Switch ``model`` (a transformers ``PreTrainedModel``) to the ``"rw4_kv"`` attention
    implementation.  Caches other than a fused :class:`RW4KVCache` are unaffected: their keys
    carry no tag and go to SDPA."""
    register_kv_attention()
    if hasattr(model, "set_attn_implementation"):
        model.set_attn_implementation(ATTN_NAME)
    else:
        model.config._attn_implementation = ATTN_NAME
    return model


def resolve_kv_cache(setting, weight_bytes=None, device_bytes=None, headroom=0.15):
    """``(choice, reason)`` for a ``kv_cache=`` setting (``kv_cache.py:449-486``): ``"auto"`` keeps
    the context exact when the weights fit resident with ``headroom`` to spare, and quantizes it
    when they do not; an explicit setting passes through."""
    if setting not in KV_CHOICES:
        raise ValueError(f"kv_cache must be one of {', '.join(KV_CHOICES)}, not {setting!r}")
    if setting != KV_AUTO:
        return setting, "requested explicitly"
    if not weight_bytes or not device_bytes:
        return KV_FP16, "no measured weight or device size to decide from"
    if weight_bytes * (1.0 + max(0.0, headroom)) <= device_bytes:
        return KV_FP16, "the weights fit resident, so the context is kept exact"
    return KV_INT4, "the weights do not fit resident, so the context is quantized"


def build_kv_cache(choice, config=None, fused=True):
    """The cache a resolved choice names, or ``None`` for the stock cache (``kv_cache.py:489-503``).
    ``hqq`` / ``quanto`` (transformers' own quantized caches on optional packages) are not part of
    this package and fall back to the stock cache, as the reference does when they are missing."""
    if choice == KV_INT4:
        return RW4KVCache(config, fused=fused)
    return None

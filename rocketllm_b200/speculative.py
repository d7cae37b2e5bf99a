"""Speculative decoding: a resident draft proposes k tokens, one pass of the RW4 target checks them.

Counterpart of the reference's ``rocketllm/spec/draft.py``.  The point on this path is the target
pass: the k+1 candidate positions go through every ``RW4Linear`` as one M = k+1 activation block,
which the dequant-GEMV serves with ONE read of each weight (M <= 16), so a streamed or HBM-bound
pass costs about what a one-token step costs and a fully accepted pass yields k+1 tokens.

What follows the reference's contract (``draft.py:262-592``): the sampling warp shared by draft and
target (``SamplingParams``), the accept rule min(1, p/q) with the rejected position redrawn from
(p - q)+ and the bonus token from the spare distribution when everything is accepted (exactly
distribution-preserving; greedy is the same rule with point masses), the loop invariant (the target
cache holds every token but the last one emitted), cropping the target and draft caches after a
rejection, the adaptive lookahead a/(1-a), end-of-sequence handling and the statistics.

What is this package's own: the accept test runs on the device over all proposals at once (one
host read per pass instead of one per proposal), and the draft keeps its proposals' distributions
as one [k, vocab] tensor.
"""
import dataclasses
import time

import torch

SPEC_AUTO = "auto"
SPEC_ON = "on"
SPEC_OFF = "off"
SPEC_CHOICES = (SPEC_AUTO, SPEC_ON, SPEC_OFF)

# strings two tokenizers with the same vocabulary size must still encode identically
_TOKENIZER_PROBES = (
    "Speculative decoding checks k draft tokens in one pass.",
    "\tindented\n  and trailing spaces   ",
    "3.14159 2.71828 1e-9 0x7F",
    "for i in range(10): print(i ** 2)",
    "it's -- \"quoted\" (and) [bracketed]",
)


class DraftIncompatible(ValueError):
    """The draft does not share the target's token language (``draft.py:95-104``)."""


def check_compatible(target_config, target_tokenizer, draft_config, draft_tokenizer):
    """Refuse a draft whose vocabulary or tokenizer differs from the target's (``draft.py:107-153``):
    the vocabulary sizes, bos / eos ids and the encodings of a few probe strings must agree."""
    problems = []
    tv = getattr(target_config, "vocab_size", None)
    dv = getattr(draft_config, "vocab_size", None)
    if tv and dv and int(tv) != int(dv):
        problems.append(f"vocabulary sizes differ: target {tv}, draft {dv}")
    if target_tokenizer is not None and draft_tokenizer is not None:
        for name in ("bos_token_id", "eos_token_id"):
            a = getattr(target_tokenizer, name, None)
            b = getattr(draft_tokenizer, name, None)
            if a != b:
                problems.append(f"{name} differs: target {a!r}, draft {b!r}")
        for probe in _TOKENIZER_PROBES:
            if target_tokenizer.encode(probe) != draft_tokenizer.encode(probe):
                problems.append(f"the tokenizers encode {probe!r} differently")
                break
    if problems:
        raise DraftIncompatible("the draft cannot verify against this target: "
                                + "; ".join(problems))
    return True


@dataclasses.dataclass(frozen=True)
class SamplingParams:
    """The warp applied to logits before drawing, shared by draft and target
    (``draft.py:159-227``)."""

    do_sample: bool = False
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0

    @classmethod
    def from_generation(cls, config=None, **overrides):
        def pick(name, default):
            v = overrides.get(name)
            if v is None and config is not None:
                v = getattr(config, name, None)
            return default if v is None else v

        return cls(do_sample=bool(pick("do_sample", False)),
                   temperature=float(pick("temperature", 1.0) or 1.0),
                   top_k=int(pick("top_k", 0) or 0), top_p=float(pick("top_p", 1.0) or 1.0))

    @property
    def greedy(self):
        return not self.do_sample or self.temperature <= 0.0

    def distribution(self, logits):
        """Logits ``[..., V]`` -> the sampled probability vectors (one-hot argmax when greedy)."""
        logits = logits.float()
        if self.greedy:
            return torch.zeros_like(logits).scatter_(-1, logits.argmax(-1, keepdim=True), 1.0)
        logits = logits / self.temperature
        if 0 < self.top_k < logits.shape[-1]:
            kth = torch.topk(logits, self.top_k, dim=-1).values[..., -1:]
            logits = logits.masked_fill(logits < kth, float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        if 0.0 < self.top_p < 1.0:
            sorted_p, order = torch.sort(probs, dim=-1, descending=True)
            before = sorted_p.cumsum(-1) - sorted_p        # mass strictly ahead of each token
            sorted_p = sorted_p.masked_fill(before >= self.top_p, 0.0)
            probs = torch.zeros_like(probs).scatter_(-1, order, sorted_p)
            probs = probs / probs.sum(-1, keepdim=True)
        return probs


def _draw(probs, generator=None):
    """Token ids from probability rows ``[n, V]`` (a point mass draws its token)."""
    if generator is not None and probs.device != generator.device:
        probs = probs.to(generator.device)
    return torch.multinomial(probs, 1, generator=generator)[:, 0]


def verify(proposals, draft_probs, target_probs, generator=None):
    """Accept / reject ``k`` proposals at once.  Returns ``(accepted, next_token)`` as ints.

    ``proposals`` int64 ``[k]``, ``draft_probs`` ``[k, V]`` (the distribution each proposal was
    drawn from), ``target_probs`` ``[k + 1, V]``.  Proposal i survives when ``p_i >= q_i`` or a
    uniform draw falls below ``p_i / q_i`` (a proposal the draft gave no mass survives only where
    the target gives it some); the first failure is replaced by a draw from ``(p - q)+``
    renormalised (``p`` where that vanishes), and when all survive the bonus token is drawn from
    the spare ``target_probs[k]`` (``draft.py:413-456``).  One device->host read.
    """
    k = int(proposals.shape[0])
    dev = target_probs.device
    if k == 0:
        return 0, int(_draw(target_probs[:1], generator)[0])
    idx = proposals.to(dev).view(k, 1)
    p = target_probs[:k].gather(1, idx)[:, 0]
    q = draft_probs.to(dev).gather(1, idx)[:, 0]
    ratio = torch.where(q > 0, p / q.clamp_min(1e-30), (p > 0).to(p.dtype))
    gdev = generator.device if generator is not None else dev
    u = torch.rand(k, generator=generator, device=gdev).to(dev)
    keep = (ratio >= 1.0) | ((ratio > 0.0) & (u < ratio))
    failed = (~keep).to(torch.int64)
    # first rejected position, or k when all were kept
    first = torch.where(failed.any(), torch.argmax(failed), torch.tensor(k, device=dev))
    # the replacement distribution at `first`: (p - q)+ normalised at a rejection, else the spare
    pf = target_probs[first.clamp(max=k)]
    qf = draft_probs.to(dev)[first.clamp(max=k - 1)]
    residual = (pf - qf).clamp_min(0.0)
    total = residual.sum()
    repl = torch.where(total > 0, residual / total.clamp_min(1e-30), pf)
    dist = torch.where(first < k, repl, target_probs[k])
    tok = _draw(dist.view(1, -1), generator)[0]
    accepted, token = torch.stack([first, tok.to(first.dtype)]).tolist()
    return int(accepted), int(token)


@dataclasses.dataclass
class SpeculationStats:
    """What speculation did (``draft.py:367-410``)."""

    passes: int = 0
    proposed: int = 0
    accepted: int = 0
    emitted: int = 0
    target_seconds: float = 0.0
    draft_seconds: float = 0.0
    lookahead_sum: int = 0

    @property
    def acceptance_rate(self):
        return self.accepted / self.proposed if self.proposed else 0.0

    @property
    def tokens_per_pass(self):
        return self.emitted / self.passes if self.passes else 0.0

    @property
    def mean_lookahead(self):
        return self.lookahead_sum / self.passes if self.passes else 0.0

    def to_dict(self):
        d = dataclasses.asdict(self)
        d.update(acceptance_rate=self.acceptance_rate, tokens_per_pass=self.tokens_per_pass,
                 mean_lookahead=self.mean_lookahead)
        return d


class DraftModel:
    """A small resident model that proposes tokens with its own cache (``draft.py:262-362``)."""

    def __init__(self, model, tokenizer=None, name=""):
        self.model = model
        self.tokenizer = tokenizer
        self.name = name or getattr(getattr(model, "config", None), "name_or_path", "draft")
        self.cache = None
        self.forwards = 0
        self.seconds = 0.0

    @classmethod
    def load(cls, path, target_config=None, target_tokenizer=None, device=None, dtype=None):
        """Load a draft and refuse it before placing its weights if it cannot verify."""
        from transformers import AutoConfig, AutoModelForCausalLM, AutoTokenizer
        config = AutoConfig.from_pretrained(path)
        try:
            tokenizer = AutoTokenizer.from_pretrained(path)
        except Exception:  # noqa: BLE001 - no tokenizer: the config check still runs
            tokenizer = None
        if target_config is not None:
            check_compatible(target_config, target_tokenizer, config, tokenizer)
        model = AutoModelForCausalLM.from_pretrained(path, dtype=dtype).eval()
        if device is not None:
            model.to(device)
        return cls(model, tokenizer, name=str(path))

    def device_bytes(self):
        return sum(t.numel() * t.element_size()
                   for t in list(self.model.parameters()) + list(self.model.buffers())
                   if t.device.type != "meta")

    def reset(self):
        self.cache = None

    def crop(self, length):
        if self.cache is not None and length >= 0:
            self.cache.crop(length)

    def propose(self, sequence, cached, k, sampling, generator=None):
        """``k`` tokens after ``sequence`` (one draft forward each; the last proposal is not fed
        back).  Returns ``(tokens int64 [n], probs [n, V], cached)``."""
        from transformers import DynamicCache
        if self.cache is None:
            self.cache = DynamicCache()
        tokens, probs = [], []
        t0 = time.perf_counter()
        seq = sequence
        with torch.inference_mode():
            for _ in range(k):
                chunk = seq[:, cached:]
                if chunk.shape[1] == 0:
                    break
                logits = self.model(input_ids=chunk, past_key_values=self.cache,
                                    use_cache=True).logits[:, -1]
                cached += chunk.shape[1]
                self.forwards += 1
                dist = sampling.distribution(logits)
                tok = _draw(dist, generator).to(seq.device)
                tokens.append(tok)
                probs.append(dist[0])
                seq = torch.cat([seq, tok.view(1, 1).to(seq.dtype)], dim=1)
        self.seconds += time.perf_counter() - t0
        if not tokens:
            return (torch.zeros(0, dtype=torch.int64, device=sequence.device), None, cached)
        return torch.cat(tokens).to(torch.int64), torch.stack(probs), cached


class SpeculativeDecoder:
    """Draft k, verify in one target pass, repeat (``draft.py:459-592``).

    ``target`` is callable as ``target(input_ids=..., past_key_values=..., use_cache=True)`` and
    returns ``.logits`` -- a transformers model (RW4 or not) or a ``RocketModel``.
    """

    def __init__(self, target, draft, lookahead=4, max_lookahead=8, new_cache=None,
                 eos_token_id=None, on_pass=None):
        self.target = target
        self.draft = draft
        self.max_lookahead = max(1, int(max_lookahead))
        self.lookahead = max(1, min(int(lookahead), self.max_lookahead))
        self.new_cache = new_cache
        if eos_token_id is None:
            self.eos = frozenset()
        elif isinstance(eos_token_id, int):
            self.eos = frozenset({eos_token_id})
        else:
            self.eos = frozenset(int(t) for t in eos_token_id)
        self.on_pass = on_pass
        self.stats = SpeculationStats()

    def adapt(self):
        """Next lookahead from the measured acceptance rate a: about a / (1 - a) proposals."""
        if not self.stats.proposed:
            return self.lookahead
        a = self.stats.acceptance_rate
        want = float(self.max_lookahead) if a >= 1.0 else a / (1.0 - a)
        self.lookahead = max(1, min(self.max_lookahead, int(round(want))))
        return self.lookahead

    def generate(self, input_ids, max_new_tokens, sampling=None, generator=None,
                 past_key_values=None, min_new_tokens=0):
        """The prompt plus up to ``max_new_tokens`` tokens (one sequence).  An end-of-sequence
        token ends the run once at least ``min_new_tokens`` tokens are out (it is not masked
        before that, only not acted on)."""
        from transformers import DynamicCache
        sampling = sampling or SamplingParams()
        if input_ids.shape[0] != 1:
            raise ValueError("speculative decoding runs one sequence at a time")
        if past_key_values is not None:
            cache = past_key_values
        else:
            cache = self.new_cache() if self.new_cache is not None else DynamicCache()
        if not hasattr(cache, "crop"):
            raise TypeError(f"{type(cache).__name__} cannot crop; speculation takes rejected "
                            f"proposals back out of the cache")
        self.draft.reset()
        sequence = input_ids
        prompt = sequence.shape[1]
        cached = int(cache.get_seq_length()) if past_key_values is not None else 0
        if cached > prompt:
            raise ValueError(f"the cache holds {cached} positions, the prompt only {prompt}")
        draft_cached = 0
        emitted = 0
        while emitted < max_new_tokens:
            k = max(0, min(self.lookahead, max_new_tokens - emitted - 1))
            proposals, draft_probs, draft_cached = self.draft.propose(
                sequence, draft_cached, k, sampling, generator)
            n = int(proposals.shape[0])
            pending = sequence[:, cached:]
            candidate = torch.cat([pending, proposals.view(1, -1).to(sequence.dtype)], dim=1)
            t0 = time.perf_counter()
            with torch.inference_mode():
                logits = self.target(input_ids=candidate, past_key_values=cache,
                                     use_cache=True).logits[0, -(n + 1):]
            target_probs = sampling.distribution(logits)
            accepted, corrected = verify(proposals, draft_probs, target_probs, generator)
            self.stats.target_seconds += time.perf_counter() - t0
            self.stats.passes += 1
            self.stats.lookahead_sum += n
            self.stats.proposed += n
            self.stats.accepted += accepted
            new = (proposals[:accepted].tolist() + [corrected])[:max_new_tokens - emitted]
            ends = next((i for i, t in enumerate(new)
                         if t in self.eos and emitted + i + 1 >= min_new_tokens), None) \
                if self.eos else None
            sequence = torch.cat([sequence, torch.tensor([new], dtype=sequence.dtype,
                                                         device=sequence.device)], dim=1)
            emitted += len(new)
            self.stats.emitted += len(new)
            self.stats.draft_seconds = self.draft.seconds
            if self.on_pass is not None:
                self.on_pass(len(new))
            # the pass wrote every candidate position; the rejected proposals come back out
            cached += pending.shape[1] + accepted
            cache.crop(cached)
            draft_cached = min(draft_cached, cached)
            self.draft.crop(draft_cached)
            if ends is not None:
                return sequence[:, :prompt + emitted - len(new) + ends + 1]
            self.adapt()
        return sequence


def resolve_speculation(setting, draft=None, streamed=False):
    """``(enabled, reason)`` for a ``speculative=`` setting (``draft.py:613-656``): never without a
    draft; ``"auto"`` turns it on exactly when the target's weights stream (a pass then costs a
    host->device transfer that k+1 positions share), off when they are resident."""
    if setting not in SPEC_CHOICES:
        raise ValueError(f"speculative must be one of {', '.join(SPEC_CHOICES)}, not {setting!r}")
    if draft is None:
        return False, "no draft model"
    if setting == SPEC_OFF:
        return False, "turned off explicitly"
    if setting == SPEC_ON:
        return True, "turned on explicitly"
    if streamed:
        return True, "the weights stream, so one pass is worth several tokens"
    return False, "the weights are resident; pass speculative='on' to force it"

"""Generate ``reference_spec.npz`` by running the REFERENCE speculative-decoding rules.

Run once in a checkout that has the RocketLLM sources (read-only is fine)::

    python tests/golden/make_spec_golden.py /path/to/RocketLLM

It imports the reference's ``rocketllm/spec/draft.py`` (bound without the package ``__init__``, as
``make_golden.py`` does) and records, on seeded logits, what its ``SamplingParams.distribution``
returns for a greedy and three sampling warps, and what its ``verify`` returns for greedy
proposals (point masses: no randomness is consumed, so the outcome is fixed).
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bind_reference(root):
    for name, sub in (("rocketllm", "rocketllm"), ("rocketllm.spec", "rocketllm/spec"),
                      ("rocketllm.hw", "rocketllm/hw")):
        if name not in sys.modules:
            pkg = types.ModuleType(name)
            pkg.__path__ = [os.path.join(root, sub)]
            sys.modules[name] = pkg
    sys.path.insert(0, root)
    from rocketllm.spec import draft
    return draft


WARPS = {"greedy": dict(do_sample=False), "t07": dict(do_sample=True, temperature=0.7),
         "k5": dict(do_sample=True, temperature=1.3, top_k=5),
         "p08": dict(do_sample=True, temperature=0.9, top_p=0.8)}


def main(root):
    draft = bind_reference(root)
    out = {}
    g = torch.Generator().manual_seed(40)
    logits = torch.randn(6, 50, generator=g) * 3.0
    out["logits"] = logits.numpy()
    for name, kw in WARPS.items():
        out[f"dist.{name}"] = draft.SamplingParams(**kw).distribution(logits).numpy()
    greedy = draft.SamplingParams()
    cases = []
    for c in range(12):
        k = 1 + c % 5
        tl = torch.randn(k + 1, 50, generator=g) * 3.0
        target = greedy.distribution(tl)
        agree = int(torch.randint(0, k + 1, (1,), generator=g))   # first `agree` proposals match
        props = []
        for i in range(k):
            top = int(target[i].argmax())
            props.append(top if i < agree else (top + 1 + i) % 50)
        dq = torch.zeros(k, 50)
        dq[torch.arange(k), torch.tensor(props)] = 1.0
        acc, tok = draft.verify(props, list(dq), list(target))
        out[f"case{c}.target_logits"] = tl.numpy()
        out[f"case{c}.proposals"] = np.array(props, dtype=np.int64)
        out[f"case{c}.result"] = np.array([acc, tok], dtype=np.int64)
        cases.append(c)
    out["cases"] = np.array(cases, dtype=np.int64)
    path = os.path.join(HERE, "reference_spec.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ROCKETLLM_REFERENCE", "."))

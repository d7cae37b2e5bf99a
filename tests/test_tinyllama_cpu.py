"""The TinyLlama RW4 configuration on the CPU: the checkpoint and the CPU decode port against the
reference's own run (``tests/golden/reference_tinyllama_2l.npz``, made by
``tests/golden/make_tinyllama_golden.py``, which ran the reference's ``RocketModel`` on the CPU).

The 2-layer cut of the configuration keeps this in the CPU suite's time; the full 22 layers are
checked the same way against ``reference_tinyllama.npz`` on the GPU (``test_tinyllama_gpu.py``) and
timed by ``bench.py``.  Bars: the checkpoint's RW4 bytes identical (SHA-256) when encoded by the
oracle codec instead of the reference's; the port's greedy tokens identical; its scores within
1e-4 of the reference's (both fp32 on the CPU over the same weights; only thread-count-dependent
summation order differs).
"""
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import cpu_decode
from oracle import rw4_oracle as o
from rocketllm_b200.synthetic import TINYLLAMA, tinyllama_prompt, write_rw4_llama

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "reference_tinyllama_2l.npz")


def oracle_quantize(w):
    packed, scale, zero, padding = o.quantize(w.numpy(), 64, "f32")
    assert padding == 0
    return torch.from_numpy(packed), torch.from_numpy(scale), torch.from_numpy(zero)


def rw4_digest(sd):
    h = hashlib.sha256()
    for name in sorted(sd):
        if name.endswith(("_packed", "_scale", "_zero_point")):
            h.update(name.encode())
            h.update(sd[name].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory, golden):
    path = str(tmp_path_factory.mktemp("tinyllama_2l"))
    sd = write_rw4_llama(path, dict(TINYLLAMA, num_hidden_layers=int(golden["layers"])),
                         oracle_quantize)
    return path, rw4_digest(sd)


def test_checkpoint_bytes_match_the_reference_encoding(checkpoint, golden):
    """The oracle codec encodes the whole checkpoint to the bytes the reference's quantize wrote."""
    assert checkpoint[1] == str(golden["rw4_sha256"])


def test_prompt_is_the_reference_prompt(golden):
    assert np.array_equal(tinyllama_prompt().numpy(), golden["prompt"])


def test_cpu_port_matches_the_reference_decode(checkpoint, golden):
    model = cpu_decode.load_fp32_llama(checkpoint[0])
    n = len(golden["tokens"])
    tokens, scores, rate, prefill, threads = cpu_decode.greedy_decode(
        model, torch.from_numpy(golden["prompt"]), n, threads=os.cpu_count())
    assert np.array_equal(tokens, golden["tokens"])
    ids = golden["top_ids"].astype(np.int64)
    got = np.take_along_axis(scores, ids, axis=1)
    assert np.abs(got - golden["top_values"]).max() <= 1e-4
    assert np.abs(scores[0] - golden["first_scores"]).max() <= 1e-4
    assert np.abs(scores[-1] - golden["last_scores"]).max() <= 1e-4
    assert rate is not None and rate > 0

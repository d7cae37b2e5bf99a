"""The TinyLlama RW4 configuration on the B200 against the reference's own CPU decode of it.

``tests/golden/reference_tinyllama.npz`` holds what the reference's ``RocketModel(device="cpu",
dtype=torch.float32)`` produced on this configuration (22 layers, prompt of 128 ids from seed 1,
32 greedy tokens; made by ``tests/golden/make_tinyllama_golden.py``).  Here the same checkpoint is
rebuilt from the same seed with the library's ``rw4_quantize`` and loaded through the package's
``AutoModel.from_pretrained`` (bf16 on the GPU: the tcgen05 GEMM for the 128-token prompt, the
dequant-GEMV for every decode step), resident and streamed layer by layer from shard files.

Bars.  The checkpoint's RW4 bytes are identical to the reference encoding (SHA-256).  Logits: a
bf16 run cannot come within the north star's 2e-2 of an fp32 run on this 22-layer random-init
model -- the reference's own bf16 path (``RocketModel(dtype=torch.bfloat16)``: weights
``dequantize().to(bfloat16)``, bf16 activations, recorded in the same fixture) lands 0.10-0.13
max-abs from its fp32 run -- so with the reference's tokens fed back (teacher forcing) every
step's scores must stay within the band of bf16 rounding: no further from the fp32 reference than
1.5 times the distance of the reference's own (teacher-forced) bf16 run, on its top-64 entries and
on the full first and last steps (two bf16 implementations that add in different orders land at
comparable, not equal, distances; the measured ratio is printed).  Tokens: the greedy choice equals the fp32
reference's wherever that step's top-1 margin is at least twice the bf16 floor (a narrower margin
is a tie that bf16 rounding may break either way), and free-running greedy tokens are identical
up to the first such near-tie.
"""
import hashlib
import os

import numpy as np
import pytest
import torch

from rocketllm_b200 import kernels
from rocketllm_b200.engine import AutoModel, RocketModel
from rocketllm_b200.synthetic import TINYLLAMA, write_rw4_llama

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "reference_tinyllama.npz")
BAND = 1.5


def gpu_quantize(w):
    packed, scale, zero, padding = kernels.quantize(w.cuda(), 64)
    assert padding == 0
    return packed.cpu(), scale.cpu(), zero.cpu()


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
def checkpoint(tmp_path_factory, cuda):
    path = str(tmp_path_factory.mktemp("tinyllama"))
    sd = write_rw4_llama(path, TINYLLAMA, gpu_quantize)
    digest = rw4_digest(sd)
    del sd
    return path, digest


def forced_run(model, golden):
    """Greedy decode that follows the reference's tokens: a logits processor records each step's
    raw scores, then leaves only the reference's token."""
    from transformers import LogitsProcessor, LogitsProcessorList
    want = torch.from_numpy(golden["tokens"])

    class Force(LogitsProcessor):
        def __init__(self):
            self.scores = []

        def __call__(self, input_ids, scores):
            step = len(self.scores)
            self.scores.append(scores.detach().float().cpu().clone())
            forced = torch.full_like(scores, float("-inf"))
            forced[:, int(want[step])] = 0
            return forced

    f = Force()
    prompt = torch.from_numpy(golden["prompt"]).cuda()
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=len(want), do_sample=False,
                             logits_processor=LogitsProcessorList([f]), eos_token_id=None,
                             pad_token_id=0)
    assert torch.equal(out[0, prompt.shape[1]:].cpu(), want)
    return torch.stack(f.scores)[:, 0].numpy()


def errors(golden, top, first, last):
    return (float(np.abs(top - golden["top_values"]).max()),
            float(np.abs(first - golden["first_scores"]).max()),
            float(np.abs(last - golden["last_scores"]).max()))


def bf16_floor(golden):
    """How far the reference's own bf16 run is from its fp32 run (top-64, first, last)."""
    return errors(golden, golden["bf16_top_values"], golden["bf16_first_scores"],
                  golden["bf16_last_scores"])


def near_tie(golden):
    return 2 * bf16_floor(golden)[0]


def check_against_reference(scores, golden):
    ids = golden["top_ids"].astype(np.int64)
    ours = errors(golden, np.take_along_axis(scores, ids, axis=1), scores[0], scores[-1])
    floor = bf16_floor(golden)
    print("max-abs from the reference's fp32 run (top-64, first, last): here "
          + ", ".join(f"{v:.4g}" for v in ours) + "; the reference's bf16 run "
          + ", ".join(f"{v:.4g}" for v in floor))
    print("ratio to the reference's bf16 distance: "
          + ", ".join(f"{a / b:.3f}" for a, b in zip(ours, floor)))
    assert all(a <= BAND * b for a, b in zip(ours, floor)), (ours, floor)
    clear = golden["margins"] >= near_tie(golden)
    assert clear.any()
    assert np.array_equal(scores.argmax(1)[clear], golden["tokens"][clear])


def check_free_running(model, golden):
    prompt = torch.from_numpy(golden["prompt"]).cuda()
    n = len(golden["tokens"])
    with torch.no_grad():
        out = model.generate(prompt, max_new_tokens=n, do_sample=False, eos_token_id=None,
                             pad_token_id=0)
    got = out[0, prompt.shape[1]:].cpu().numpy()
    diff = np.nonzero(got != golden["tokens"])[0]
    print(f"free-running greedy: {diff[0] if diff.size else n} of {n} tokens equal the reference's")
    if diff.size:
        j = int(diff[0])
        assert golden["margins"][j] < near_tie(golden), \
            f"diverged at step {j}, margin {golden['margins'][j]:.4g}"


def test_checkpoint_bytes_match_the_reference_encoding(checkpoint, golden):
    assert checkpoint[1] == str(golden["rw4_sha256"])


def test_resident_matches_reference_cpu_decode(checkpoint, golden):
    model = AutoModel.from_pretrained(checkpoint[0])
    assert model.streamer is None
    check_against_reference(forced_run(model, golden), golden)
    check_free_running(model, golden)
    assert kernels.device_status() == 0


def test_streamed_from_shards_matches_reference_cpu_decode(checkpoint, golden, tmp_path):
    """Layer-by-layer streaming from shard files on disk, as the configuration runs on the CPU."""
    from rocketllm_b200.shards import split_rw4_layers
    resident = AutoModel.from_pretrained(checkpoint[0])
    shards = split_rw4_layers(resident.model, str(tmp_path / "shards"))
    resident.close()
    model = RocketModel(shards, vram_budget=1, window=2, kv_cache="fp16")
    assert model.streamer is not None
    check_against_reference(forced_run(model, golden), golden)
    model.close()

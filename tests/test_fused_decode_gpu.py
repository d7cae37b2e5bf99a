"""The fused decode step (``rocketllm_b200.fused_decode``: six launches per Llama layer; the same
attention half before the model's own sparse-MoE block on a Mixtral) against the module-by-module
step (``GraphedDecoder``: transformers' modules around the RW4 GEMVs) and against the reference's
own CPU decode of the TinyLlama configuration.

Both steps run the same arithmetic in the same bf16 rounding sequence, but not bit for bit: the
concatenated q|k|v and gate|up weights may split K differently from the separate projections, and
attention reads the static cache through rw4_decode_attention (or SDPA's grouped-query path)
instead of copied keys and values.  So, with the module path's tokens fed back to both (teacher forcing), every step's logits
must agree within the linear tests' bf16 tolerance scaled to the logits, and the greedy choice must
agree wherever the module path's top-1 margin is at least 4e-2.
"""
import os

import numpy as np
import pytest
import torch

from rocketllm_b200 import kernels
from rocketllm_b200.decode import GraphedDecoder
from rocketllm_b200.engine import AutoModel
from rocketllm_b200.fused_decode import FusedDecoder, fusable
from rocketllm_b200.quant.convert import save_rw4_checkpoint

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1536, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                      max_position_embeddings=1024, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():
        for n, p in model.named_parameters():
            p.copy_(torch.ones_like(p) if "norm" in n else torch.randn_like(p) * 0.02)
    return save_rw4_checkpoint(model, str(tmp_path_factory.mktemp("rw4")), device="cuda")


def forced_steps(dec, prompt, tokens):
    """Logits of each decode step with ``tokens`` fed back (the first comes from the prefill)."""
    out = []
    dec.prefill(prompt)
    for t in tokens[:-1]:
        dec.ids.copy_(t.view(-1, 1))
        dec.step()
        out.append(dec.logits.float().clone())
    return torch.stack(out)


@pytest.mark.parametrize("batch,attention", [(1, "rw4"), (3, "rw4"), (3, "sdpa")])
def test_fused_step_matches_module_step(checkpoint, batch, attention):
    model = AutoModel.from_pretrained(checkpoint).model
    assert fusable(model)
    g = torch.Generator().manual_seed(batch)
    prompt = torch.randint(0, 2048, (batch, 37), generator=g).cuda()
    ref_dec = GraphedDecoder(model, batch, 37 + 24 + 8)
    want = ref_dec.generate(prompt, 24)                      # module path, greedy
    ref = forced_steps(GraphedDecoder(model, batch, 37 + 24 + 8), prompt, want.T)
    fdec = FusedDecoder(model, batch, 37 + 24 + 8, attention=attention)
    assert fdec.own_attention == (attention == "rw4")
    fused = forced_steps(fdec, prompt, want.T)
    assert kernels.device_status() == 0
    scale = float(ref.abs().max())
    err = float((fused - ref).abs().max())
    print(f"batch {batch}: max |fused - modules| = {err:.4g} (logits up to {scale:.3g})")
    assert err <= 2e-2 * max(1.0, scale)
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) >= 4e-2
    assert torch.equal(fused.argmax(-1)[clear], ref.argmax(-1)[clear])
    # free-running: the fused decoder's greedy tokens equal the module path's up to a near-tie
    got = FusedDecoder(model, batch, 37 + 24 + 8, attention=attention).generate(prompt, 24)
    for b in range(batch):
        diff = (got[b] != want[b]).nonzero()
        if diff.numel():
            j = int(diff[0, 0])
            assert j > 0 and float(top2[j - 1, b, 0] - top2[j - 1, b, 1]) < 4e-2


@pytest.mark.parametrize("batch", [1, 4])
def test_fused_step_on_a_mixtral_model(batch):
    """A Mixtral-architecture RW4 model: the fused attention half plus the model's own sparse-MoE
    block against the module step, teacher-forced, with the Llama test's bounds.  The router is
    drawn with std 0.5 so that its top-2 margins are wide: the attention half's rounding must not
    flip an expert choice (a flip at a near-tie is legitimate, but it is not what is tested)."""
    from transformers import MixtralConfig

    from rocketllm_b200.synthetic import build_rw4_causal_lm
    cfg = MixtralConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                        num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                        num_local_experts=4, num_experts_per_tok=2, max_position_embeddings=256,
                        tie_word_embeddings=False)
    model = build_rw4_causal_lm(cfg, device="cuda", seed=4)
    with torch.no_grad():
        g = torch.Generator(device="cuda").manual_seed(9)
        for layer in model.model.layers:
            r = layer.mlp.gate.weight
            r.copy_(torch.randn(r.shape, device="cuda", generator=g) * 0.5)
    assert fusable(model)
    prompt = torch.randint(0, 2048, (batch, 29), generator=torch.Generator().manual_seed(batch))
    prompt = prompt.cuda()
    want = GraphedDecoder(model, batch, 29 + 16 + 8).generate(prompt, 16)
    ref = forced_steps(GraphedDecoder(model, batch, 29 + 16 + 8), prompt, want.T)
    fused = forced_steps(FusedDecoder(model, batch, 29 + 16 + 8), prompt, want.T)
    assert kernels.device_status() == 0
    scale = float(ref.abs().max())
    err = float((fused - ref).abs().max())
    print(f"mixtral batch {batch}: max |fused - modules| = {err:.4g} (logits up to {scale:.3g})")
    assert err <= 2e-2 * max(1.0, scale)
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) >= 4e-2
    assert torch.equal(fused.argmax(-1)[clear], ref.argmax(-1)[clear])


def test_fused_step_on_the_reference_configuration():
    """TinyLlama RW4: the fused step, fed the reference's tokens, stays within
    the same 1.5x of the reference's own bf16 distance from its fp32 run as the module path."""
    import tempfile

    from rocketllm_b200.synthetic import TINYLLAMA, write_rw4_llama
    golden = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                       "reference_tinyllama.npz")))

    def q(w):
        p, s, z, _ = kernels.quantize(w.cuda(), 64)
        return p.cpu(), s.cpu(), z.cpu()

    with tempfile.TemporaryDirectory() as tmp:
        write_rw4_llama(tmp, TINYLLAMA, q)
        model = AutoModel.from_pretrained(tmp).model
    prompt = torch.from_numpy(golden["prompt"]).cuda()
    toks = torch.from_numpy(golden["tokens"]).cuda().view(-1, 1)
    dec = FusedDecoder(model, 1, 128 + 32 + 8)
    scores = forced_steps(dec, prompt, toks)[:, 0].cpu().numpy()     # steps 1..31
    ids = golden["top_ids"].astype(np.int64)[1:]
    err_top = float(np.abs(np.take_along_axis(scores, ids, 1) - golden["top_values"][1:]).max())
    err_last = float(np.abs(scores[-1] - golden["last_scores"]).max())
    floor_top = float(np.abs(golden["bf16_top_values"] - golden["top_values"]).max())
    floor_last = float(np.abs(golden["bf16_last_scores"] - golden["last_scores"]).max())
    print(f"fused step vs the reference's fp32 run: top-64 {err_top:.4g} (bf16 floor "
          f"{floor_top:.4g}), last {err_last:.4g} (floor {floor_last:.4g})")
    assert err_top <= 1.5 * floor_top and err_last <= 1.5 * floor_last


def test_generate_takes_the_fused_path_and_matches_transformers(checkpoint):
    """``RocketModel.generate`` for a plain greedy call runs the fused graphed step; its tokens equal
    transformers' own greedy loop over the same model up to the first near-tie, end tokens stop a
    row as there (padding after it), and calls the fused path does not honour fall back."""
    from transformers import LogitsProcessorList
    rm = AutoModel.from_pretrained(checkpoint)
    prompt = torch.randint(0, 2048, (2, 21), generator=torch.Generator().manual_seed(9)).cuda()
    with torch.no_grad():
        fast = rm.generate(prompt, max_new_tokens=20, do_sample=False, eos_token_id=None,
                           pad_token_id=0)
        slow = rm.model.generate(prompt, max_new_tokens=20, do_sample=False, eos_token_id=None,
                                 pad_token_id=0, return_dict_in_generate=True, output_logits=True)
    assert fast.shape == slow.sequences.shape and torch.equal(fast[:, :21], prompt)
    for b in range(2):
        diff = (fast[b] != slow.sequences[b]).nonzero()
        if diff.numel():
            j = int(diff[0, 0]) - 21
            top2 = slow.logits[j][b].float().topk(2).values
            assert float(top2[0] - top2[1]) < 4e-2, f"row {b} diverged at {j}"
    # an end token: make the row's third generated token the end token and rerun
    eos = int(fast[0, 23])
    with torch.no_grad():
        stopped = rm.generate(prompt[:1], max_new_tokens=20, do_sample=False, eos_token_id=eos,
                              pad_token_id=0)
    first = int((stopped[0, 21:] == eos).nonzero()[0, 0])
    assert stopped.shape[1] == 21 + first + 1      # one row: the output ends at its end token
    with torch.no_grad():      # not honoured by the fused path: transformers' loop runs
        out = rm.generate(prompt, max_new_tokens=5, do_sample=False,
                          logits_processor=LogitsProcessorList([]), eos_token_id=None,
                          pad_token_id=0)
    assert out.shape == (2, 26)


@pytest.mark.parametrize("batch", [1, 3])
def test_fused_pipeline_stage_equals_fused_decoder(checkpoint, batch):
    """A pipeline stage owning every layer (one rank) runs the fused ops over its layer range
    (``FusedLayerRange``): the same launches as the fused decoder, so the same tokens and logits
    bit for bit; with ``fused=False`` the stage runs the modules."""
    from rocketllm_b200.pipeline import GraphedPipelineDecoder
    model = AutoModel.from_pretrained(checkpoint).model
    g = torch.Generator().manual_seed(10 + batch)
    prompt = torch.randint(0, 2048, (batch, 29), generator=g).cuda()
    want = FusedDecoder(model, batch, 29 + 20 + 8).generate(prompt, 20)
    stage = GraphedPipelineDecoder(model, batch, 29 + 20 + 8, local=True)
    assert stage.fl is not None
    got = stage.generate(prompt, 20)
    assert kernels.device_status() == 0
    assert torch.equal(got, want)
    mods = GraphedPipelineDecoder(model, batch, 29 + 20 + 8, local=True, fused=False)
    assert mods.fl is None
    ref = mods.generate(prompt, 20)
    assert ref.shape == want.shape and torch.equal(ref[:, :1], want[:, :1])   # one prefill

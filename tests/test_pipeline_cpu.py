"""Pipeline parallelism over two and three gloo ranks on the CPU: splitting the decoder layers and
handing the hidden states rank to rank gives exactly the single-rank greedy tokens.  The model is a
tiny dense fp32 Llama (the pipeline is independent of the Linear implementation; the GPU test runs
it on RW4 weights)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rocketllm_b200.pipeline import layer_range


def tiny_model():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=5,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=97,
                      max_position_embeddings=64, tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" not in n:
                p.normal_(0, 0.2)
    return m


def test_layer_ranges_cover_every_layer_once():
    for layers in (1, 5, 32, 126):
        for world in (1, 2, 3, 8):
            spans = [layer_range(layers, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == layers
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def test_single_rank_decode_matches_generate():
    """The layer-by-layer loop (one rank, no communication) is transformers' own greedy decode."""
    from rocketllm_b200.pipeline import PipelineDecoder
    ids = torch.randint(0, 97, (2, 7), generator=torch.Generator().manual_seed(3))
    m = tiny_model()
    m.generation_config.eos_token_id = None
    m.generation_config.pad_token_id = 0
    with torch.no_grad():
        ref = m.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=6,
                         do_sample=False)[:, 7:]
    got = PipelineDecoder(tiny_model(), device="cpu", local=True).generate(ids, 6)
    assert torch.equal(ref, got), (ref, got)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from rocketllm_b200.pipeline import PipelineDecoder
    ids = torch.randint(0, 97, (2, 7), generator=torch.Generator().manual_seed(3))
    ref = PipelineDecoder(tiny_model(), device="cpu", local=True).generate(ids, 6)
    got = PipelineDecoder(tiny_model(), device="cpu").generate(ids, 6)
    out[rank] = bool(torch.equal(ref, got))
    dist.barrier()
    dist.destroy_process_group()


def _graphed_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from rocketllm_b200.pipeline import GraphedPipelineDecoder, PipelineDecoder
    ids = torch.randint(0, 97, (2, 7), generator=torch.Generator().manual_seed(3))
    ref = PipelineDecoder(tiny_model(), device="cpu", local=True).generate(ids, 6)
    dec = GraphedPipelineDecoder(tiny_model(), batch=2, max_len=16, device="cpu",
                                 use_graph=False)
    got = dec.generate(ids, 6)
    out[rank] = bool(torch.equal(ref, got))
    dist.barrier()
    dist.destroy_process_group()


def test_static_cache_stage_decoder_matches(tmp_path):
    """The static-cache stage decoder (eager stage on CPU) gives the dynamic-cache tokens."""
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_graphed_worker, args=(2, 29721, out), nprocs=2, join=True)
        assert all(out[r] for r in range(2)), dict(out)


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_matches_single_rank(world):
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(world, 29711 + world, out), nprocs=world, join=True)
        assert all(out[r] for r in range(world)), dict(out)


def _int4_model():
    """A bf16 Llama with head_dim 64 (the int4 cache's layout) and room for a flushed group."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=256, num_hidden_layers=4,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=97,
                      max_position_embeddings=256, tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" not in n:
                p.normal_(0, 0.2)
    return m


def _int4_decoder(local):
    from test_kv_cache_cpu import CpuKVOps

    from rocketllm_b200.kv_cache import RW4KVCache, enable_kv_attention
    from rocketllm_b200.pipeline import PipelineDecoder
    m = enable_kv_attention(_int4_model())
    return PipelineDecoder(m, device="cpu", local=local,
                           cache=RW4KVCache(ops=CpuKVOps(), fused=True))


def _int4_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ids = torch.randint(0, 97, (1, 189), generator=torch.Generator().manual_seed(5))
    ref = _int4_decoder(local=True).generate(ids, 8)     # crosses the first flush at 192 tokens
    dec = _int4_decoder(local=False)
    got = dec.generate(ids, 8)
    own = [i for i in range(dec.start, dec.stop)]
    out[rank] = bool(torch.equal(ref, got)) and all(dec.cache._kv[i].groups == 1 for i in own)
    dist.barrier()
    dist.destroy_process_group()


def test_pipeline_with_the_int4_kv_cache_matches_single_rank():
    """Each rank keeps its own layers' int4 cache (fused decode attention, a group flushed during
    the run); the tokens are the single-rank run's."""
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_int4_worker, args=(2, 29731, out), nprocs=2, join=True)
        assert all(out[r] for r in range(2)), dict(out)


def test_fused_stage_only_where_it_applies():
    """The graphed stage takes the fused decode ops only for resident RW4 Llama layers on a CUDA
    device: a plain fp32 model on the CPU runs the modules by default, and asking for the fused
    stage there is an error, not a silent fallback."""
    from rocketllm_b200.fused_decode import fusable_layers
    from rocketllm_b200.pipeline import GraphedPipelineDecoder
    model = tiny_model()
    assert not fusable_layers(model, range(5), True)
    dec = GraphedPipelineDecoder(model, batch=1, max_len=8, device="cpu", local=True,
                                 use_graph=False)
    assert dec.fl is None
    with pytest.raises(ValueError):
        GraphedPipelineDecoder(tiny_model(), batch=1, max_len=8, device="cpu", local=True,
                               fused=True)

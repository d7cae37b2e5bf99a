"""Worker for tests/test_pipeline_gpu.py: run under torchrun, one rank per GPU (NCCL).

Every rank builds the same seeded RW4 Llama-architecture model, decodes it alone (one rank, all
layers) and then as one stage of the pipeline over all ranks; the greedy tokens must be identical,
and the pipeline ranks must hold only their own layers."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    from transformers import LlamaConfig
    from rocketllm_b200 import kernels
    from rocketllm_b200.pipeline import GraphedPipelineDecoder, PipelineDecoder, layer_range
    from rocketllm_b200.synthetic import build_rw4_causal_lm
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    cfg = LlamaConfig(hidden_size=1024, intermediate_size=2816,
                      num_hidden_layers=max(5, world + 1), num_attention_heads=16,
                      num_key_value_heads=4, vocab_size=4096, max_position_embeddings=256,
                      tie_word_embeddings=False)
    ids = torch.randint(0, cfg.vocab_size, (3, 19), generator=torch.Generator().manual_seed(5))
    ref = PipelineDecoder(build_rw4_causal_lm(cfg, device=dev, seed=0, std=0.05), device=dev,
                          local=True).generate(ids, 10)
    pp = PipelineDecoder(build_rw4_causal_lm(cfg, device=dev, seed=0, std=0.05), device=dev)
    got = pp.generate(ids, 10)
    torch.cuda.synchronize()
    start, stop = layer_range(cfg.num_hidden_layers, rank, world)
    kept = sum(not isinstance(layer, torch.nn.Identity) for layer in pp.layers)
    ok = torch.equal(ref, got) and kept == stop - start and kernels.device_status() == 0
    if not ok:
        print(f"rank {rank}: kept {kept} layers, tokens\n{ref}\n{got}", flush=True)
    # static cache + CUDA-graphed stages on a model each rank built only partly (its layers,
    # the embedding on the first rank, the head on the last): the single-rank graphed decode
    gref = GraphedPipelineDecoder(build_rw4_causal_lm(cfg, device=dev, seed=0, std=0.05), 3, 40,
                                  device=dev, local=True).generate(ids, 10)
    stage = build_rw4_causal_lm(cfg, device=dev, seed=0, std=0.05, layers=(start, stop),
                                keep_embed=rank == 0, keep_head=rank == world - 1)
    ggot = GraphedPipelineDecoder(stage, 3, 40, device=dev).generate(ids, 10)
    torch.cuda.synchronize()
    if not torch.equal(gref, ggot):
        ok = False
        print(f"rank {rank}: graphed pipeline tokens\n{gref}\n{ggot}", flush=True)
    f = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(f)
    dist.destroy_process_group()
    if rank == 0:
        print("PP_OK" if int(f) == 0 else f"PP_FAIL {int(f)}", flush=True)
    sys.exit(0 if int(f) == 0 else 1)


if __name__ == "__main__":
    main()

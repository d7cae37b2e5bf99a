"""Benchmark of the RW4 4-bit dequant-GEMV hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rw4|reference]

Workload (the isolated 4-bit dequant-matmul sweep at decode batch M=1): the five RW4 weight shapes
(K, N) = (4096, 4096), (4096, 14336), (14336, 4096), (8192, 28672), (16384, 53248) -- uniform
random codes, scales U[0.005, 0.02], zero = -8 * scale, group 64 -- times a bf16 N(0, 1) activation
row.  One step = one rw4_linear call per shape (five kernel launches).  698 MB of packed weights per
step, so every step streams its inputs from HBM (inputs larger than the 126 MB L2).

Printed metric: whole-job GB/s of algorithmic bytes (codes + fp16 scales + fp16 zeros + x + y,
each counted once).  `roofline` is the dominant launch (16384 x 53248) timed with CUDA events inside
the timed region against the measured HBM copy bandwidth.  `e2e` is the same metric through the
public API with the weights in pinned host memory: every step streams them through the transfer
engine (chunked copies on dedicated copy streams) into two device slots while the GEMV of the
previous weight runs, then reads the outputs back.  `cpu_baseline` / `--impl reference` time the
CPU oracle (the reference's dequantize-then-matmul algorithm) on the host cores over a row sample.

Multi-GPU (torchrun): every rank runs the same workload on its own GPU (weak scaling, no data-path
collective); the step time is the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = ((4096, 4096), (4096, 14336), (14336, 4096), (8192, 28672), (16384, 53248))
M = 1
GROUP = 64
DOMINANT = 4
METRIC = "dequant-GEMV HBM GB/s (4-bit RW4 group 64, decode M=1, isolated sweep shapes)"
FALLBACK_HBM_GBS = 6650.0
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "gemv_traffic.json")


def alg_bytes(m, k, n):
    return n * k // 2 + 2 * 2 * (k // GROUP) * n + 2 * m * k + 2 * m * n


STEP_BYTES = sum(alg_bytes(M, k, n) for k, n in SHAPES)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001 - absent on a box the driver did not prepare
        return FALLBACK_HBM_GBS, "fallback"


def traffic_per_launch():
    try:
        with open(TRAFFIC_FILE) as f:
            rec = json.load(f)
        return float(rec["dram_bytes_per_launch"])
    except Exception:  # noqa: BLE001
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001 - no nvidia-smi: no clock record
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------------
# CPU: the oracle (test infrastructure) as the reported baseline and the reference arm
# ----------------------------------------------------------------------------------------------

def cpu_sample_step(weights, x):
    """Dequantize-then-matmul (fp32) of the sampled rows of every shape: the reference's
    dequant-to-scratch + F.linear, restated in torch on the CPU (``oracle/cpu_decode.py``), on the
    thread count ``run_cpu`` fixed."""
    from oracle import cpu_decode
    for xi, (p, s, z) in zip(x, weights):
        cpu_decode.dequant_linear(xi, p, s, z)


def cpu_workload(rows_per_shape, seed=0):
    from oracle import rw4_oracle as o
    weights, xs, nbytes = [], [], 0
    rng = np.random.default_rng(seed)
    for k, n in SHAPES:
        rows = min(n, rows_per_shape)
        p, s, z = o.synthetic_weight(rows, k, GROUP, seed=seed + k + n)
        weights.append((torch.from_numpy(p), torch.from_numpy(s), torch.from_numpy(z)))
        xs.append(torch.from_numpy(rng.standard_normal((M, k)).astype(np.float32)))
        nbytes += alg_bytes(M, k, rows)
    return weights, xs, nbytes


def run_cpu(steps, warmup, rows_per_shape=None, budget_s=None):
    """Time the CPU port on every host core.  The thread count is set explicitly (torch's intra-op
    pool, whatever OMP_NUM_THREADS a launcher exported), so the figure is the same workload on the
    same threads at every N.  With `budget_s`, the per-step row sample is sized from a calibration
    step so that warmup + steps take about `budget_s` seconds."""
    threads = os.cpu_count() or 1
    before = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        if budget_s is not None:
            weights, xs, _ = cpu_workload(512)
            cpu_sample_step(weights, xs)
            t0 = time.perf_counter()
            cpu_sample_step(weights, xs)
            per_row = (time.perf_counter() - t0) / 512
            rows_per_shape = int(max(64, min(16384, budget_s / max(1, steps + warmup) / per_row)))
        weights, xs, nbytes = cpu_workload(rows_per_shape)
        for _ in range(warmup):
            cpu_sample_step(weights, xs)
        t0 = time.perf_counter()
        for _ in range(steps):
            cpu_sample_step(weights, xs)
        dt = (time.perf_counter() - t0) / steps
    finally:
        torch.set_num_threads(before)
    sample = (f"dequantize + fp32 F.linear of {rows_per_shape} sampled rows of each of the five "
              f"shapes at M=1 ({nbytes / 1e6:.2f} MB algorithmic per step), torch port of the "
              f"reference's dequant-to-scratch path, {threads} threads set explicitly")
    return nbytes / dt / 1e9, dt * 1e3, threads, sample


def reference_arm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    value, ms, threads, sample = run_cpu(args.steps, args.warmup, budget_s=90.0)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_block(),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def config_block():
    return {"workload": "isolated 4-bit dequant-matmul sweep, decode M=1, five weight shapes per "
                        "step",
            "shapes_kn": [list(s) for s in SHAPES], "M": M, "group": GROUP,
            "weights": "uniform random codes, scale U[0.005,0.02], zero=-8*scale",
            "activations": "bf16 N(0,1)",
            "l2": "inputs larger than L2 (698 MB of weights per step, no flush needed)",
            "launch": "each step replays two CUDA graphs (four shapes, then the dominant one) of "
                      "rw4_linear launches captured from the public API"}


# ----------------------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------------------

def h2d_probe(device, nbytes=256 << 20, reps=10):
    """Best-of-N pinned host->device copy bandwidth (the method of the reference's profile
    probe, rocketllm/hw/profile.py:245-269, with more iterations)."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return best


LLAMA_8B = dict(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                num_attention_heads=32, num_key_value_heads=8, vocab_size=128256,
                max_position_embeddings=8192, rope_theta=500000.0, tie_word_embeddings=False)


LLAMA_405B = dict(hidden_size=16384, intermediate_size=53248, num_hidden_layers=126,
                  num_attention_heads=128, num_key_value_heads=8, vocab_size=128256,
                  max_position_embeddings=8192, rope_theta=500000.0, tie_word_embeddings=False)


def pp_decode(args):
    """Pipeline-parallel greedy decode (not the driver's line): the model's decoder layers split
    over the ranks (contiguous ranges; each rank builds only its own layers), hidden states handed
    rank to rank over NCCL (NVLink), every rank's per-token stage replayed from a CUDA graph.
    Default: the Llama-3.1-405B architecture in RW4 (several GPUs), batch 1 and 32, prompt
    1024, 64 new tokens.  Prints one JSON line on rank 0; timings are CUDA events, max over
    ranks."""
    import datetime

    import torch.distributed as dist
    from transformers import LlamaConfig

    from rocketllm_b200.pipeline import GraphedPipelineDecoder, layer_range
    from rocketllm_b200.synthetic import build_rw4_causal_lm
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    spec = dict(LLAMA_405B if args.pp_model == "405b" else LLAMA_8B)
    if args.pp_layers:
        spec["num_hidden_layers"] = args.pp_layers
    cfg = LlamaConfig(**spec)
    n_layers = cfg.num_hidden_layers
    start, stop = layer_range(n_layers, rank, world)
    t0 = time.time()
    model = build_rw4_causal_lm(cfg, device=device, seed=0, layers=(start, stop),
                                keep_embed=rank == 0, keep_head=rank == world - 1)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    out = {"mode": "pipeline-parallel greedy decode", "model":
           f"Llama-3.1-{args.pp_model.upper()} architecture ({n_layers} layers), RW4 group 64, "
           "random init N(0,0.02)", "data": "synthetic", "n_gpus": world,
           "layers_per_rank": [list(layer_range(n_layers, r, world)) for r in range(world)],
           "prompt_tokens": args.pp_prompt, "new_tokens": args.pp_tokens,
           "rank0_weight_bytes": weight_bytes, "rank0_build_s": round(build_s, 1)}

    def worst(v):
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for b in tuple(int(v) for v in args.pp_batches.split(",")):
        dec = GraphedPipelineDecoder(model, b, args.pp_prompt + args.pp_tokens + 8, device=device)
        ids = torch.randint(0, cfg.vocab_size, (b, args.pp_prompt),
                            generator=torch.Generator().manual_seed(1))
        dist.barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        dec.prefill(ids)
        a1.record()
        for _ in range(3):   # capture + warm-up replays
            dec.step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.pp_tokens):
            dec.step()
        e1.record()
        torch.cuda.synchronize()
        ms = worst(e0.elapsed_time(e1) / args.pp_tokens)
        out[f"b{b}"] = {"tok_s": round(b * 1000.0 / ms, 2), "ms_per_token": round(ms, 3),
                        "prefill_ms": round(worst(a0.elapsed_time(a1)), 1)}
        del dec
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


MIXTRAL_8X7B = dict(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                    num_attention_heads=32, num_key_value_heads=8, vocab_size=32000,
                    num_local_experts=8, num_experts_per_tok=2, max_position_embeddings=4096,
                    rope_theta=1000000.0, tie_word_embeddings=False)


def moe_decode(args):
    """Mixtral-8x7B-architecture RW4 greedy decode with routed experts streamed one by one from
    pinned host memory into an expert cache (a separate line from the headline one): random
    init N(0, 0.02) incl. the router, prompt ``--moe-prompt``, ``--moe-tokens`` new tokens per
    batch size, under ``--moe-budget-gb`` of VRAM.  Prints one JSON line."""
    from transformers import MixtralConfig

    from rocketllm_b200.decode import GraphedDecoder
    from rocketllm_b200.engine import RocketModel
    from rocketllm_b200.synthetic import build_rw4_causal_lm
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = MixtralConfig(**MIXTRAL_8X7B)
    t0 = time.time()
    model = build_rw4_causal_lm(cfg, device=device, seed=0)
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    streamed = RocketModel(model, device=device, vram_budget=int(args.moe_budget_gb * 1e9),
                           window=2, kv_cache="fp16", expert_routing=args.moe_routing,
                           expert_policy=args.expert_policy)
    del model
    torch.cuda.empty_cache()
    setup_s = time.time() - t0
    st = streamed.streamer
    out = {"mode": "streamed mixture-of-experts greedy decode",
           "model": "Mixtral-8x7B architecture, RW4 group 64 (random init N(0,0.02))",
           "data": "synthetic", "weight_bytes": weight_bytes,
           "vram_budget_bytes": int(args.moe_budget_gb * 1e9),
           "pinned_layers": st.pinned, "streamed_layers": st.streamed,
           "expert_routing": args.moe_routing,
           "expert_policy": st.experts.stats()["policy"] if st.experts else None,
           "expert_slots": st.experts.stats()["expert_slots"] if st.experts else 0,
           "expert_blob_bytes": st.experts.stats()["slot_bytes"] if st.experts else 0,
           "prompt_tokens": args.moe_prompt, "setup_s": round(setup_s, 1)}
    gen = torch.Generator().manual_seed(1)
    for b in tuple(int(v) for v in args.moe_batches.split(",")):
        ids = torch.randint(0, cfg.vocab_size, (b, args.moe_prompt), generator=gen).to(device)
        dec = GraphedDecoder(streamed.model, b, args.moe_prompt + args.moe_tokens + 8,
                             device=device, use_graph=False)
        p0 = time.time()
        dec.prefill(ids)
        dec.step()
        torch.cuda.synchronize()
        prefill_s = time.time() - p0
        s0 = st.stats()
        e0 = st.experts.stats() if st.experts else {"bytes": 0, "fetches": 0, "hits": 0}
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.moe_tokens):
            dec.step()
        c.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(c) / args.moe_tokens
        s1 = st.stats()
        e1 = st.experts.stats() if st.experts else {"bytes": 0, "fetches": 0, "hits": 0}
        layer_bytes = (s1["bytes"] - s0["bytes"]) / args.moe_tokens
        expert_bytes = (e1["bytes"] - e0["bytes"]) / args.moe_tokens
        out[f"b{b}"] = {"tok_s": round(b * 1000.0 / ms, 2), "ms_per_token": round(ms, 2),
                        "prefill_s": round(prefill_s, 2),
                        "h2d_bytes_per_token": int(layer_bytes + expert_bytes),
                        "expert_bytes_per_token": int(expert_bytes),
                        "h2d_gbs": round((layer_bytes + expert_bytes) / (ms * 1e-3) / 1e9, 2),
                        "expert_fetches": e1["fetches"] - e0["fetches"],
                        "expert_hits": e1["hits"] - e0["hits"]}
        del dec
        torch.cuda.empty_cache()
    out["h2d_probe_gbs"] = round(h2d_probe(device), 2)
    routing = st.experts.stats().get("routing") if st.experts is not None else None
    if isinstance(routing, dict):
        # lifetime routing skew over the whole run (prefills included; host routing only)
        out["routing"] = {k: round(v, 4) if isinstance(v, float) else v
                          for k, v in routing.items()}
    print(json.dumps(out), flush=True)
    streamed.close()
    return 0


def ep_decode(args):
    """Expert-parallel greedy decode over the torchrun ranks (not the driver's line): the
    Mixtral-8x7B architecture in RW4 with its routed experts split E/G per rank (NCCL all-to-all
    dispatch and return in every MoE layer), attention replicated, every rank decoding its own
    batch.  Eager steps (the exchange sizes are read on the host).  One JSON line on rank 0;
    throughput summed over ranks, step time the slowest rank's."""
    import datetime

    import torch.distributed as dist
    from transformers import MixtralConfig

    from rocketllm_b200.expert_parallel import enable_expert_parallel
    from rocketllm_b200.pipeline import PipelineDecoder
    from rocketllm_b200.synthetic import build_rw4_causal_lm
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    cfg = MixtralConfig(**MIXTRAL_8X7B)
    model = build_rw4_causal_lm(cfg, device=device, seed=0)
    enable_expert_parallel(model, fixed_capacity=args.ep_graph)
    torch.cuda.empty_cache()
    out = {"mode": "expert-parallel greedy decode" + (
               ", fixed-capacity exchange, CUDA-graphed steps" if args.ep_graph else ""),
           "model": "Mixtral-8x7B architecture, RW4 group 64 (random init N(0,0.02))",
           "data": "synthetic", "n_gpus": world, "experts_per_rank": 8 // world,
           "rank0_weight_bytes": sum(p.numel() * p.element_size() for p in model.parameters()),
           "prompt_tokens": args.moe_prompt, "new_tokens": args.moe_tokens}

    def reduce(v, op):
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=op)
        return float(t.item())

    from rocketllm_b200.decode import GraphedDecoder
    for b in tuple(int(v) for v in args.moe_batches.split(",")):
        ids = torch.randint(0, cfg.vocab_size, (b, args.moe_prompt),
                            generator=torch.Generator().manual_seed(100 + rank))
        dist.barrier()
        if args.ep_graph:
            dec = GraphedDecoder(model, b, args.moe_prompt + args.moe_tokens + 8, device=device)
            dec.prefill(ids)
            for _ in range(3):   # capture (collectives inside the graph) + warm-up replays
                dec.step()
            step = dec.step
        else:
            dec = PipelineDecoder(model, device=device, local=True, drop_remote=False)
            tok = dec._forward(ids, b, args.moe_prompt)    # prefill
            tok = dec._forward(tok, b, 1)                   # one warm-up step
            state = {"tok": tok}

            def step():
                state["tok"] = dec._forward(state["tok"], b, 1)
        torch.cuda.synchronize()
        dist.barrier()
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.moe_tokens):
            step()
        c.record()
        torch.cuda.synchronize()
        ms = reduce(a.elapsed_time(c) / args.moe_tokens, dist.ReduceOp.MAX)
        out[f"b{b}_per_rank"] = {"tok_s": round(world * b * 1000.0 / ms, 2),
                                 "ms_per_token": round(ms, 2)}
        del dec, step   # a graph holding NCCL calls goes before the process group
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def _timed_streamed_decode(streamed, vocab, gen, device, tokens, prompt=128, batch=1):
    """ms per token and streamed bytes per token of ``tokens`` greedy steps at ``batch`` after a
    ``prompt``-token prompt (eager steps: the streaming hooks run every token)."""
    from rocketllm_b200.decode import GraphedDecoder
    ids = torch.randint(0, vocab, (batch, prompt), generator=gen).to(device)
    dec = GraphedDecoder(streamed.model, batch, prompt + tokens + 8, device=device,
                         use_graph=False)
    dec.prefill(ids)
    dec.step()
    torch.cuda.synchronize()
    st0 = streamed.stats()["streaming"]
    a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(tokens):
        dec.step()
    c.record()
    torch.cuda.synchronize()
    st1 = streamed.stats()["streaming"]
    del dec
    return a.elapsed_time(c) / tokens, st0, st1


def decode_bench(device, prompt, new_tokens, batches, stream_tokens, vram_budget,
                 storage_dir=None, host_budget=None, profile_window=False, stream_prompt=128,
                 stream_batches=(1,)):
    """Greedy decode tok/s of a Llama-3.1-8B-architecture RW4 model (random init N(0, 0.02),
    every Linear incl. lm_head in RW4): resident with a CUDA-graphed step, then streamed from
    pinned host memory under a VRAM budget, then (with ``storage_dir``) from layer shards written
    there, with only ``host_budget`` bytes of layer blobs in host memory and the rest read from
    the files every token (the storage tier)."""
    from transformers import LlamaConfig

    from rocketllm_b200.decode import GraphedDecoder
    from rocketllm_b200.engine import RocketModel
    from rocketllm_b200.synthetic import build_rw4_causal_lm

    from rocketllm_b200.fused_decode import FusedDecoder, fusable

    cfg = LlamaConfig(**LLAMA_8B)
    model = build_rw4_causal_lm(cfg, device=device, seed=0)
    step_cls = FusedDecoder if fusable(model) else GraphedDecoder
    out = {"model": "Llama-3.1-8B architecture, RW4 group 64 (random init N(0,0.02))",
           "prompt_tokens": prompt, "greedy": True,
           "resident_step": "fused (rocketllm_b200.fused_decode), CUDA graph"
           if step_cls is FusedDecoder else "transformers modules, CUDA graph"}
    gen = torch.Generator().manual_seed(1)
    if step_cls is FusedDecoder:
        # the module-by-module graphed step, for comparison (batch 1, 64 tokens)
        ids = torch.randint(0, cfg.vocab_size, (1, prompt), generator=gen).to(device)
        dec = GraphedDecoder(model, 1, prompt + 64 + 8, device=device)
        dec.prefill(ids)
        dec.capture()
        for _ in range(3):
            dec.step()
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(64):
            dec.step()
        c.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(c) / 64
        out["resident_b1_modules"] = {"tok_s": round(1000.0 / ms, 1), "ms_per_token": round(ms, 4),
                                      "decode_tokens": 64}
        del dec
        torch.cuda.empty_cache()
    for b in batches:
        ids = torch.randint(0, cfg.vocab_size, (b, prompt), generator=gen).to(device)
        dec = step_cls(model, b, prompt + new_tokens + 8, device=device)  # + 3 warm-up steps
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        dec.prefill(ids)
        t1.record()
        dec.capture()
        for _ in range(3):
            dec.step()
        if profile_window:   # the timed steps alone, for `ncu --profile-from-start off`
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(new_tokens):
            dec.step()
        c.record()
        torch.cuda.synchronize()
        if profile_window:
            torch.cuda.cudart().cudaProfilerStop()
        ms = a.elapsed_time(c) / new_tokens
        out[f"resident_b{b}"] = {"tok_s": round(b * 1000.0 / ms, 1), "ms_per_token": round(ms, 4),
                                 "prefill_ms": round(t0.elapsed_time(t1), 2),
                                 "decode_tokens": new_tokens}
        del dec
        torch.cuda.empty_cache()
    if stream_tokens <= 0:
        del model
        torch.cuda.empty_cache()
        return out
    # streamed: the decoder layers leave HBM and stream from pinned host RAM every token
    streamed = RocketModel(model, device=device, vram_budget=vram_budget, window=2,
                           kv_cache="fp16")
    for b in stream_batches:
        ms, st0, st1 = _timed_streamed_decode(streamed, cfg.vocab_size, gen, device,
                                              stream_tokens, stream_prompt, b)
        nbytes = (st1["bytes"] - st0["bytes"]) / stream_tokens
        out[f"streamed_b{b}"] = {"tok_s": round(b * 1000.0 / ms, 2), "ms_per_token": round(ms, 3),
                                 "vram_budget_bytes": vram_budget,
                                 "window": streamed.streamer.window,
                                 "pinned_layers": streamed.streamer.pinned,
                                 "streamed_layers": streamed.streamer.streamed,
                                 "h2d_bytes_per_token": int(nbytes),
                                 "h2d_gbs": round(nbytes / (ms * 1e-3) / 1e9, 2),
                                 "prompt_tokens": stream_prompt, "decode_tokens": stream_tokens}
    streamed.close()
    del streamed
    if storage_dir is not None:
        from rocketllm_b200.shards import split_rw4_layers
        split_rw4_layers(model, storage_dir)
        del model
        torch.cuda.empty_cache()
        stored = RocketModel(storage_dir, device=device, vram_budget=vram_budget, window=2,
                             kv_cache="fp16", host_budget=host_budget)
        ms, st0, st1 = _timed_streamed_decode(stored, cfg.vocab_size, gen, device,
                                              stream_tokens)
        s0, s1 = st0["storage"] or {}, st1["storage"] or {}
        disk = (s1.get("bytes", 0) - s0.get("bytes", 0)) / stream_tokens
        h2d = (st1["bytes"] - st0["bytes"]) / stream_tokens
        out["storage_b1"] = {"tok_s": round(1000.0 / ms, 2), "ms_per_token": round(ms, 3),
                             "host_budget_bytes": host_budget,
                             "storage_layers": len(stored.streamer.storage.order)
                             if stored.streamer.storage else 0,
                             "storage_bytes_per_token": int(disk),
                             "storage_gbs": round(disk / (ms * 1e-3) / 1e9, 2),
                             "h2d_bytes_per_token": int(h2d),
                             "reads_waited": s1.get("waits", 0) - s0.get("waits", 0),
                             "io_workers": stored.shards.io_workers,
                             "decode_tokens": stream_tokens}
        # the storage tier's roofline on this box: the same reader (positioned reads, O_DIRECT
        # where the file system takes it, io_workers stretches) over the storage-tier layers'
        # files, alone
        order = stored.streamer.storage.order if stored.streamer.storage else []
        if order:
            sizes = [stored.shards.plan(i)[1] for i in order]
            buf = torch.empty(max(sizes), dtype=torch.uint8).pin_memory()
            t0 = time.perf_counter()
            for i in order:
                stored.shards.read_into(i, buf)
            dt = time.perf_counter() - t0
            out["storage_b1"]["read_probe_gbs"] = round(sum(sizes) / dt / 1e9, 2)
            out["storage_b1"]["read_probe_note"] = (
                "the storage-tier layers read once by the package's reader alone; the decode's "
                "storage_gbs against it is the tier's fraction of this box's read rate")
        stored.close()
        del stored
    else:
        del model
    torch.cuda.empty_cache()
    return out


def partitioned_decode(device, dist, batch=32, prompt=512, tokens=32, profile_window=False):
    """Greedy decode of the Mixtral-8x7B architecture in RW4 (random init N(0, 0.02), router
    N(0, 0.02): near-uniform routing) at ``batch`` sequences per GPU after a ``prompt``-token prompt,
    every step a CUDA graph: one GPU holds the whole model (routed experts run by the grouped RW4
    GEMV, no exchange); on G > 1 GPUs the 8 experts of every layer are split 8/G per rank and each
    MoE layer exchanges its rows with a fixed-capacity NCCL all-to-all (out and back) inside the
    graph, attention and the router replicated, every rank decoding its own batch.  Throughput is
    summed over ranks, the step time is the slowest rank's (CUDA events)."""
    from transformers import MixtralConfig

    from rocketllm_b200.decode import GraphedDecoder
    from rocketllm_b200.expert_parallel import enable_expert_parallel
    from rocketllm_b200.fused_decode import FusedDecoder, fusable
    from rocketllm_b200.synthetic import build_rw4_causal_lm

    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    cfg = MixtralConfig(**MIXTRAL_8X7B)
    model = build_rw4_causal_lm(cfg, device=device, seed=0)
    if world > 1:
        enable_expert_parallel(model, fixed_capacity=True)
    torch.cuda.empty_cache()
    ids = torch.randint(0, cfg.vocab_size, (batch, prompt),
                        generator=torch.Generator().manual_seed(100 + rank))
    if dist is not None:
        dist.barrier()
    fused = fusable(model)
    dec = (FusedDecoder if fused else GraphedDecoder)(model, batch, prompt + tokens + 8,
                                                      device=device)
    dec.prefill(ids)
    for _ in range(3):   # capture (with the exchange's collectives inside) + warm-up replays
        dec.step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if profile_window:   # the timed steps alone, for `ncu --profile-from-start off`
        torch.cuda.cudart().cudaProfilerStart()
    a.record()
    for _ in range(tokens):
        dec.step()
    c.record()
    torch.cuda.synchronize()
    if profile_window:
        torch.cuda.cudart().cudaProfilerStop()
    ms = a.elapsed_time(c) / tokens
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del dec   # a graph holding NCCL calls goes before the process group
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    del model
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    h = cfg.hidden_size
    rows = batch * cfg.num_experts_per_tok
    return {"model": "Mixtral-8x7B architecture, RW4 group 64 (random init N(0,0.02))",
            "mode": "resident, grouped RW4 GEMV" if world == 1 else
                    "expert-parallel: 8/G experts per rank, fixed-capacity NCCL all-to-all out "
                    "and back per MoE layer inside the CUDA-graphed step",
            "step": "fused attention half + the model's sparse-MoE block (rocketllm_b200."
                    "fused_decode), CUDA graph" if fused else "transformers modules, CUDA graph",
            "n_gpus": world, "batch_per_gpu": batch, "prompt_tokens": prompt,
            "decode_tokens": tokens, "tok_s": round(world * batch * 1000.0 / ms, 1),
            "ms_per_token": round(ms, 3), "weight_bytes_per_gpu": weight_bytes,
            "exchange_bytes_per_token_per_gpu": 0 if world == 1 else
            2 * cfg.num_hidden_layers * (world - 1) * rows * h * 2,
            "scaling": "weak (fixed batch per GPU)"}


def tinyllama_bench(device, with_cpu, new_tokens=32):
    """The TinyLlama-1.1B RW4 configuration (22 layers, prompt of 128 ids from CPU seed 1, greedy
    decode with the KV cache): the configuration the reference's own CPU path is compared on.

    The checkpoint is rebuilt from its seed (weights N(0, 0.02) from CPU seed 0, encoded by
    ``rw4_quantize``).  GPU: the package's model (``AutoModel.from_pretrained``, bf16, resident),
    timed as the reference's harness times decode -- logits-processor marks around ``generate``
    (``tests/bench_streaming.py:474-502``) -- and as the CUDA-graphed step.  CPU (rank 0, one GPU):
    the port of the reference's path (``oracle/cpu_decode.py``: the reference codec's fp32 weights
    in transformers' Llama, every layer resident) on all of this host's cores.  The GPU figures:
    the fused decode step in a CUDA graph, the public ``generate()`` call as a whole (it takes
    that step), and transformers' own loop over the modules (logits-processor marks).  Each run's greedy
    tokens are compared with the reference's own (``tests/golden/reference_tinyllama.npz``, which
    also records the reference's decode rate where it was made)."""
    from transformers import LogitsProcessor, LogitsProcessorList

    from rocketllm_b200 import kernels
    from rocketllm_b200.decode import GraphedDecoder
    from rocketllm_b200.engine import AutoModel
    from rocketllm_b200.synthetic import TINYLLAMA, write_rw4_llama

    golden = dict(np.load(os.path.join(ROOT, "tests", "golden", "reference_tinyllama.npz")))
    ref_tokens = golden["tokens"][:new_tokens]
    prompt = torch.from_numpy(golden["prompt"])

    def agree(tokens):
        diff = np.nonzero(np.asarray(tokens)[:len(ref_tokens)] != ref_tokens)[0]
        return int(diff[0]) if diff.size else len(ref_tokens)

    def quantize_on_gpu(w):
        packed, scale, zero, _ = kernels.quantize(w.to(device), 64)
        return packed.cpu(), scale.cpu(), zero.cpu()

    class Marks(LogitsProcessor):
        def __init__(self):
            self.times = []

        def __call__(self, input_ids, scores):
            torch.cuda.synchronize()
            self.times.append(time.perf_counter())
            return scores

    out = {"model": "TinyLlama-1.1B architecture, RW4 group 64 (random init N(0,0.02), seed 0)",
           "prompt_tokens": int(prompt.shape[1]), "decode_tokens": new_tokens, "greedy": True,
           "reference_tokens": "tests/golden/reference_tinyllama.npz"}
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "tinyllama_rw4")
        write_rw4_llama(path, TINYLLAMA, quantize_on_gpu)
        model = AutoModel.from_pretrained(path)
        ids = prompt.to(device)
        with torch.no_grad():
            # transformers' own loop over the modules, timed as the reference's harness times it
            # (a logits processor, which also keeps generate() off the fused path)
            model.generate(ids, max_new_tokens=4, do_sample=False, eos_token_id=None,
                           pad_token_id=0, logits_processor=LogitsProcessorList([Marks()]))
            marks = Marks()
            model.generate(ids, max_new_tokens=new_tokens, do_sample=False,
                           logits_processor=LogitsProcessorList([marks]),
                           eos_token_id=None, pad_token_id=0)
            eager = (len(marks.times) - 1) / (marks.times[-1] - marks.times[0])
            # the public generate() (fused, graphed step): whole call, prefill and capture included
            model.generate(ids, max_new_tokens=4, do_sample=False, eos_token_id=None,
                           pad_token_id=0)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            seq = model.generate(ids, max_new_tokens=new_tokens, do_sample=False,
                                 eos_token_id=None, pad_token_id=0)
            torch.cuda.synchronize()
            call_s = time.perf_counter() - t0
        gpu_tokens = seq[0, prompt.shape[1]:].cpu().numpy()
        from rocketllm_b200.fused_decode import FusedDecoder
        dec = FusedDecoder(model.model, 1, prompt.shape[1] + new_tokens + 8, device=device)
        dec.prefill(ids)
        dec.capture()
        for _ in range(3):
            dec.step()
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(new_tokens):
            dec.step()
        c.record()
        torch.cuda.synchronize()
        graphed_ms = a.elapsed_time(c) / new_tokens
        del dec
        out["gpu"] = {"tok_s": round(1000.0 / graphed_ms, 1),
                      "timing": "fused decode step in a CUDA graph (CUDA events)",
                      "ms_per_token": round(graphed_ms, 4),
                      "generate_call_s": round(call_s, 4),
                      "generate_tok_s": round(new_tokens / call_s, 1),
                      "generate_note": "the public generate(): prefill, graph capture and all "
                                       f"{new_tokens} steps in one call",
                      "modules_eager_tok_s": round(eager, 2),
                      "modules_eager_timing": "transformers' loop over the modules, "
                                              "logits-processor marks",
                      "tokens_equal_reference": agree(gpu_tokens)}
        model.close()
        del model
        torch.cuda.empty_cache()
        if with_cpu:
            from oracle import cpu_decode
            cores = os.cpu_count() or 1
            cpu_model = cpu_decode.load_fp32_llama(path)
            tokens, _, rate, prefill, threads = cpu_decode.greedy_decode(cpu_model, prompt,
                                                                         new_tokens, cores)
            out["cpu_port"] = {"tok_s": round(rate, 3), "cores": threads, "kind": "port",
                               "prefill_s": round(prefill, 2),
                               "tokens_equal_reference": agree(tokens),
                               "sample": f"the whole {new_tokens}-token greedy decode after the "
                                         f"128-token prompt, fp32, every layer resident"}
            del cpu_model
            out["gpu_over_cpu_port"] = round(1000.0 / graphed_ms / rate, 1)
    out["reference_cpu_where_recorded"] = {
        "tok_s": round(float(golden["decode_tok_s"]), 3), "threads": int(golden["threads"]),
        "note": "the reference's own RocketModel(device='cpu', fp32) in the container that made "
                "the fixture (its per-layer shards, streaming hooks and dequant-to-scratch seam); "
                "its code does not travel to the GPU box"}
    return out


def rw4_arm(args):
    from rocketllm_b200 import kernels
    from rocketllm_b200.streaming import WeightTransfer
    from rocketllm_b200.synthetic import make_activation, make_weight

    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)

    def barrier():
        if dist is not None:
            dist.barrier()

    weights = [make_weight(n, k, device=device, seed=10 * i + rank) for i, (k, n) in
               enumerate(SHAPES)]
    xs = [make_activation(M, k, device=device, seed=100 + i) for i, (k, n) in enumerate(SHAPES)]
    ys = [torch.empty(M, n, dtype=torch.bfloat16, device=device) for k, n in SHAPES]

    def launch(i):
        kernels.linear(xs[i], *weights[i], out=ys[i])

    # warm-up eagerly (sets every kernel's launch attributes), then capture the step as two CUDA
    # graphs -- the four other shapes, and the dominant launch alone -- so that the timed region
    # replays them with events on the launching stream around the dominant kernel
    for _ in range(args.warmup):
        for i in range(len(SHAPES)):
            launch(i)
    torch.cuda.synchronize()
    if kernels.device_status():
        raise RuntimeError("a kernel reported a timed-out wait during warm-up")
    g_rest, g_dom = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_rest):
        for i in range(len(SHAPES)):
            if i != DOMINANT:
                launch(i)
    with torch.cuda.graph(g_dom):
        launch(DOMINANT)
    for _ in range(3):
        g_rest.replay()
        g_dom.replay()
    torch.cuda.synchronize()

    dom = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.25)  # let the sampler start before the timed region
    start.record()
    for s in range(args.steps):
        g_rest.replay()
        dom[s][0].record()
        g_dom.replay()
        dom[s][1].record()
    end.record()
    torch.cuda.synchronize()
    barrier()
    clock = clocks.stop()
    ms_step = start.elapsed_time(end) / args.steps
    dom_ms = sum(a.elapsed_time(b) for a, b in dom) / args.steps
    if dist is not None:
        t = torch.tensor([ms_step], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())
    del g_rest, g_dom

    status = kernels.device_status()

    # ---- end to end: weights streamed from pinned host memory each step ----
    host_w = [tuple(t.cpu().pin_memory() for t in w) for w in weights]
    host_x = [x.cpu().pin_memory() for x in xs]
    host_y = [torch.empty(M, n, dtype=torch.bfloat16).pin_memory() for k, n in SHAPES]
    xfer = WeightTransfer(device=device, copy_streams=2, chunk_bytes=16 << 20)
    cap = [max(hw[i].numel() * hw[i].element_size() for hw in host_w) for i in range(3)]
    slots = [[torch.empty(c, dtype=torch.uint8, device=device) for c in cap] for _ in range(2)]
    dev_x = [torch.empty_like(x) for x in xs]
    compute = torch.cuda.current_stream()

    def e2e_step():
        for i, (k, n) in enumerate(SHAPES):
            dev_x[i].copy_(host_x[i], non_blocking=True)
            slot = slots[i % 2]
            views = []
            for j, t in enumerate(host_w[i]):
                nb = t.numel() * t.element_size()
                dst = slot[j][:nb]
                h = xfer.send_buffer(t.view(torch.uint8).view(-1), out=dst, after=compute)
                h.resolve(compute)
                views.append(dst.view(t.dtype).view(t.shape))
            kernels.linear(dev_x[i], *views, out=ys[i])
            host_y[i].copy_(ys[i], non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e2e_steps):
        e2e_step()
    b.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = a.elapsed_time(b) / e2e_steps
    if dist is not None:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = sum(sum(t.numel() * t.element_size() for t in hw) for hw in host_w) + sum(
        x.numel() * 2 for x in host_x)
    d2h = sum(y.numel() * 2 for y in host_y)
    h2d_peak = h2d_probe(device) if rank == 0 else None
    xfer.close()

    decode = None
    if not args.no_decode:
        del weights, host_w, slots
        torch.cuda.empty_cache()
        decode = decode_bench(device, args.decode_prompt, args.decode_tokens,
                              tuple(int(b) for b in args.decode_batches.split(",")),
                              args.stream_tokens, int(4e9))
        if dist is not None:
            # every rank decodes its own model copy (data-parallel replicas, no exchange): the
            # job's throughput is the sum over ranks, its per-token latency the slowest rank's
            for key in sorted(k for k, v in decode.items() if isinstance(v, dict) and "tok_s" in v):
                t = torch.tensor([decode[key]["tok_s"], decode[key]["ms_per_token"]],
                                 dtype=torch.float64, device=device)
                tot, worst = t.clone(), t.clone()
                dist.all_reduce(tot, op=dist.ReduceOp.SUM)
                dist.all_reduce(worst, op=dist.ReduceOp.MAX)
                decode[key]["aggregate_tok_s"] = round(float(tot[0]), 2)
                decode[key]["max_ms_per_token"] = round(float(worst[1]), 4)
            decode["replicas"] = world

    partitioned = None
    if not args.no_decode and args.partitioned:
        partitioned = partitioned_decode(device, dist)

    if rank == 0 and world == 1 and not args.no_decode and args.tinyllama:
        decode = decode if decode is not None else {}
        decode["tinyllama"] = tinyllama_bench(device, with_cpu=not args.no_cpu)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        value, ms, threads, sample = run_cpu(max(1, args.cpu_steps), 1, budget_s=args.cpu_seconds)
        cpu = {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": sample}

    if rank == 0:
        peak, peak_kind = measured_peak()
        k, n = SHAPES[DOMINANT]
        achieved = alg_bytes(M, k, n) / (dom_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(world * STEP_BYTES / (ms_step * 1e-3) / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_block(),
            "roofline": {"bound": "hbm", "kernel": f"rw4 gemv (K={k}, N={n}, M={M})",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": traffic_per_launch(),
                         "algorithmic_bytes": alg_bytes(M, k, n),
                         "avg_launch_ms": round(dom_ms, 5)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4), "path": "pinned host weights -> rw4_xfer "
                    "(2 copy streams, 16 MB chunks) -> 2 device slots -> rw4_linear -> D2H",
                    "h2d_gbs": round(h2d / (e2e_ms * 1e-3) / 1e9, 2),
                    "h2d_probe_gbs": round(h2d_peak, 2) if h2d_peak else None,
                    "h2d_frac": round(h2d / (e2e_ms * 1e-3) / 1e9 / h2d_peak, 4)
                    if h2d_peak else None},
            "decode": decode,
            "partitioned_decode": partitioned,
            "gpu_launches": len(SHAPES) * args.steps,
            "clocks": clock,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def moe_sweep(args):
    """Routed-experts kernel timing (not the driver's line): the grouped RW4 GEMV at the
    Mixtral-8x7B expert shapes (8 experts, gate/up 2 x 14336 x 4096 with the SwiGLU epilogue, down
    4096 x 14336) for ``--moe-tokens-list`` tokens routed top-2 (distinct random experts per token,
    seeded), one JSON line per (tokens, projection) with the launch's CUDA-event time over
    ``--steps`` graphed back-to-back launches and the routed experts' weight bytes per second
    against the measured HBM peak."""
    from rocketllm_b200 import kernels
    from rocketllm_b200.synthetic import make_weight
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peak()
    n_exp, hid, inter, top = 8, 4096, 14336, 2
    gate_up = [make_weight(2 * inter, hid, device=device, seed=e) for e in range(n_exp)]
    down = [make_weight(hid, inter, device=device, seed=100 + e) for e in range(n_exp)]

    def nbytes(trip):
        return sum(t.numel() * t.element_size() for t in trip)

    for t in (int(v) for v in args.moe_tokens_list.split(",")):
        g = torch.Generator(device=device).manual_seed(t)
        x = torch.randn(t, hid, device=device, generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(n_exp, device=device, generator=g)[:top]
                           for _ in range(t)])
        perm, inv, off = kernels.moe_permute(idx, n_exp)
        routed = sorted(set(idx.flatten().tolist()))
        xp = kernels.moe_gather(x, perm, top)
        act = kernels.moe_grouped(xp, off, gate_up, act=1, max_rows=t)
        yp = kernels.moe_grouped(act, off, down, act=0, max_rows=t)
        for name, weights, fn in (
                ("gate_up", gate_up,
                 lambda: kernels.moe_grouped(xp, off, gate_up, act=1, max_rows=t, out=act)),
                ("down", down,
                 lambda: kernels.moe_grouped(act, off, down, act=0, max_rows=t, out=yp))):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(args.steps):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.steps
            wb = sum(nbytes(weights[e]) for e in routed)
            gbs = wb / (ms * 1e-3) / 1e9
            print(json.dumps({"moe": "Mixtral-8x7B experts, RW4 group 64", "tokens": t,
                              "top_k": top, "projection": name, "routed_experts": len(routed),
                              "us": round(ms * 1e3, 1), "weight_gbs": round(gbs, 1),
                              "hbm_frac": round(gbs / peak, 4), "peaks": peak_kind,
                              "launches": args.steps}), flush=True)
            del graph
    assert kernels.device_status() == 0
    return 0


def sweep(args):
    """Kernel sweep (not the driver's line): every (K, N) x M of the isolated sweep, one JSON line
    each with the launch's CUDA-event time over ``--steps`` graphed back-to-back launches (cycling
    through enough copies of the weight that none is still in L2), its algorithmic GB/s and
    TFLOP/s against the measured peaks, and which kernel ran (1 GEMV, 2 tcgen05 GEMM, 3 GEMV
    slices, 4 tcgen05 decode GEMM)."""
    from rocketllm_b200 import kernels
    from rocketllm_b200.synthetic import make_activation, make_weight
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peak()
    tflops_peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops_peak = float(json.load(f)["bf16_tflops"])
    except Exception:  # noqa: BLE001
        tflops_peak = 1590.0
    shapes = SHAPES if args.sweep_shapes == "all" else tuple(
        tuple(int(v) for v in s.split("x")) for s in args.sweep_shapes.split(","))
    ms_list = [int(v) for v in args.sweep_m.split(",")]
    l2_bytes = 126 << 20
    for i, (k, n) in enumerate(shapes):
        # enough distinct copies of the weight that consecutive launches never find it in L2
        wbytes = n * k // 2 + 4 * n * (k // GROUP)
        copies = max(1, min(64, -(-3 * l2_bytes // wbytes)))
        ws = [make_weight(n, k, device=device, seed=10 * i + c) for c in range(copies)]
        for m in ms_list:
            x = make_activation(m, k, device=device, seed=100 + i)
            y = torch.empty(m, n, dtype=torch.bfloat16, device=device)
            path = args.sweep_path or None
            if (path == 2 and m <= 16) or (path == 4 and not 16 < m <= 64):
                continue
            for _ in range(args.warmup):
                for w in ws:
                    kernels.linear(x, *w, out=y, path=path)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            reps = max(args.steps, copies)
            with torch.cuda.graph(g):
                for r in range(reps):
                    kernels.linear(x, *ws[r % copies], out=y, path=path)
            g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            gbs = alg_bytes(m, k, n) / (ms * 1e-3) / 1e9
            tfl = 2 * m * n * k / (ms * 1e-3) / 1e12
            print(json.dumps({"K": k, "N": n, "M": m,
                              "path": path or kernels.linear_path(m, k, n),
                              "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                              "hbm_frac": round(gbs / peak, 4), "tflops": round(tfl, 1),
                              "tensor_frac": round(tfl / tflops_peak, 4),
                              "peaks": peak_kind, "weight_copies": copies, "launches": reps}),
                  flush=True)
            del g
        del ws
        torch.cuda.empty_cache()
    if kernels.device_status():
        raise RuntimeError("a kernel reported a timed-out wait")
    return 0


KV_CASES = (   # (model architecture, batch, query heads, kv heads, head_dim, context tokens)
    ("llama3-8b", 1, 32, 8, 128, 4096), ("llama3-8b", 1, 32, 8, 128, 32768),
    ("llama3-8b", 16, 32, 8, 128, 4096), ("llama3-8b", 16, 32, 8, 128, 32768),
    ("llama3-70b", 1, 64, 8, 128, 32768), ("llama3-405b", 4, 128, 8, 128, 32768),
)


def kv_attn_bench(args):
    """Decode attention of one layer over an int4 KV cache: the packed-history kernel vs the
    reference's behaviour on the same device (expand every quantized group to bf16, then SDPA over
    the whole history) and vs SDPA over an unquantized bf16 cache.  L2 is flushed (a 256 MB write)
    before every timed launch; each launch is timed alone with CUDA events.  One JSON line per
    case: algorithmic bytes (codes + scales + zeros of the quantized groups, the bf16 window) per
    launch, GB/s, and the fraction of the measured HBM copy bandwidth."""
    import torch.nn.functional as F

    from rocketllm_b200 import kernels
    from rocketllm_b200.kv_cache import RW4KVCache
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak, peak_kind = measured_peak()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    iters = max(5, min(args.steps, 50))

    def timed(fn):
        for _ in range(3):
            fn()
        total = 0.0
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        return total / iters

    picked = KV_CASES if args.kv_cases == "all" else tuple(
        KV_CASES[int(i)] for i in args.kv_cases.split(","))
    for name, bsz, h, kvh, d, ctx in picked:
        g = torch.Generator(device=device).manual_seed(ctx + bsz)
        cache = RW4KVCache(fused=True)
        k = torch.randn(bsz, kvh, ctx - 1, d, device=device, generator=g).to(torch.bfloat16)
        v = torch.randn(bsz, kvh, ctx - 1, d, device=device, generator=g).to(torch.bfloat16)
        cache.update(k, v, 0)
        del k, v
        cache.update(torch.randn(bsz, kvh, 1, d, device=device, generator=g).to(torch.bfloat16),
                     torch.randn(bsz, kvh, 1, d, device=device, generator=g).to(torch.bfloat16), 0)
        layer = cache._kv[0]
        nq = args.kv_q
        q = torch.randn(bsz, h, nq, d, device=device, generator=g).to(torch.bfloat16)
        scaling = d ** -0.5
        ms = timed(lambda: cache.attend(0, q, scaling))
        # the query positions are the last nq of the ctx tokens (causal, aligned to the cache end)
        mask = None if nq == 1 else (torch.arange(ctx, device=device)[None, :] <=
                                     (ctx - nq + torch.arange(nq, device=device))[:, None])

        def reference_step():
            hk, hv = cache.history(0)
            F.scaled_dot_product_attention(q, hk, hv, attn_mask=mask, scale=scaling,
                                           enable_gqa=True)

        ms_ref = timed(reference_step)
        hk, hv = cache.history(0)
        ms_bf16 = timed(lambda: F.scaled_dot_product_attention(q, hk, hv, attn_mask=mask,
                                                               scale=scaling, enable_gqa=True))
        vg = d // 64
        alg = bsz * kvh * (layer.groups * (36 * d + 32 * d + 64 * vg * 4) + layer.rlen * 4 * d) \
            + 2 * bsz * h * nq * d * 2
        bf16_bytes = 2 * hk.numel() * 2
        gbs = alg / (ms * 1e-3) / 1e9
        print(json.dumps({
            "kv_attention": name, "batch": bsz, "heads": h, "kv_heads": kvh, "head_dim": d,
            "query_positions": nq,
            "context": ctx, "quantized_tokens": layer.groups * 64, "window_tokens": layer.rlen,
            "us": round(ms * 1e3, 2), "alg_bytes": alg, "gbs": round(gbs, 1),
            "hbm_frac": round(gbs / peak, 4), "peak": peak_kind,
            "reference_us": round(ms_ref * 1e3, 2), "speedup_vs_reference": round(ms_ref / ms, 2),
            "bf16_cache_sdpa_us": round(ms_bf16 * 1e3, 2), "bf16_cache_bytes": bf16_bytes,
            "speedup_vs_bf16_cache": round(ms_bf16 / ms, 2), "l2": "flushed before each launch",
            "launches_timed": iters}), flush=True)
        del cache, hk, hv
        torch.cuda.empty_cache()
    if kernels.device_status():
        raise RuntimeError("a kernel reported a timed-out wait")
    return 0


class _ReplayDraft:
    """A draft that proposes the target's own greedy continuation (an ideal draft): the spec-decode
    lines then measure what one verify pass of k+1 positions costs against k+1 one-token steps."""

    def __init__(self, continuation, prompt, vocab):
        self.cont, self.prompt, self.vocab = continuation, prompt, vocab
        self.seconds = 0.0

    def reset(self):
        pass

    def crop(self, length):
        pass

    def propose(self, sequence, cached, k, sampling, generator=None):
        at = sequence.shape[1] - self.prompt
        toks = self.cont[at:at + k]
        probs = torch.zeros(toks.shape[0], self.vocab, device=toks.device)
        probs.scatter_(1, toks.view(-1, 1), 1.0)
        return toks, probs if toks.shape[0] else None, cached


def spec_decode(args):
    """Speculative decoding on the streamed Llama-3-8B architecture (the decode bench's 4 GB
    budget: 19 layers pinned, 13 streamed every pass).  A one-token step streams the 13 layers; a
    verify pass streams them once for k+1 positions (RW4 GEMV at M = k+1).  The draft replays the
    target's greedy continuation (the plain run's tokens); the acceptance rate is measured, not
    assumed.  Both runs start from the same prefilled cache (the prompt but its last token, one
    pass), and a (k+1)-position pass gives each position the bits of a one-position step (RW4
    rows do not depend on the batch, SDPA's rows do not depend on the query count), so the
    replayed tokens are the target's own choices.  ``verify_pass_ms`` (k+1 positions) against
    ``step_ms`` (one position) is the exchange rate; ``tok_s_per_accepted_pass`` = (k+1) /
    verify_pass_ms is what each fully accepted pass delivers.  The timed regions exclude the
    prefill.  One JSON line per lookahead, each after its own warm-up run."""
    from transformers import DynamicCache, LlamaConfig

    from rocketllm_b200.engine import RocketModel
    from rocketllm_b200.speculative import SpeculativeDecoder
    from rocketllm_b200.synthetic import build_rw4_causal_lm
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = LlamaConfig(**LLAMA_8B)
    model = build_rw4_causal_lm(cfg, device=device, seed=0)
    target = RocketModel(model, device=device, vram_budget=int(4e9), window=2, kv_cache="fp16")
    n = args.spec_tokens
    ids = torch.randint(0, cfg.vocab_size, (1, 128),
                        generator=torch.Generator().manual_seed(0)).to(device)

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def prefilled():
        """A cache holding the prompt but its last token, made by one pass (the same pass for the
        plain and the speculative runs, so their caches hold the same bits)."""
        cache = DynamicCache()
        with torch.inference_mode():
            target(input_ids=ids[:, :-1], past_key_values=cache, use_cache=True)
        return cache

    def plain():
        cache = prefilled()
        torch.cuda.synchronize()
        a.record()
        with torch.inference_mode():
            tok, out = ids[:, -1:], []
            for _ in range(n):
                tok = target(input_ids=tok, past_key_values=cache, use_cache=True) \
                    .logits[:, -1:].argmax(-1)
                out.append(tok)
        b.record()
        torch.cuda.synchronize()
        return torch.cat(out, dim=1)[0], a.elapsed_time(b)

    plain()                                   # warm-up (first-touch of every slot and stream)
    cont, plain_ms = plain()
    base = {"spec_decode": "llama3-8b architecture, RW4, streamed (4 GB budget)",
            "prompt_tokens": 128, "new_tokens": n, "draft": "replay of the target's greedy tokens"}
    print(json.dumps({**base, "lookahead": 0, "tok_s": round(n / (plain_ms * 1e-3), 2),
                      "passes": n, "ms_per_pass": round(plain_ms / n, 2)}), flush=True)
    # raw target passes of w positions over the same 129-position cache (cropped back after each)
    cache = DynamicCache()
    with torch.inference_mode():
        target(input_ids=ids, past_key_values=cache, use_cache=True)
        widths = {}
        for w in (1, 2, 3, 4, 8):
            x = cont[:w].view(1, -1)
            for rep in range(4):
                if rep == 1:
                    a.record()
                target(input_ids=x, past_key_values=cache, use_cache=True)
                cache.crop(128)
            b.record()
            torch.cuda.synchronize()
            widths[w] = round(a.elapsed_time(b) / 3, 2)
    print(json.dumps({**base, "pass_ms_by_width": widths}), flush=True)
    for k in args.spec_lookaheads:
        # warm-up: a whole untimed run (the first speculative run of a process measured 2.3x
        # slower per pass than the same run repeated)
        SpeculativeDecoder(target, _ReplayDraft(cont, 128, cfg.vocab_size), lookahead=k,
                           max_lookahead=k).generate(ids, n, past_key_values=prefilled())
        dec = SpeculativeDecoder(target, _ReplayDraft(cont, 128, cfg.vocab_size), lookahead=k,
                                 max_lookahead=k)
        cache = prefilled()
        torch.cuda.synchronize()
        a.record()
        out = dec.generate(ids, n, past_key_values=cache)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        st = dec.stats
        # every pass carries the last accepted token and k proposals
        verify_ms = 1e3 * st.target_seconds / max(1, st.passes)
        print(json.dumps({**base, "lookahead": k, "tok_s": round(n / (ms * 1e-3), 2),
                          "speedup_vs_plain": round(plain_ms / ms, 2), "passes": st.passes,
                          "ms_per_pass": round(ms / st.passes, 2),
                          "verify_pass_ms": round(verify_ms, 2),
                          "step_ms": round(plain_ms / n, 2),
                          "pass_cost_ratio": round(verify_ms / (plain_ms / n), 3),
                          "tok_s_per_accepted_pass": round((k + 1) / (verify_ms * 1e-3), 1),
                          "acceptance_rate": round(st.acceptance_rate, 4),
                          "tokens_per_pass": round(st.tokens_per_pass, 2),
                          "same_tokens_as_plain": bool(torch.equal(out[0, 128:], cont))}),
              flush=True)
    target.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("rw4", "reference"), default="rw4")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the model decode section")
    ap.add_argument("--tinyllama", type=int, default=1,
                    help="1: include the TinyLlama configuration beside its reference (decode "
                         "section, one GPU)")
    ap.add_argument("--partitioned", type=int, default=1,
                    help="1: include the Mixtral decode, resident on one GPU and expert-parallel "
                         "(NCCL all-to-all) on several")
    ap.add_argument("--partitioned-only", action="store_true",
                    help="only the Mixtral decode of --partitioned, one JSON line (one GPU)")
    ap.add_argument("--partitioned-tokens", type=int, default=32)
    ap.add_argument("--tinyllama-only", action="store_true",
                    help="only the TinyLlama GPU / CPU-port decode comparison, one JSON line")
    ap.add_argument("--decode-prompt", type=int, default=2048)
    ap.add_argument("--decode-tokens", type=int, default=256)
    ap.add_argument("--stream-tokens", type=int, default=16)
    ap.add_argument("--stream-prompt", type=int, default=128,
                    help="prompt of the streamed decode (2048 for the streamed 8B configuration)")
    ap.add_argument("--stream-batches", default="1",
                    help="batch sizes of the streamed decode (1,16 for the streamed 8B "
                         "configuration)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="approximate CPU time of the CPU baseline leg")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--sweep", action="store_true",
                    help="kernel sweep over the sweep shapes x --sweep-m (one JSON line each)")
    ap.add_argument("--sweep-m", default="1,4,16,64,512,2048")
    ap.add_argument("--moe-sweep", action="store_true",
                    help="routed-experts grouped GEMV timing at the Mixtral expert shapes")
    ap.add_argument("--moe-tokens-list", default="1,8,32,128")
    ap.add_argument("--sweep-shapes", default="all", help="'all' or KxN[,KxN...]")
    ap.add_argument("--sweep-path", type=int, default=0,
                    help="force a kernel in --sweep: 2 tcgen05 GEMM, 3 GEMV slices, 4 tcgen05 "
                         "decode GEMM (0 = the "
                         "library's choice)")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the model decode section (one JSON line)")
    ap.add_argument("--decode-batches", default="1,16")
    ap.add_argument("--profile-window", action="store_true",
                    help="with --decode-only or --partitioned-only: bracket the timed steps with "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--storage-dir", default=None,
                    help="with --decode-only: also write the model as layer shards here and "
                         "decode from them with --host-budget-gb of layer blobs in host memory")
    ap.add_argument("--host-budget-gb", type=float, default=1.0)
    ap.add_argument("--pp-decode", action="store_true",
                    help="pipeline-parallel decode over the torchrun ranks (one JSON line)")
    ap.add_argument("--pp-model", choices=("405b", "8b"), default="405b")
    ap.add_argument("--pp-layers", type=int, default=0, help="override the layer count")
    ap.add_argument("--pp-batches", default="1,32")
    ap.add_argument("--pp-prompt", type=int, default=1024)
    ap.add_argument("--pp-tokens", type=int, default=64)
    ap.add_argument("--moe-decode", action="store_true",
                    help="streamed Mixtral-architecture decode with per-expert streaming")
    ap.add_argument("--moe-budget-gb", type=float, default=8.0)
    ap.add_argument("--moe-batches", default="1,32")
    ap.add_argument("--moe-prompt", type=int, default=512)
    ap.add_argument("--moe-tokens", type=int, default=16)
    ap.add_argument("--moe-routing", choices=("host", "device"), default="host",
                    help="routed-set read back to the host per MoE layer, or decided on the device")
    ap.add_argument("--expert-policy", choices=("lfu", "lru"), default=None,
                    help="expert cache eviction (default: lfu with host routing, lru with device)")
    ap.add_argument("--kv-attn", action="store_true",
                    help="decode attention over the int4 KV cache (one JSON line per case)")
    ap.add_argument("--kv-cases", default="all", help="'all' or indices into KV_CASES")
    ap.add_argument("--kv-q", type=int, default=1,
                    help="query positions per call (a speculative verify chunk when > 1)")
    ap.add_argument("--spec-decode", action="store_true",
                    help="speculative decoding on the streamed 8B (one JSON line per lookahead)")
    ap.add_argument("--spec-tokens", type=int, default=48)
    ap.add_argument("--spec-lookaheads", type=lambda v: [int(x) for x in v.split(",")],
                    default=[1, 3, 7])
    ap.add_argument("--ep-decode", action="store_true",
                    help="expert-parallel Mixtral-architecture decode over the torchrun ranks")
    ap.add_argument("--ep-graph", type=int, default=1,
                    help="1: fixed-capacity exchange and CUDA-graphed steps; 0: eager")
    args = ap.parse_args()
    if args.kv_attn:
        return kv_attn_bench(args)
    if args.spec_decode:
        return spec_decode(args)
    if args.sweep:
        return sweep(args)
    if args.moe_sweep:
        return moe_sweep(args)
    if args.ep_decode:
        return ep_decode(args)
    if args.moe_decode:
        return moe_decode(args)
    if args.pp_decode:
        return pp_decode(args)
    if args.decode_only:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        batches = tuple(int(b) for b in args.decode_batches.split(","))
        print(json.dumps(decode_bench(
            device, args.decode_prompt, args.decode_tokens, batches, args.stream_tokens,
            int(4e9), storage_dir=args.storage_dir,
            host_budget=int(args.host_budget_gb * 1e9) if args.storage_dir else None,
            profile_window=args.profile_window, stream_prompt=args.stream_prompt,
            stream_batches=tuple(int(v) for v in args.stream_batches.split(",")))), flush=True)
        return 0
    if args.partitioned_only:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps(partitioned_decode(device, None, tokens=args.partitioned_tokens,
                                            profile_window=args.profile_window)), flush=True)
        return 0
    if args.tinyllama_only:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps(tinyllama_bench(device, with_cpu=not args.no_cpu)), flush=True)
        return 0
    if args.impl == "reference":
        return reference_arm(args)
    return rw4_arm(args)


if __name__ == "__main__":
    sys.exit(main())

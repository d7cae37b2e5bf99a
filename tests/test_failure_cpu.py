"""Failure paths, made on the host (nothing here faults, traps or hangs a GPU).

* A shard file cut short: the reader raises on the short read instead of returning a partial layer.
* A pipeline rank that fails between steps: its peers' next receive / broadcast ends with an error
  within the short process-group timeout, instead of waiting for good.
* An expert-parallel rank that fails before a layer's exchange: the other rank's all-to-all ends
  with an error the same way.

Every rank takes the same collective steps in the same order until the injected failure; the
failing rank raises an exception of its own and leaves.
"""
import datetime
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TIMEOUT_S = 5


def test_a_short_shard_file_raises(tmp_path):
    from test_shards_cpu import tiny_rw4_model

    from rocketllm_b200.shards import LayerShardReader, split_rw4_layers
    root = split_rw4_layers(tiny_rw4_model(3), str(tmp_path / "shards"))
    reader = LayerShardReader(root)
    rec = reader.layers[1]
    path = os.path.join(root, rec["file"])
    with open(path, "r+b") as f:                       # lose the last 1000 bytes of layer 1
        f.truncate(rec["data_start"] + rec["nbytes"] - 1000)
    buf = torch.empty(rec["nbytes"] + 4096, dtype=torch.uint8)
    with pytest.raises(IOError, match="short read"):
        reader.read_into(1, buf)
    last = reader.plan(1)[0][-1]
    key = f"{last[0]}.{last[1]}" if last[0] else last[1]
    with pytest.raises(IOError, match="short read"):
        reader.read_tensor(1, key)
    reader.read_into(0, buf)                           # the intact layers still read
    assert reader.stats()["reads"] == 1


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))


def _pipeline_worker(rank, world, port, out):
    _init(rank, world, port)
    from test_pipeline_cpu import tiny_model

    from rocketllm_b200.pipeline import PipelineDecoder
    dec = PipelineDecoder(tiny_model(), device="cpu")
    if rank == world - 1:   # the last rank fails in its third forward, between steps
        calls = [0]
        layer = dec.layers[dec.start]
        original = layer.forward

        def failing(*a, **k):
            calls[0] += 1
            if calls[0] == 3:
                raise RuntimeError("injected failure")
            return original(*a, **k)

        layer.forward = failing
    ids = torch.randint(0, 97, (1, 5), generator=torch.Generator().manual_seed(2))
    t0 = time.monotonic()
    try:
        dec.generate(ids, 6)
        out[rank] = ("finished", 0.0)
    except Exception as e:  # noqa: BLE001 - the failure being tested
        out[rank] = (type(e).__name__ + ": " + str(e)[:120], time.monotonic() - t0)
    # no destroy_process_group: a peer is gone; the process ends here


def test_a_failed_pipeline_rank_ends_its_peers_collectives_with_an_error():
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_pipeline_worker, args=(2, 29741, out), nprocs=2, join=True)
        failed, peer = out[1], out[0]
        assert failed[0].startswith("RuntimeError: injected failure"), failed
        assert peer[0] != "finished", peer                     # the peer saw an error ...
        assert peer[1] < 6 * TIMEOUT_S, peer                     # ... within the timeout's reach


def _ep_worker(rank, world, port, out):
    _init(rank, world, port)
    from test_expert_parallel_cpu import CpuOps, E, K_TOP, make_problem, tokens

    from rocketllm_b200.expert_parallel import ExpertParallelMoE
    weights = make_problem(0)
    per = E // world
    mine = weights[rank * per:(rank + 1) * per]
    moe = ExpertParallelMoE(E, [a for a, _ in mine], [b for _, b in mine], ops=CpuOps(None))
    x, idx, w = tokens(rank, 6)
    t0 = time.monotonic()
    try:
        moe(x, idx, w)                                         # one exchange together
        if rank == 1:
            raise RuntimeError("injected failure")             # leaves before the next layer
        moe(x, idx, w)
        out[rank] = ("finished", 0.0)
    except Exception as e:  # noqa: BLE001 - the failure being tested
        out[rank] = (type(e).__name__ + ": " + str(e)[:120], time.monotonic() - t0)
    assert K_TOP >= 1


def test_a_failed_expert_parallel_rank_ends_the_exchange_with_an_error():
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_ep_worker, args=(2, 29751, out), nprocs=2, join=True)
        assert out[1][0].startswith("RuntimeError: injected failure"), dict(out)
        assert out[0][0] != "finished" and out[0][1] < 6 * TIMEOUT_S, dict(out)


def test_injected_read_faults_raise_and_the_reader_carries_on(tmp_path, monkeypatch):
    """Host-side fault injection (``faults=`` pairs, a spec string, or ``"env"`` for
    ``RW4_FAULT``): the listed (layer, read) pairs raise IOError, the others read normally; reads
    are counted per layer, so a fault lands on the same read whatever the threads' timing; the
    environment is read only when asked for."""
    from test_shards_cpu import tiny_rw4_model

    from rocketllm_b200.shards import LayerShardReader, split_rw4_layers
    root = split_rw4_layers(tiny_rw4_model(6), str(tmp_path / "shards"))
    reader = LayerShardReader(root, faults={(0, 2)})
    buf = torch.empty(max(l["nbytes"] for l in reader.layers), dtype=torch.uint8)
    reader.read_into(0, buf)
    reader.read_into(1, buf)
    with pytest.raises(IOError, match="injected read fault"):
        reader.read_into(0, buf)
    reader.read_into(0, buf)
    assert reader.stats()["reads"] == 3
    monkeypatch.setenv("RW4_FAULT", "read:layer=0:pass=1, read:layer=2")
    assert LayerShardReader(root).faults == set()          # not read unless asked for
    env = LayerShardReader(root, faults="env")
    assert env.faults == {(0, 1), (2, 1)}
    with pytest.raises(IOError, match="injected read fault"):
        env.read_tensor(0, "mlp.up_proj.weight_packed")
    env.read_tensor(0, "mlp.up_proj.weight_packed")
    with pytest.raises(ValueError):
        LayerShardReader(root, faults="read:8")

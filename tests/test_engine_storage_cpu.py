"""The engine's layer streaming and its storage tier, run on the CPU.

The copy mechanism is the only GPU part of the layer path, so here it is a fake transfer engine
that copies at once and releases the lease it was given (as the real one does when a copy has
finished); pinning is the identity and there are no CUDA streams.  Everything else -- the host and
storage tier split under ``host_budget``, ``LayerStager``'s read-ahead into leases, the layer
pre-hooks with their window prefetch, the binding of parameters into the slots -- is the
engine's own code, driving a plain fp32 Llama written as layer shards.  Logits and greedy tokens
must equal the model's own, and every pass must read the storage layers from their files again.
"""
import pytest
import torch

from rocketllm_b200 import engine
from rocketllm_b200.shards import split_rw4_layers


class _Handle:
    def resolve(self, stream=None):
        return None


class _FakeTransfer:
    def __init__(self, device_caps=None, pool=None, device=None, copy_streams=2,
                 chunk_bytes=1 << 24):
        self.pool = pool
        self.sent = 0
        self.leases = 0
        if pool is not None:
            pool.set_reclaim_hook(self.reclaim)

    def send_buffer(self, host, lease=None, out=None, after=None):
        n = host.numel() * host.element_size()
        out.view(-1)[:n].copy_(host.reshape(-1).view(torch.uint8)[:n])
        if lease is not None:
            self.leases += 1
            lease.release()
        self.sent += 1
        return _Handle()

    def reclaim(self):
        return 0

    def drain(self):
        return 0

    def stats(self):
        return {"transfers": self.sent, "leased_sends": self.leases}

    def close(self):
        pass


def _plain_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=64, intermediate_size=160, num_hidden_layers=5,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=96,
                      max_position_embeddings=64, tie_word_embeddings=False)
    return LlamaForCausalLM(cfg).float().eval()


@pytest.fixture
def cpu_engine(monkeypatch):
    import rocketllm_b200.quant.hf as hf
    monkeypatch.setattr(hf, "convert_modules", lambda model, skip=(): [])   # a plain model
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self, *a, **k: self)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: None)
    monkeypatch.setattr(engine, "WeightTransfer", _FakeTransfer)


@pytest.mark.parametrize("host_layers,depth,pinned", [(0, 1, 0), (1, 2, 0), (2, 3, 0), (1, 2, 1)])
def test_storage_tier_streams_the_models_own_logits(tmp_path, cpu_engine, host_layers, depth,
                                                    pinned):
    model = _plain_llama()
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    rest, layers = engine.footprint(model)
    blob = max(layers)
    rm = engine.RocketModel(root, device="cpu", dtype=torch.float32,
                            vram_budget=rest + (2 + pinned) * blob + 64 * 1024, window=2,
                            kv_cache="fp16",
                            host_budget=sum(layers[:host_layers]) + 4096 * host_layers,
                            storage_depth=depth)
    st = rm.streamer
    assert st is not None and st.window == 2 and st.pinned == pinned
    assert st.storage is not None and st.storage.order == list(range(host_layers, st.streamed))
    assert all(st.blobs[i].host is None for i in st.storage.order)
    assert all(st.blobs[i].host is not None for i in range(host_layers))
    ids = torch.randint(0, 96, (1, 9), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        want = model(ids).logits
        assert torch.equal(rm(ids).logits, want)
        a = model.generate(ids, max_new_tokens=5, do_sample=False, min_new_tokens=5)
        b = rm.generate(ids, max_new_tokens=5, do_sample=False, min_new_tokens=5)
    assert torch.equal(a, b)
    before = rm.stats()["streaming"]
    with torch.no_grad():
        rm(ids)
    after = rm.stats()["streaming"]
    # a pass over the layers in steady state sends each streamed layer exactly once and reads
    # each storage layer exactly once (the window is a FIFO pipeline over the cyclic scan)
    assert after["fetches"] - before["fetches"] == st.streamed
    assert after["storage"]["reads"] - before["storage"]["reads"] == len(st.storage.order)
    stats = after
    n_store = len(st.storage.order)
    assert stats["storage"]["reads"] >= 6 * n_store          # re-read from the files every pass
    assert stats["transfer"]["leased_sends"] == stats["storage"]["reads"]
    ahead = list(st.storage._pending.values())              # read-ahead nobody took
    assert ahead
    rm.close()
    assert all(f.result().released for f in ahead)          # released by close


def test_without_a_host_budget_every_blob_stays_in_host_memory(tmp_path, cpu_engine):
    model = _plain_llama()
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    rest, layers = engine.footprint(model)
    rm = engine.RocketModel(root, device="cpu", dtype=torch.float32,
                            vram_budget=rest + 2 * max(layers) + 64 * 1024, window=2,
                            kv_cache="fp16")
    assert rm.streamer.storage is None
    ids = torch.randint(0, 96, (1, 7), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        assert torch.equal(rm(ids).logits, model(ids).logits)
    rm.close()


@pytest.mark.parametrize("window,pinned", [(1, 0), (2, 1), (3, 0), (2, 2)])
def test_in_memory_streaming_windows_and_pins(cpu_engine, window, pinned):
    """A model already in host memory streams through ``window`` slots with the last ``pinned``
    layers resident: the model's own logits, and each streamed layer that shares its slot crosses
    once per pass (also when the layer count is not a multiple of the window and the prefetch
    wraps); a layer alone in its slot crosses once."""
    model = _plain_llama()
    ref = _plain_llama()                    # the same seed: RocketModel takes over ``model``
    rest, layers = engine.footprint(model)
    budget = rest + window * max(layers) + sum(layers[len(layers) - pinned:]) + 64 * 1024
    rm = engine.RocketModel(model, device="cpu", dtype=torch.float32, vram_budget=budget,
                            window=window, kv_cache="fp16")
    st = rm.streamer
    assert (st.window, st.pinned, st.streamed) == (window, pinned, 5 - pinned)
    ids = torch.randint(0, 96, (2, 6), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        want = ref(ids).logits
        assert torch.equal(rm(ids).logits, want)
        before = rm.stats()["streaming"]["fetches"]
        assert torch.equal(rm(ids).logits, want)
    per_pass = rm.stats()["streaming"]["fetches"] - before
    # layer i lives in slot i % window; a layer alone in its slot stays there between passes
    sharing = [sum(1 for j in range(st.streamed) if j % window == i % window)
               for i in range(st.streamed)]
    assert per_pass == sum(1 for n in sharing if n > 1)
    rm.close()


def test_host_budget_needs_a_shard_directory():
    with pytest.raises(ValueError, match="layer-shard directory"):
        engine.RocketModel(_plain_llama(), device="cpu", vram_budget=1, host_budget=1)


def test_an_injected_storage_read_fault_fails_one_pass_and_the_next_reads_again(
        tmp_path, cpu_engine, monkeypatch):
    """``RW4_FAULT=read:layer=1:pass=2`` (read because ``read_faults="env"``): the second read of
    layer 1's shard raises (host-side injection, nothing on a device).  The pass that needs it ends
    with that IOError, no lease is left behind, and the next pass reads the layer again and gives
    the model's own logits."""
    model = _plain_llama()
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    rest, layers = engine.footprint(model)
    monkeypatch.setenv("RW4_FAULT", "read:layer=1:pass=2")
    rm = engine.RocketModel(root, device="cpu", dtype=torch.float32,
                            vram_budget=rest + 2 * max(layers) + 64 * 1024, window=2,
                            kv_cache="fp16", host_budget=0, storage_depth=2, read_faults="env")
    st = rm.streamer
    assert st.storage.reader.faults == {(1, 2)} and 1 in st.storage.order
    ids = torch.randint(0, 96, (1, 7), generator=torch.Generator().manual_seed(8))
    with torch.no_grad():
        want = model(ids).logits
        failed = 0
        for _ in range(4):
            try:
                got = rm(ids).logits
            except IOError as e:
                assert "injected read fault" in str(e)
                failed += 1
                continue
            assert torch.equal(got, want)
        assert failed == 1
    assert st.storage.reader.stats()["reads"] >= 3 * 5          # three whole passes read
    ahead = list(st.storage._pending.values())
    rm.close()
    assert all(f.result().released for f in ahead)


def test_unknown_constructor_arguments_are_rejected():
    """A misspelt knob is an error; the reference's own knobs that have no effect here are
    accepted (code written for the reference runs unchanged); compression= raises as there."""
    with pytest.raises(TypeError, match="windw"):
        engine.RocketModel(_plain_llama(), device="cpu", windw=3)
    rm = engine.RocketModel(_plain_llama(), device="cpu", dtype=torch.float32, max_seq_len=512,
                            pin_policy="auto", vram_reserve=None)
    assert rm.streamer is None
    with pytest.raises(ValueError, match="pre-quantized"):
        engine.RocketModel(_plain_llama(), device="cpu", compression="4bit")

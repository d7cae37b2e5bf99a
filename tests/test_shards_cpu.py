"""RW4 layer shards (the reference's per-layer split + byte-range reader, rocketllm/utils.py:470-621,
streaming/shards.py, streaming/loader.py:161-236), on the CPU: every file is a valid safetensors
container whose tensors equal the model's, a layer's blob read by positioned reads (one, or
byte-balanced stretches on I/O threads) holds every tensor at the engine's aligned offset, the
index alone plans a layer, a finished layer (.done marker) is not rewritten, and the storage tier
reads ahead in scan order into leases it gives back."""
import os

import pytest
import torch

from rocketllm_b200.engine import _layer_tensors, _pack_layer
from rocketllm_b200.shards import INDEX, LayerShardReader, layer_entries, split_rw4_layers


def tiny_rw4_model(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM

    from rocketllm_b200.quant.hf import convert_modules
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=320,
                      max_position_embeddings=64, tie_word_embeddings=False)
    model = LlamaForCausalLM(cfg)
    convert_modules(model)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dtype == torch.uint8:
                p.copy_(torch.randint(0, 256, p.shape, generator=g, dtype=torch.uint8))
            else:
                p.copy_(torch.randn(p.shape, generator=g).to(p.dtype))
    return model


def test_files_are_safetensors_with_the_models_tensors(tmp_path):
    from safetensors import safe_open
    model = tiny_rw4_model()
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    reader = LayerShardReader(root)
    assert len(reader) == 3
    for i, layer in enumerate(model.model.layers):
        path = os.path.join(root, reader.layers[i]["file"])
        assert os.path.exists(path + ".done")
        names = {id(m): n for n, m in layer.named_modules()}
        with safe_open(path, framework="pt") as f:
            keys = set(f.keys())
            for module, leaf, kind, t in _layer_tensors(layer):
                key = f"{names[id(module)]}.{leaf}" if names[id(module)] else leaf
                assert key in keys
                assert torch.equal(f.get_tensor(key), t)
        assert reader.layers[i]["data_start"] % 4096 == 0


def test_read_into_gives_the_engines_blob(tmp_path):
    model = tiny_rw4_model(1)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    reader = LayerShardReader(root)
    for i, layer in enumerate(model.model.layers):
        entries, nbytes = reader.plan(i)
        want, want_bytes = layer_entries(layer)
        assert nbytes == want_bytes
        assert [e[:2] + e[3:] for e in entries] == [e[:2] + e[3:] for e in want]
        buf = torch.zeros(nbytes + 4096, dtype=torch.uint8)
        reader.read_into(i, buf)
        packed = _pack_layer(layer) if torch.cuda.is_available() else None
        for (m, leaf, kind, dt, shape, off), (_, _, _, t) in zip(entries, _layer_tensors(layer)):
            n = t.numel() * t.element_size()
            assert torch.equal(buf[off:off + n], t.contiguous().view(-1).view(torch.uint8))
        if packed is not None:
            assert torch.equal(buf[:nbytes], packed.host[:nbytes])
    assert reader.stats()["bytes_read"] == sum(l["nbytes"] for l in reader.layers)


def test_done_layers_are_not_rewritten(tmp_path):
    model = tiny_rw4_model(2)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    path = os.path.join(root, "layers", "layer.1.safetensors")
    before = os.stat(path).st_mtime_ns
    os.remove(os.path.join(root, INDEX))
    split_rw4_layers(model, root)
    assert os.stat(path).st_mtime_ns == before
    assert os.path.exists(os.path.join(root, INDEX))


def test_a_subset_or_row_slice_costs_only_its_bytes(tmp_path):
    """One tensor of a layer, or a row range of it, is one positioned read of exactly those bytes
    (the reference loader's subset and per-expert row reads, streaming/loader.py:161-236)."""
    model = tiny_rw4_model(2)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    reader = LayerShardReader(root)
    mlp = model.model.layers[1].mlp
    key = "mlp.up_proj.weight_packed"
    got = reader.read_tensor(1, key)
    assert torch.equal(got, mlp.up_proj.weight_packed)
    assert reader.stats()["bytes_read"] == got.numel()
    before = reader.stats()["bytes_read"]
    rows = reader.read_tensor(1, "mlp.up_proj.weight_scale", rows=(5, 9))
    assert torch.equal(rows, mlp.up_proj.weight_scale[5:9])
    assert reader.stats()["bytes_read"] - before == rows.numel() * rows.element_size()
    out = torch.empty_like(mlp.down_proj.weight_zero_point[:3])
    assert reader.read_tensor(1, "mlp.down_proj.weight_zero_point", rows=(0, 3), out=out) is out
    assert torch.equal(out, mlp.down_proj.weight_zero_point[:3])
    import pytest
    with pytest.raises(KeyError):
        reader.read_tensor(1, "mlp.no_such.weight")
    with pytest.raises(ValueError):
        reader.read_tensor(1, key, rows=(0, 10 ** 6))


def test_stretches_are_adjacent_aligned_and_byte_balanced():
    """The io-worker partition (the reference's ``partition``, streaming/shards.py:664-700):
    adjacent stretches covering the blob, cut on 4096-byte boundaries, balanced by bytes."""
    reader = object.__new__(LayerShardReader)
    reader.io_workers = 4
    mb = LayerShardReader.MIN_STRETCH
    for n in (0, 1, mb - 1, 3 * mb, 4 * mb + 12345, 10 * mb + 1, 1 << 31):
        parts = reader.stretches(n)
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        assert all(hi % 4096 == 0 for _, hi in parts[:-1])
        assert len(parts) <= max(1, min(4, n // mb))
        sizes = [hi - lo for lo, hi in parts]
        assert max(sizes) - min(sizes) <= 4096 * len(parts) or len(parts) == 1
    assert len(reader.stretches(1 << 31)) == 4 and len(reader.stretches(mb)) == 1
    assert len(reader.stretches(1 << 31, ways=2)) == 2


def test_parallel_reads_give_the_same_blob_and_fail_loudly(tmp_path):
    model = tiny_rw4_model(3)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    one = LayerShardReader(root)
    many = LayerShardReader(root, io_workers=3)
    many.MIN_STRETCH = 4096                 # force several stretches on these small layers
    for i in range(len(one)):
        n = one.layers[i]["nbytes"]
        assert len(many.stretches(n)) > 1
        a = torch.zeros(n + 4096, dtype=torch.uint8)
        b = torch.full((n + 4096,), 7, dtype=torch.uint8)
        one.read_into(i, a)
        many.read_into(i, b)
        assert torch.equal(a[:n], b[:n]) and int((b[n:] != 7).sum()) == 0
    assert many.stats()["parallel_reads"] == len(one) and many.stats()["io_workers"] == 3
    rec = many.layers[2]
    with open(os.path.join(root, rec["file"]), "r+b") as f:        # lose the last stretch's tail
        f.truncate(rec["data_start"] + rec["nbytes"] - 100)
    with pytest.raises(IOError, match="short read"):
        many.read_into(2, torch.zeros(rec["nbytes"], dtype=torch.uint8))
    many.close()


class _CountingPool:
    """A staging pool that hands out plain CPU buffers and records what comes back."""

    def __init__(self):
        self.leased, self.returned = 0, []

    def lease(self, count, dtype):
        from rocketllm_b200.streaming import BufferLease
        self.leased += 1
        return BufferLease(torch.zeros(count, dtype=dtype), self, self.leased)

    def _return(self, slot):
        self.returned.append(slot)


def test_the_storage_tier_reads_ahead_in_scan_order(tmp_path):
    """``LayerStager``: each take hands over the layer's blob (== a direct read) and starts the
    next ``depth`` storage layers' reads, wrapping around the scan."""
    from rocketllm_b200.shards import LayerStager
    model = tiny_rw4_model(4)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    direct = LayerShardReader(root)
    pool = _CountingPool()
    st = LayerStager(LayerShardReader(root), [0, 2], pool, depth=1)
    for rnd in range(3):
        for i in (0, 2):
            lease = st.take(i)
            want = direct.read_into(i, torch.zeros(direct.layers[i]["nbytes"], dtype=torch.uint8))
            assert torch.equal(lease.view, want)
            assert set(st._pending) == {2 if i == 0 else 0}     # the next one, wrapping
            lease.release()
    with pytest.raises(KeyError):
        st.take(1)                                           # not a storage layer
    assert st.stats()["reads"] == 6 and st.stats()["bytes"] == 3 * (
        direct.layers[0]["nbytes"] + direct.layers[2]["nbytes"])
    st.close()
    assert len(pool.returned) == pool.leased                # the pending read-ahead came back too


def test_a_failed_storage_read_releases_its_lease_and_raises(tmp_path):
    from rocketllm_b200.shards import LayerStager
    model = tiny_rw4_model(5)
    root = split_rw4_layers(model, str(tmp_path / "shards"))
    reader = LayerShardReader(root)
    rec = reader.layers[1]
    with open(os.path.join(root, rec["file"]), "r+b") as f:
        f.truncate(rec["data_start"] + rec["nbytes"] // 2)
    pool = _CountingPool()
    st = LayerStager(reader, [0, 1], pool, depth=1)
    st.take(0).release()
    with pytest.raises(IOError, match="short read"):
        st.take(1)
    assert pool.returned.count(2) == 1                      # the failed read's own lease
    st.close()
    assert sorted(pool.returned) == list(range(1, pool.leased + 1))

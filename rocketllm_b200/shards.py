"""RW4 layer shards on disk, laid out exactly as the engine's pinned host blobs.

Counterpart of the reference's per-layer checkpoint split (``rocketllm/utils.py:470-621``,
``split_and_save_layers``: one safetensors file per layer plus a ``.done`` marker) and of its
byte-range reader (``rocketllm/streaming/shards.py``, ``streaming/loader.py:161-236``:
``LayerLoader.plan`` reads only the header, ``load``/``_fill`` read the tensors into one leased
buffer).  Here a layer file's data section IS the layer's host blob: every tensor sits at the
256-byte aligned offset the engine binds device views at, so loading a layer is one positioned
read (or a few adjacent ones on I/O threads, for a large layer) straight into pinned memory -- no
per-tensor copy, no repacking -- and the data section starts on a 4096-byte boundary so the read
can bypass the page cache (``O_DIRECT``) where the file system allows it.

Each file is still a valid safetensors container: the JSON header names every tensor with its
dtype, shape and data offsets, gaps between aligned tensors are covered by ``__rw4_pad_<n>`` uint8
entries (safetensors wants the offsets contiguous), and the header is padded with spaces up to the
aligned data start.  ``rw4_layers.json`` indexes the layers (module path, leaf, dtype, shape,
offset of every tensor; the blob size), ``rest.safetensors`` holds everything outside the decoder
layers, ``config.json`` the model config with its ``quantization_config``.
"""
import json
import os
import threading

import torch

ALIGN = 256
DATA_ALIGN = 4096
INDEX = "rw4_layers.json"
REST = "rest.safetensors"

_ST_DTYPES = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16",
              torch.uint8: "U8", torch.int8: "I8", torch.int32: "I32", torch.int64: "I64",
              torch.bool: "BOOL", torch.float64: "F64", torch.int16: "I16"}
_FROM_ST = {v: k for k, v in _ST_DTYPES.items()}


def _dtype_name(dtype):
    return str(dtype).replace("torch.", "")


def _layer_file(i):
    return os.path.join("layers", f"layer.{i}.safetensors")


def layer_entries(layer, skip_experts=False):
    """``[(module_path, leaf, kind, dtype, shape, offset)]`` and the blob size: the engine's blob
    layout of ``layer`` (parameters and persistent buffers, 256-byte aligned, in module order)."""
    from .engine import _layer_tensors
    names = {id(m): n for n, m in layer.named_modules()}
    entries, off = [], 0
    for module, leaf, kind, t in _layer_tensors(layer, skip_experts):
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        entries.append((names[id(module)], leaf, kind, t.dtype, tuple(t.shape), off))
        off += t.numel() * t.element_size()
    return entries, (off + ALIGN - 1) // ALIGN * ALIGN


def _write_layer_file(path, layer, entries, nbytes):
    from .engine import _layer_tensors
    tensors = [t for *_, t in _layer_tensors(layer)]
    header, pos, pad = {}, 0, 0
    for (mname, leaf, kind, dtype, shape, off), t in zip(entries, tensors):
        if off > pos:
            header[f"__rw4_pad_{pad}"] = {"dtype": "U8", "shape": [off - pos],
                                          "data_offsets": [pos, off]}
            pad += 1
        n = t.numel() * t.element_size()
        key = f"{mname}.{leaf}" if mname else leaf
        header[key] = {"dtype": _ST_DTYPES[dtype], "shape": list(shape),
                       "data_offsets": [off, off + n]}
        pos = off + n
    if nbytes > pos:
        header[f"__rw4_pad_{pad}"] = {"dtype": "U8", "shape": [nbytes - pos],
                                      "data_offsets": [pos, nbytes]}
    header["__metadata__"] = {"format": "pt", "layout": "rw4-layer-blob"}
    text = json.dumps(header, separators=(",", ":")).encode()
    hlen = (8 + len(text) + DATA_ALIGN - 1) // DATA_ALIGN * DATA_ALIGN - 8
    text = text + b" " * (hlen - len(text))
    blob = bytearray(nbytes)
    for (mname, leaf, kind, dtype, shape, off), t in zip(entries, tensors):
        raw = t.detach().contiguous().cpu().view(-1).view(torch.uint8).numpy().tobytes()
        blob[off:off + len(raw)] = raw
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(len(text).to_bytes(8, "little"))
        f.write(text)
        f.write(blob)
    os.replace(tmp, path)
    return 8 + len(text)


def split_rw4_layers(model, out_dir):
    """Write ``model`` (an RW4 ``*ForCausalLM``) as per-layer blob files under ``out_dir``.

    Returns ``out_dir``.  A layer whose ``.done`` marker exists is not rewritten (the reference's
    resumable split)."""
    from safetensors.torch import save_file

    from .engine import _decoder_layers, _layers_path
    os.makedirs(os.path.join(out_dir, "layers"), exist_ok=True)
    layers = _decoder_layers(model)
    index = {"align": ALIGN, "data_align": DATA_ALIGN, "layers_path": _layers_path(model),
             "layers": []}
    for i, layer in enumerate(layers):
        entries, nbytes = layer_entries(layer)
        rel = _layer_file(i)
        path = os.path.join(out_dir, rel)
        done = path + ".done"
        if os.path.exists(done):
            with open(path, "rb") as f:
                data_start = 8 + int.from_bytes(f.read(8), "little")
        else:
            data_start = _write_layer_file(path, layer, entries, nbytes)
            open(done, "w").close()
        index["layers"].append({
            "file": rel, "data_start": data_start, "nbytes": nbytes,
            "entries": [[m, leaf, kind, _dtype_name(dt), list(shape), off]
                        for m, leaf, kind, dt, shape, off in entries]})
    lp = index["layers_path"] + "."
    rest = {k: v.detach().contiguous().cpu() for k, v in model.state_dict().items()
            if not k.startswith(lp)}
    seen = {}
    for k, v in list(rest.items()):   # tied weights: safetensors refuses aliases
        key = (v.data_ptr(), v.numel()) if v.numel() else None
        if key is not None and key in seen:
            rest[k] = v.clone()
        elif key is not None:
            seen[key] = k
    save_file(rest, os.path.join(out_dir, REST), metadata={"format": "pt"})
    cfg = model.config.to_dict()
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    with open(os.path.join(out_dir, INDEX), "w") as f:
        json.dump(index, f)
    return out_dir


def parse_faults(spec):
    """Injected read faults as a set of ``(layer, read)`` pairs: the ``read``-th read (1-based) of
    ``layer``'s file fails.  ``spec`` is None (no faults), such a set, a string of
    ``read:layer=L[:pass=P]`` items (comma-separated; ``pass`` defaults to 1), or ``"env"`` to take
    that string from the ``RW4_FAULT`` environment variable (read only when asked for).  Counting
    per layer makes a fault land on the same read whatever the I/O threads' timing."""
    if spec is None:
        return set()
    if spec == "env":
        spec = os.environ.get("RW4_FAULT", "")
    if not isinstance(spec, str):
        return {(int(a), int(b)) for a, b in spec}
    out = set()
    for item in spec.split(","):
        item = item.strip()
        if not item:
            continue
        kind, _, rest = item.partition(":")
        fields = dict(f.split("=", 1) for f in rest.split(":") if "=" in f)
        if kind != "read" or "layer" not in fields:
            raise ValueError(f"fault {item!r}: expected read:layer=L[:pass=P]")
        out.add((int(fields["layer"]), int(fields.get("pass", 1))))
    return out


class LayerShardReader:
    """Reads layer blobs of a directory written by :func:`split_rw4_layers`.

    ``io_workers`` > 1 reads a layer of at least ``io_workers`` x ``MIN_STRETCH`` bytes as that
    many adjacent, byte-balanced stretches on as many threads (positioned reads release the
    interpreter lock): the reference loader's ``io_workers`` partition (``streaming/loader.py:
    214-236``, ``streaming/shards.py:664-700``: batches balanced by bytes, each one a contiguous
    sweep of the file, the submitting thread taking the first).  A layer here is one blob, so the
    stretches are cut at 4096-byte boundaries of the blob itself rather than between tensors."""

    MIN_STRETCH = 4 << 20

    def __init__(self, root, io_workers=1, faults=None):
        self.root = str(root)
        # host-side fault injection (parse_faults): the listed (layer, read) pairs raise IOError
        # instead of reading, read_into and read_tensor alike counting per layer
        self.faults = parse_faults(faults)
        self._layer_reads = {}
        with open(os.path.join(self.root, INDEX)) as f:
            self.index = json.load(f)
        self.layers = self.index["layers"]
        self.io_workers = max(1, int(io_workers))
        self._executor = None
        self._lock = threading.Lock()   # reads may come from several I/O threads
        self.reads = 0
        self.bytes_read = 0
        self.direct_reads = 0
        self.parallel_reads = 0

    def __len__(self):
        return len(self.layers)

    def plan(self, i):
        """``(entries, nbytes)`` of layer ``i`` from the index alone (nothing else is read)."""
        rec = self.layers[i]
        entries = [(m, leaf, kind, getattr(torch, dt), tuple(shape), off)
                   for m, leaf, kind, dt, shape, off in rec["entries"]]
        return entries, rec["nbytes"]

    def stretches(self, nbytes, ways=None):
        """``[(lo, hi), ...]``: ``[0, nbytes)`` cut into at most ``ways`` adjacent stretches of
        nearly equal bytes, every cut on a 4096-byte boundary, none under ``MIN_STRETCH``."""
        if nbytes <= 0:
            return [(0, 0)]
        ways = self.io_workers if ways is None else max(1, int(ways))
        ways = max(1, min(ways, nbytes // self.MIN_STRETCH))
        step = -(-nbytes // ways)
        step = -(-step // DATA_ALIGN) * DATA_ALIGN
        return [(lo, min(nbytes, lo + step)) for lo in range(0, nbytes, step)]

    def _read_stretch(self, path, view, start, lo, hi, direct_ok):
        """Positioned reads of blob bytes ``[lo, hi)`` (file offset ``start + lo``) into
        ``view[lo:hi]``; ``O_DIRECT`` for the whole 4096-byte blocks when the file system accepts
        it, the ragged tail buffered.  Returns whether any of it bypassed the page cache."""
        fd, direct = None, False
        if direct_ok:
            try:
                fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
                direct = True
            except OSError:
                fd = None
        if fd is None:
            fd = os.open(path, os.O_RDONLY)
        used_direct = False
        try:
            done = lo
            while done < hi:
                want = hi - done
                if direct:
                    # O_DIRECT moves whole 4096-byte blocks: the aligned part goes direct, a ragged
                    # tail through the page cache
                    want -= want % DATA_ALIGN
                    if not want:
                        os.close(fd)
                        fd, direct = os.open(path, os.O_RDONLY), False
                        continue
                    want = min(want, 1 << 30)
                try:
                    got = os.preadv(fd, [view[done:done + want]], start + done)
                except OSError:
                    if not direct:
                        raise
                    os.close(fd)
                    fd, direct = os.open(path, os.O_RDONLY), False
                    continue
                if got <= 0:
                    raise IOError(f"{path}: short read at {start + done}")
                used_direct |= direct
                done += got
        finally:
            os.close(fd)
        return used_direct

    def read_into(self, i, buffer):
        """Read layer ``i``'s blob into ``buffer`` (a CPU uint8 tensor of at least ``nbytes``,
        pinned or not) with positioned reads, over ``io_workers`` threads for a large layer;
        ``O_DIRECT`` when the buffer, size and file offset are 4096-aligned and the file system
        accepts it.  A short file raises ``IOError``."""
        rec = self.layers[i]
        nbytes, start = rec["nbytes"], rec["data_start"]
        if buffer.dtype != torch.uint8 or buffer.numel() < nbytes or buffer.is_cuda:
            raise ValueError("read_into needs a CPU uint8 buffer of at least the blob's size")
        path = os.path.join(self.root, rec["file"])
        self._maybe_fault(path, i)
        view = memoryview(buffer[:nbytes].numpy()).cast("B")
        direct_ok = (hasattr(os, "O_DIRECT") and buffer.data_ptr() % DATA_ALIGN == 0
                     and start % DATA_ALIGN == 0)
        parts = self.stretches(nbytes)
        if len(parts) == 1:
            direct = self._read_stretch(path, view, start, 0, nbytes, direct_ok)
        else:
            with self._lock:
                if self._executor is None:
                    from concurrent.futures import ThreadPoolExecutor
                    self._executor = ThreadPoolExecutor(max_workers=self.io_workers - 1,
                                                        thread_name_prefix="rw4-shard-read")
                executor = self._executor
            futures = [executor.submit(self._read_stretch, path, view, start, lo, hi,
                                             direct_ok) for lo, hi in parts[1:]]
            first_error = None
            try:
                direct = self._read_stretch(path, view, start, *parts[0], direct_ok)
            except BaseException as e:  # noqa: BLE001 - re-raised once the others are done
                first_error, direct = e, False
            for f in futures:              # every stretch finishes before the buffer is handed on
                try:
                    direct |= f.result()
                except BaseException as e:  # noqa: BLE001
                    first_error = first_error or e
            if first_error is not None:
                raise first_error
            with self._lock:
                self.parallel_reads += 1
        with self._lock:
            self.reads += 1
            self.bytes_read += nbytes
            self.direct_reads += int(direct)
        return buffer

    def close(self):
        with self._lock:
            executor, self._executor = self._executor, None
        if executor is not None:
            executor.shutdown(wait=True)

    def read_tensor(self, i, key, rows=None, out=None):
        """One tensor of layer ``i`` -- ``key`` is ``"<module path>.<leaf>"`` as in the index -- or
        the rows ``[start, stop)`` of its leading dimension (one expert of a stacked tensor), read
        with one positioned read of exactly those bytes (``loader.py:161-236``: a subset of a
        layer costs only its own bytes).  Returns a CPU tensor of the entry's dtype (``out``, a CPU
        tensor of that shape and dtype, is filled instead of allocating)."""
        rec = self.layers[i]
        for m, leaf, kind, dt, shape, off in rec["entries"]:
            if (f"{m}.{leaf}" if m else leaf) == key:
                break
        else:
            raise KeyError(f"layer {i} has no tensor {key!r}")
        dtype = getattr(torch, dt)
        shape = list(shape)
        item = torch.empty((), dtype=dtype).element_size()
        row_elems = 1
        for d in shape[1:]:
            row_elems *= d
        start, stop = (0, shape[0]) if rows is None else (int(rows[0]), int(rows[1]))
        if not shape or not 0 <= start <= stop <= shape[0]:
            raise ValueError(f"rows {rows} outside {key!r} of shape {tuple(shape)}")
        shape[0] = stop - start
        nbytes = (stop - start) * row_elems * item
        if out is None:
            out = torch.empty(shape, dtype=dtype)
        elif (tuple(out.shape) != tuple(shape) or out.dtype != dtype or out.is_cuda
              or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous CPU {dtype} tensor of shape {shape}")
        view = memoryview(out.view(-1).view(torch.uint8).numpy()).cast("B")
        self._maybe_fault(os.path.join(self.root, rec["file"]), i)
        fd = os.open(os.path.join(self.root, rec["file"]), os.O_RDONLY)
        try:
            done = 0
            pos = rec["data_start"] + off + start * row_elems * item
            while done < nbytes:
                got = os.preadv(fd, [view[done:nbytes]], pos + done)
                if got <= 0:
                    raise IOError(f"{rec['file']}: short read at {pos + done}")
                done += got
        finally:
            os.close(fd)
        with self._lock:
            self.reads += 1
            self.bytes_read += nbytes
        return out

    def _maybe_fault(self, path, layer):
        with self._lock:
            n = self._layer_reads.get(layer, 0) + 1
            self._layer_reads[layer] = n
        if (layer, n) in self.faults:
            raise IOError(f"{path}: injected read fault (layer {layer}, read {n})")

    def stats(self):
        return {"layers": len(self.layers), "reads": self.reads, "bytes_read": self.bytes_read,
                "direct_reads": self.direct_reads, "parallel_reads": self.parallel_reads,
                "io_workers": self.io_workers}


class LayerStager:
    """The storage tier: streamed layers whose blobs stay in their shard files and are read, ahead
    of use, into leased staging buffers -- the reference cache's miss path (``memory/cache.py:
    236-250`` ``_fetch``, run ahead on prefetch workers by ``prefetch_window`` ``:254-272``; the
    loader's ``load`` into one leased buffer, ``streaming/loader.py:196-207``).

    ``order`` lists the storage-tier layers in the order the forward visits them (cyclically).
    ``take(i)`` returns layer ``i``'s blob in a :class:`~rocketllm_b200.streaming.BufferLease`,
    waiting for its read if it is still running, and starts the reads of the next ``depth``
    storage layers in that order on the I/O threads.  The caller hands the lease to
    ``WeightTransfer.send_buffer``, which releases it only once the copy has finished, so a staging
    buffer is never refilled while a copy still reads it.  A read that fails releases its lease and
    raises from ``take``.  Leases come from ``pool`` (a ``HostStagingPool``): pinned while its
    budget lasts, a transient pageable buffer after that.
    """

    def __init__(self, reader, order, pool, depth=2):
        from concurrent.futures import ThreadPoolExecutor
        self.reader = reader
        self.order = list(order)
        if not self.order:
            raise ValueError("a storage tier needs at least one layer")
        self.pos = {layer: k for k, layer in enumerate(self.order)}
        self.pool = pool
        self.depth = max(1, int(depth))
        self._executor = ThreadPoolExecutor(max_workers=self.depth,
                                            thread_name_prefix="rw4-storage")
        self._pending = {}
        self._lock = threading.Lock()
        self.reads = 0
        self.bytes = 0
        self.waits = 0

    def _load(self, i):
        lease = self.pool.lease(self.reader.layers[i]["nbytes"], torch.uint8)
        try:
            self.reader.read_into(i, lease.view)
        except BaseException:
            lease.release()
            raise
        return lease

    def request(self, i):
        """Start reading layer ``i`` unless its read is already pending."""
        if i not in self.pos:
            raise KeyError(f"layer {i} is not in the storage tier")
        with self._lock:
            if i not in self._pending:
                self._pending[i] = self._executor.submit(self._load, i)

    def take(self, i):
        """Layer ``i``'s blob in a lease (the caller owns it), then read ahead ``depth`` layers."""
        self.request(i)
        with self._lock:
            future = self._pending.pop(i)
        if not future.done():
            self.waits += 1
        lease = future.result()
        self.reads += 1
        self.bytes += self.reader.layers[i]["nbytes"]
        k = self.pos[i]
        for d in range(1, self.depth + 1):
            self.request(self.order[(k + d) % len(self.order)])
        return lease

    def stats(self):
        return {"layers": len(self.order), "depth": self.depth, "reads": self.reads,
                "bytes": self.bytes, "waits": self.waits}

    def close(self):
        """Wait for the reads in flight and release what nobody took."""
        with self._lock:
            pending, self._pending = list(self._pending.values()), {}
        for future in pending:
            try:
                future.result().release()
            except BaseException:  # noqa: BLE001 - a failed read already released its lease
                pass
        self._executor.shutdown(wait=True)
        self.reader.close()


def build_skeleton(root, dtype=torch.bfloat16):
    """The RW4 ``*ForCausalLM`` of ``root`` on the meta device (no storage allocated)."""
    from transformers import AutoConfig, AutoModelForCausalLM

    from .quant.hf import convert_modules
    config = AutoConfig.from_pretrained(root)
    q = getattr(config, "quantization_config", None)
    skip = (q.get("modules_to_not_convert") if isinstance(q, dict)
            else getattr(q, "modules_to_not_convert", None)) or ()
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(config, dtype=dtype)
    convert_modules(model, skip)
    return model


def _materialize_rest(model, root, device, layers_path):
    """Allocate everything outside the decoder layers on ``device`` and fill it from
    ``rest.safetensors``; rebuild non-persistent buffers (rotary frequencies)."""
    from safetensors.torch import load_file
    parent_path, _, leaf = layers_path.rpartition(".")
    parent = model.get_submodule(parent_path) if parent_path else model
    layers = getattr(parent, leaf)
    setattr(parent, leaf, torch.nn.ModuleList())
    model.to_empty(device=device)
    setattr(parent, leaf, layers)
    rest = load_file(os.path.join(root, REST), device=str(device))
    missing = []
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.startswith(layers_path + "."):
                continue
            if name in rest:
                p.copy_(rest[name])
            else:
                missing.append(name)
    if missing:
        raise ValueError(f"{REST} lacks {missing[:4]}")
    for mod in model.modules():
        if "inv_freq" in mod._buffers and hasattr(mod, "config"):
            fresh = type(mod)(mod.config, device=device)
            for bname, buf in fresh._buffers.items():
                mod._buffers[bname] = buf
            if hasattr(fresh, "attention_scaling"):
                mod.attention_scaling = fresh.attention_scaling
    if getattr(model.config, "tie_word_embeddings", False) and hasattr(model, "tie_weights"):
        model.tie_weights()

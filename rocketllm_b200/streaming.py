"""Host staging pool and host->device weight transfer, on the RW4 C ABI.

Drop-in counterparts of RocketLLM's ``rocketllm/streaming/staging.py`` (``BufferLease``,
``HostStagingPool``) and ``rocketllm/streaming/transfer.py`` (``TransferHandle``,
``WeightTransfer``): same method names, argument meaning and lease discipline, with the work done
by ``rw4_pool_*`` (pinned buffers in power-of-two size classes, leased) and ``rw4_xfer_*`` (chunked
copies on several dedicated copy streams, completion events, device-side waits).

The lease rule is the reference's (``transfer.py:61-77``): a staged host buffer goes back to the
pool only through :meth:`TransferHandle._release_source`, which refuses to release it before the
copy's events have fired.
"""
import ctypes
import threading

import torch

from . import _lib

_MIN_POOLED_BYTES = 1 << 16
DEFAULT_CHUNK_BYTES = 16 << 20


def _host_tensor(ptr, nbytes, dtype, count):
    """A CPU tensor viewing ``nbytes`` of host memory at ``ptr`` (no copy, no ownership)."""
    if nbytes == 0:
        return torch.empty(0, dtype=dtype)
    raw = (ctypes.c_uint8 * nbytes).from_address(ptr)
    return torch.frombuffer(raw, dtype=torch.uint8).view(dtype)[:count]


class BufferLease:
    """A host buffer checked out of the pool (``staging.py:33-66``)."""

    __slots__ = ("view", "_pool", "_slot", "released")

    def __init__(self, view, pool=None, slot=None):
        self.view = view
        self._pool = pool
        self._slot = slot
        self.released = False

    @property
    def pooled(self):
        return self._slot is not None

    def release(self):
        if self.released:
            return
        self.released = True
        if self._pool is not None and self._slot is not None:
            self._pool._return(self._slot)
        self.view = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()
        return False


class HostStagingPool:
    """Pinned, leased host buffers with a byte budget (``staging.py:80-273``).

    ``budget_bytes == 0`` is supported: no pinned memory, every lease a transient pageable buffer.
    Over the budget a lease also falls back to a transient buffer rather than recycling one that a
    copy may still be reading (``staging.py:218-227``).
    """

    def __init__(self, device_caps=None, budget_bytes=0):
        self.caps = device_caps
        self.budget_bytes = max(0, int(budget_bytes or 0))
        handle = ctypes.c_void_p()
        _lib.call("rw4_pool_create", self.budget_bytes, ctypes.byref(handle))
        self._handle = handle
        self._reclaim = None
        self._lock = threading.RLock()
        self._buffers = {}
        self.transient = 0

    @staticmethod
    def _size_class(count):
        """Next power of two, at least 2^16 (``staging.py:112-117``)."""
        if count <= _MIN_POOLED_BYTES:
            return _MIN_POOLED_BYTES
        return 1 << (count - 1).bit_length()

    def buffer(self, count, dtype):
        """A host buffer valid until the next ``buffer`` call (``staging.py:119-176``)."""
        lease = self.lease(count, dtype)
        view = lease.view
        with self._lock:
            old = self._buffers.pop(dtype, None)
            self._buffers[dtype] = lease
        if old is not None:
            old.release()
        return view

    def lease(self, count, dtype=torch.uint8):
        if count <= 0:
            return BufferLease(torch.empty(0, dtype=dtype))
        itemsize = torch.empty((), dtype=dtype).element_size()
        nbytes = count * itemsize
        slot = ctypes.c_int32()
        host = ctypes.c_void_p()
        with self._lock:
            st = _lib.lib().rw4_pool_lease(self._handle, nbytes, ctypes.byref(slot),
                                           ctypes.byref(host))
            if st == _lib.RW4_EBUSY and self._reclaim is not None:
                self._lock.release()
                try:
                    self._reclaim()
                finally:
                    self._lock.acquire()
                st = _lib.lib().rw4_pool_lease(self._handle, nbytes, ctypes.byref(slot),
                                               ctypes.byref(host))
        if st == _lib.RW4_OK:
            return BufferLease(_host_tensor(host.value, nbytes, dtype, count), self, slot.value)
        if st not in (_lib.RW4_EBUSY, _lib.RW4_ENOMEM):
            _lib.check(st, "rw4_pool_lease")
        self.transient += 1
        return BufferLease(torch.empty(count, dtype=dtype))

    def _return(self, slot):
        _lib.call("rw4_pool_release", self._handle, slot)

    def set_reclaim_hook(self, hook):
        self._reclaim = hook

    @property
    def leased(self):
        return self.stats()["leased"]

    def stats(self):
        resident = ctypes.c_uint64()
        buffers = ctypes.c_int32()
        leased = ctypes.c_int32()
        hits = ctypes.c_uint64()
        misses = ctypes.c_uint64()
        _lib.call("rw4_pool_stats", self._handle, ctypes.byref(resident), ctypes.byref(buffers),
                  ctypes.byref(leased), ctypes.byref(hits), ctypes.byref(misses))
        return {"buffers": len(self._buffers), "slots": buffers.value, "leased": leased.value,
                "resident_bytes": resident.value, "budget_bytes": self.budget_bytes,
                "hits": hits.value, "misses": misses.value + self.transient, "pinned": True}

    def clear(self):
        """Drop the ``buffer()`` views; pinned slots stay allocated for reuse."""
        with self._lock:
            old, self._buffers = self._buffers, {}
        for lease in old.values():
            lease.release()

    def close(self):
        if self._handle:
            _lib.call("rw4_pool_destroy", self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class TransferHandle:
    """One in-flight host->device copy and the host buffer it must outlive (``transfer.py:30-104``)."""

    __slots__ = ("device_buffer", "ticket", "_lease", "_transfer", "_resolved", "nbytes", "_lock")

    def __init__(self, device_buffer, ticket, lease, transfer):
        self.device_buffer = device_buffer
        self.ticket = ticket
        self._lease = lease
        self._transfer = transfer
        self._resolved = False
        self._lock = threading.Lock()
        self.nbytes = device_buffer.numel() * device_buffer.element_size()

    def is_complete(self):
        return _lib.check(_lib.lib().rw4_xfer_query(self._transfer._handle, self.ticket),
                          "rw4_xfer_query") == 1

    def synchronize(self, timeout_ms=-1):
        _lib.call("rw4_xfer_sync", self._transfer._handle, self.ticket, timeout_ms)

    def _release_source(self):
        """THE GUARD: the staged buffer goes back only once its copy has provably finished."""
        with self._lock:
            lease = self._lease
            if lease is None:
                return False
            if not self.is_complete():
                self.synchronize()
            self._lease = None
        lease.release()
        return True

    def reclaim_if_complete(self):
        if self._lease is None:
            return True
        if not self.is_complete():
            return False
        return self._release_source()

    def resolve(self, stream=None):
        """The device buffer, with ``stream`` (default: current) ordered behind the copy."""
        if not self._resolved:
            self._transfer._await(self, stream)
            self._resolved = True
        return self.device_buffer

    def __repr__(self):
        return f"<TransferHandle {self.nbytes}B ticket {self.ticket}>"


class WeightTransfer:
    """Host->device path on dedicated copy streams (``transfer.py:124-292``).

    A send is split into ``chunk_bytes`` pieces spread over ``copy_streams`` streams; compute waits
    on the send's events device-side.  ``out`` lets a caller refill a preallocated device slot, and
    ``after`` (a stream) makes the copy wait for that stream's queued work first, so a slot is not
    overwritten while compute still reads it.
    """

    def __init__(self, device_caps=None, pool=None, device=None, copy_streams=2,
                 chunk_bytes=DEFAULT_CHUNK_BYTES):
        self.caps = device_caps
        dev = torch.device(device if device is not None else "cuda")
        if dev.type != "cuda":
            raise ValueError("WeightTransfer moves weights to a CUDA device; there is no CPU path")
        self.device = torch.device("cuda", dev.index if dev.index is not None
                                   else torch.cuda.current_device())
        self.pool = pool
        self.chunk_bytes = int(chunk_bytes)
        handle = ctypes.c_void_p()
        _lib.call("rw4_xfer_create", self.device.index, int(copy_streams), ctypes.byref(handle))
        self._handle = handle
        self.is_async = True
        self._in_flight = []
        self._lock = threading.Lock()
        self.transfers = 0
        self.bytes_sent = 0
        self.stalls = 0
        if pool is not None and hasattr(pool, "set_reclaim_hook"):
            pool.set_reclaim_hook(self.reclaim)

    def send(self, staged):
        return self.send_buffer(staged.buffer, staged.lease)

    def send_buffer(self, host, lease=None, out=None, after=None):
        """Send ``host`` (a CPU tensor) to the device, taking ownership of ``lease``."""
        if host.is_cuda:
            raise ValueError("send_buffer takes a host tensor")
        host = host if host.is_contiguous() else host.contiguous()
        nbytes = host.numel() * host.element_size()
        if out is None:
            out = torch.empty(host.shape, dtype=host.dtype, device=self.device)
        elif out.numel() * out.element_size() < nbytes:
            raise ValueError("send_buffer: destination smaller than the host buffer")
        ticket = ctypes.c_uint64()
        # NULL means "no ordering" to the C ABI, so the legacy default stream (handle 0) is passed
        # as cudaStreamLegacy (handle 1).
        after_ptr = (after.cuda_stream or 1) if after is not None else None
        _lib.call("rw4_xfer_send", self._handle, out.data_ptr(), host.data_ptr(), nbytes,
                  self.chunk_bytes, after_ptr, ctypes.byref(ticket))
        handle = TransferHandle(out, ticket.value, lease, self)
        with self._lock:
            if lease is not None:
                self._in_flight.append(handle)
            self.transfers += 1
            self.bytes_sent += nbytes
        return handle

    def _await(self, handle, stream=None):
        stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.call("rw4_xfer_wait", self._handle, handle.ticket, stream.cuda_stream)
        try:
            handle.device_buffer.record_stream(stream)
        except Exception:  # noqa: BLE001 - preallocated slots are not allocator-owned
            pass
        self.reclaim()

    def reclaim(self):
        """Release the staging buffers of every finished transfer; never blocks."""
        with self._lock:
            pending = list(self._in_flight)
        still = [h for h in pending if not h.reclaim_if_complete()]
        with self._lock:
            done = {id(h) for h in pending} - {id(h) for h in still}
            self._in_flight = [h for h in self._in_flight if id(h) not in done]
        return len(still)

    def drain(self):
        with self._lock:
            pending, self._in_flight = list(self._in_flight), []
        for handle in pending:
            if not handle.is_complete():
                self.stalls += 1
            handle._release_source()
        return len(pending)

    def stats(self):
        sends = ctypes.c_uint64()
        nbytes = ctypes.c_uint64()
        chunks = ctypes.c_uint64()
        live = ctypes.c_int32()
        _lib.call("rw4_xfer_stats", self._handle, ctypes.byref(sends), ctypes.byref(nbytes),
                  ctypes.byref(chunks), ctypes.byref(live))
        with self._lock:
            in_flight = len(self._in_flight)
        return {"backend": "cuda", "async": True, "transfers": self.transfers,
                "bytes_sent": self.bytes_sent, "in_flight": in_flight, "stalls": self.stalls,
                "chunks": chunks.value, "copy_streams_tickets": live.value}

    def close(self):
        self.drain()
        if self._handle:
            _lib.call("rw4_xfer_destroy", self._handle)
            self._handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def __del__(self):
        try:
            if self._handle:
                _lib.lib().rw4_xfer_destroy(self._handle)
                self._handle = None
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


__all__ = ["BufferLease", "HostStagingPool", "TransferHandle", "WeightTransfer"]


class StagingRing:
    """A fixed ring of pinned staging slots feeding the device (``rw4_ring_*``).

    I/O workers fill slots (:meth:`stage`, or :meth:`slot` for a CPU tensor view to read into);
    the forward thread sends a slot to a device buffer (:meth:`submit`) and makes compute wait on
    the device (:meth:`wait_compute`).  A slot whose last send is still in flight raises
    :class:`~rocketllm_b200._lib.RW4Error` (``RW4_EBUSY``) on stage / submit.
    """

    def __init__(self, slot_bytes, slots, copy_streams=2, device=None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.slot_bytes, self.slots = int(slot_bytes), int(slots)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("rw4_ring_create", self.slot_bytes, self.slots, int(copy_streams),
                      ctypes.byref(handle))
        self._h = handle

    def slot(self, i):
        """Slot ``i`` as a CPU uint8 tensor view (no copy)."""
        ptr = ctypes.c_void_p()
        _lib.call("rw4_ring_slot", self._h, int(i), ctypes.byref(ptr))
        return _host_tensor(ptr.value, self.slot_bytes, torch.uint8, self.slot_bytes)

    def stage(self, i, src, offset=0):
        """Copy the bytes of CPU tensor ``src`` into slot ``i`` at ``offset``."""
        src = src.contiguous()
        _lib.call("rw4_ring_stage", self._h, int(i), int(offset), src.data_ptr(),
                  src.numel() * src.element_size())

    def submit(self, i, dst, nbytes=None, done=None):
        """Send slot ``i``'s first ``nbytes`` (default: ``dst``'s size) into CUDA tensor ``dst``;
        ``done`` (a recorded-before ``torch.cuda.Event``) is recorded behind the copies."""
        n = dst.numel() * dst.element_size() if nbytes is None else int(nbytes)
        _lib.call("rw4_ring_submit", self._h, int(i), dst.data_ptr(), n,
                  ctypes.c_void_p(done.cuda_event) if done is not None else None)

    def wait_compute(self, stream=None):
        stream = torch.cuda.current_stream(self.device) if stream is None else stream
        _lib.call("rw4_ring_wait_compute", self._h, ctypes.c_void_p(stream.cuda_stream))

    def close(self):
        if self._h:
            _lib.call("rw4_ring_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

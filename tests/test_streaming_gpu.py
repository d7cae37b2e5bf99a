"""Staging pool and transfer engine: byte-exact transfers, lease discipline, ordering.

Mirrors the reference's tests/test_staging_pool.py (reuse, size classes, budget, zero budget) and
tests/test_streaming_io.py (lease guard, staged bytes equal the source) on the CUDA path.
"""
import pytest
import torch

from rocketllm_b200.streaming import HostStagingPool, WeightTransfer

pytestmark = pytest.mark.gpu


def test_pool_reuses_and_respects_size_classes(cuda):
    pool = HostStagingPool(budget_bytes=64 << 20)
    a = pool.lease(100_000, torch.uint8)
    assert a.pooled and a.view.numel() == 100_000
    st = pool.stats()
    assert st["resident_bytes"] == 1 << 17  # next power of two
    a.release()
    b = pool.lease(70_000, torch.uint8)  # fits the same buffer: a hit, no new allocation
    assert pool.stats()["resident_bytes"] == 1 << 17 and pool.stats()["hits"] >= 1
    c = pool.lease(10, torch.float32)  # a second concurrent lease gets its own buffer
    assert pool.stats()["leased"] == 2
    b.release(), c.release()
    assert pool.stats()["leased"] == 0


def test_pool_budget_and_zero_budget_fall_back_to_transient(cuda):
    pool = HostStagingPool(budget_bytes=1 << 16)
    a = pool.lease(1 << 16)
    b = pool.lease(1 << 16)  # over budget while a is leased: transient, still correct
    assert a.pooled and not b.pooled
    assert pool.stats()["resident_bytes"] <= 1 << 16
    none = HostStagingPool(budget_bytes=0)
    c = none.lease(1000)
    assert not c.pooled and c.view.numel() == 1000


@pytest.mark.parametrize("nbytes,chunk", [(0, 0), (1, 0), (12345, 4096), (33 << 20, 8 << 20)])
def test_transfer_is_byte_exact(cuda, nbytes, chunk):
    pool = HostStagingPool(budget_bytes=128 << 20)
    xfer = WeightTransfer(pool=pool, device=cuda, copy_streams=3, chunk_bytes=chunk)
    lease = pool.lease(nbytes)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8)
    lease.view.copy_(src)
    h = xfer.send_buffer(lease.view, lease)
    dev = h.resolve()
    assert torch.equal(dev.cpu(), src)
    xfer.drain()
    assert pool.stats()["leased"] == 0
    xfer.close()


def test_lease_is_released_only_after_the_copy(cuda):
    pool = HostStagingPool(budget_bytes=64 << 20)
    xfer = WeightTransfer(pool=pool, device=cuda)
    lease = pool.lease(32 << 20)
    h = xfer.send_buffer(lease.view, lease)
    h._release_source()  # blocks until the copy is done, then releases
    assert h.is_complete() and pool.stats()["leased"] == 0
    xfer.close()


def test_after_stream_keeps_a_slot_from_being_overwritten(cuda):
    """A refill of a device slot waits for compute already queued on the slot."""
    xfer = WeightTransfer(device=cuda, chunk_bytes=1 << 20)
    slot = torch.zeros(8 << 20, dtype=torch.uint8, device=cuda)
    first = torch.full((8 << 20,), 7, dtype=torch.uint8).pin_memory()
    second = torch.full((8 << 20,), 9, dtype=torch.uint8).pin_memory()
    xfer.send_buffer(first, out=slot).resolve()
    compute = torch.cuda.current_stream()
    torch.cuda._sleep(50_000_000)  # compute is busy for a while ...
    seen = slot.clone()            # ... and then reads the slot
    xfer.send_buffer(second, out=slot, after=compute).resolve()
    torch.cuda.synchronize()
    assert int(seen.min()) == 7 and int(seen.max()) == 7
    assert int(slot.min()) == 9
    xfer.close()


def test_staging_ring_round_trip_and_busy_slot(cuda):
    """Slots staged on the host land byte-exact in device buffers; the done event and the device-
    side wait both cover the copies; a slot in flight refuses new bytes."""
    from rocketllm_b200._lib import RW4Error
    from rocketllm_b200.streaming import StagingRing
    ring = StagingRing(1 << 20, 3, copy_streams=2)
    src = [torch.randint(0, 256, (1 << 20,), dtype=torch.uint8) for _ in range(3)]
    dst = [torch.empty(1 << 20, dtype=torch.uint8, device=cuda) for _ in range(3)]
    done = torch.cuda.Event()
    done.record()                                   # creates the event the ring records into
    for i in range(3):
        ring.stage(i, src[i])
    ring.slot(2)[:16].fill_(7)                      # a worker writing straight into a slot
    src[2][:16] = 7
    for i in range(3):
        ring.submit(i, dst[i], done=done if i == 0 else None)
    done.synchronize()
    assert torch.equal(dst[0].cpu(), src[0])
    ring.wait_compute()
    for i in range(3):
        assert torch.equal(dst[i].cpu(), src[i])
    big = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    ring.submit(1, big)
    try:                                            # either refused while in flight, or done
        ring.stage(1, src[0])
    except RW4Error as e:
        assert "RW4_EBUSY" in str(e)
    torch.cuda.synchronize()
    ring.close()


def test_pool_buffers_pack_losslessly_cast_on_the_way_in_and_do_not_leak(cuda):
    """The reference pool's packing properties (tests/test_staging_pool.py:137-174): several
    tensors packed into one buffer read back exactly, a reused buffer carries nothing of the
    previous layer once rewritten, and packing in a narrower dtype casts on the way in."""
    pool = HostStagingPool(None, 64 << 20)
    g = torch.Generator().manual_seed(0)
    tensors = [torch.randn(shape, generator=g) for shape in ((16, 32), (32,), (8, 8, 4), (100,))]
    buf = pool.buffer(sum(t.numel() for t in tensors), torch.float32)
    off = 0
    for t in tensors:
        buf.narrow(0, off, t.numel()).copy_(t.reshape(-1))
        off += t.numel()
    off = 0
    for t in tensors:
        assert torch.equal(buf.narrow(0, off, t.numel()).view(t.shape), t)
        off += t.numel()
    first = pool.buffer(1000, torch.float32)
    first.fill_(7.0)
    second = pool.buffer(1000, torch.float32)
    second.copy_(torch.zeros(1000))
    assert torch.equal(second, torch.zeros(1000))
    src = torch.randn(64, generator=g)
    narrow = pool.buffer(64, torch.bfloat16)
    narrow.copy_(src)
    assert narrow.dtype == torch.bfloat16 and torch.allclose(narrow.float(), src, atol=1e-2)
    pool.close()

// A fixed ring of pinned staging slots in front of the transfer engine: the slot-ring form of the
// streaming boundary.  I/O workers fill slots on the host (rw4_ring_stage, or a read straight into
// the address rw4_ring_slot returns); the forward thread submits a slot's bytes to a device buffer
// (rw4_ring_submit: a chunked send over the engine's copy streams, optionally recording the
// caller's event behind it) and makes compute wait for the copies on the device
// (rw4_ring_wait_compute).  A slot is refused for staging while its last submit is in flight, so a
// worker never overwrites bytes a copy is still reading -- the lease rule of the reference's
// BufferLease (rocketllm/streaming/staging.py:33-66) applied per slot -- and refused for submitting
// (and for a second stage) while a stage into it is still copying on the host, so a copy never
// reads bytes a worker is still writing.  rw4_ring_slot hands out the slot's address for direct
// reads: the caller owns that slot until it submits it, and must not stage into it meanwhile.  Built on rw4_pool_* (the
// slots are leased once) and rw4_xfer_* (the copies).
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "rw4_common.cuh"

struct rw4_ring {
  std::mutex mu;
  rw4_pool* pool = nullptr;
  rw4_xfer* xfer = nullptr;
  cudaStream_t signal = nullptr;  // records the caller's done events behind a send
  int device = 0;
  size_t slot_bytes = 0;
  std::vector<void*> host;
  std::vector<int32_t> lease;
  std::vector<uint64_t> ticket;  // last submit of each slot (0: none)
  std::vector<uint8_t> staging;  // 1 while rw4_ring_stage copies into the slot (host memcpy)
};

namespace {

using rw4::fail;

constexpr size_t kChunkBytes = size_t(16) << 20;

size_t pool_class(size_t bytes) {  // the pool's power-of-two size classes (>= 64 KiB)
  size_t c = size_t(1) << 16;
  while (c < bytes) c <<= 1;
  return c;
}

void teardown(rw4_ring* r) {
  if (r->xfer) rw4_xfer_destroy(r->xfer);  // waits for the copies still in flight
  if (r->pool) {
    for (int32_t id : r->lease) rw4_pool_release(r->pool, id);
    rw4_pool_destroy(r->pool);
  }
  if (r->signal) cudaStreamDestroy(r->signal);
  delete r;
}

// 1 if the slot has no submit in flight, 0 if it has, < 0 on error (caller holds the lock).
int slot_free(rw4_ring* r, int slot) {
  if (!r->ticket[slot]) return 1;
  const int q = rw4_xfer_query(r->xfer, r->ticket[slot]);
  if (q == 1) r->ticket[slot] = 0;
  return q;
}

}  // namespace

extern "C" int rw4_ring_create(size_t slot_bytes, int32_t slots, int32_t copy_streams,
                               rw4_ring** out) {
  if (!out) return fail(RW4_EINVAL, "rw4_ring_create: null output");
  *out = nullptr;
  if (slot_bytes == 0 || slots < 1 || slots > 64 || copy_streams < 1 || copy_streams > 8)
    return fail(RW4_EINVAL, "rw4_ring_create: %zu-byte slots x %d, %d copy streams (1..64 slots, "
                "1..8 streams)", slot_bytes, slots, copy_streams);
  auto* r = new (std::nothrow) rw4_ring();
  if (!r) return fail(RW4_ENOMEM, "rw4_ring_create: out of host memory");
  cudaGetDevice(&r->device);
  r->slot_bytes = slot_bytes;
  int st = rw4_pool_create(pool_class(slot_bytes) * (size_t)slots, &r->pool);
  for (int s = 0; st == RW4_OK && s < slots; ++s) {
    int32_t id = -1;
    void* h = nullptr;
    st = rw4_pool_lease(r->pool, slot_bytes, &id, &h);
    if (st == RW4_OK) {
      r->lease.push_back(id);
      r->host.push_back(h);
    }
  }
  if (st == RW4_OK) st = rw4_xfer_create(r->device, copy_streams, &r->xfer);
  if (st == RW4_OK)
    st = rw4::cuda_status(cudaStreamCreateWithFlags(&r->signal, cudaStreamNonBlocking),
                          "rw4_ring_create: stream");
  if (st != RW4_OK) {
    teardown(r);
    return st;
  }
  r->ticket.assign(slots, 0);
  r->staging.assign(slots, 0);
  *out = r;
  return RW4_OK;
}

extern "C" int rw4_ring_destroy(rw4_ring* ring) {
  if (ring) teardown(ring);
  return RW4_OK;
}

extern "C" int rw4_ring_slot(rw4_ring* ring, int32_t slot, void** host) {
  if (!ring || !host) return fail(RW4_EINVAL, "rw4_ring_slot: null argument");
  if (slot < 0 || slot >= (int)ring->host.size())
    return fail(RW4_EINVAL, "rw4_ring_slot: slot %d of %zu", slot, ring->host.size());
  *host = ring->host[slot];
  return RW4_OK;
}

extern "C" int rw4_ring_stage(rw4_ring* ring, int32_t slot, size_t offset, const void* src,
                              size_t n) {
  if (!ring || (n && !src)) return fail(RW4_EINVAL, "rw4_ring_stage: null argument");
  if (slot < 0 || slot >= (int)ring->host.size())
    return fail(RW4_EINVAL, "rw4_ring_stage: slot %d of %zu", slot, ring->host.size());
  if (offset > ring->slot_bytes || n > ring->slot_bytes - offset)
    return fail(RW4_EINVAL, "rw4_ring_stage: %zu bytes at %zu overflow a %zu-byte slot", n, offset,
                ring->slot_bytes);
  {
    std::lock_guard<std::mutex> lock(ring->mu);
    const int f = slot_free(ring, slot);
    if (f < 0) return f;
    if (f == 0) return fail(RW4_EBUSY, "rw4_ring_stage: slot %d is still being copied", slot);
    if (ring->staging[slot])
      return fail(RW4_EBUSY, "rw4_ring_stage: slot %d is being staged by another caller", slot);
    ring->staging[slot] = 1;   // the memcpy below runs without the lock
  }
  if (n) std::memcpy(static_cast<char*>(ring->host[slot]) + offset, src, n);
  std::lock_guard<std::mutex> lock(ring->mu);
  ring->staging[slot] = 0;
  return RW4_OK;
}

extern "C" int rw4_ring_submit(rw4_ring* ring, int32_t slot, void* dst, size_t n,
                               void* done_event) {
  if (!ring || (n && !dst)) return fail(RW4_EINVAL, "rw4_ring_submit: null argument");
  if (slot < 0 || slot >= (int)ring->host.size())
    return fail(RW4_EINVAL, "rw4_ring_submit: slot %d of %zu", slot, ring->host.size());
  if (n > ring->slot_bytes)
    return fail(RW4_EINVAL, "rw4_ring_submit: %zu bytes from a %zu-byte slot", n,
                ring->slot_bytes);
  std::lock_guard<std::mutex> lock(ring->mu);
  if (ring->staging[slot])
    return fail(RW4_EBUSY, "rw4_ring_submit: slot %d is still being staged", slot);
  const int f = slot_free(ring, slot);
  if (f < 0) return f;
  if (f == 0) return fail(RW4_EBUSY, "rw4_ring_submit: slot %d is still being copied", slot);
  uint64_t t = 0;
  int st = rw4_xfer_send(ring->xfer, dst, ring->host[slot], n, kChunkBytes, nullptr, &t);
  if (st) return st;
  ring->ticket[slot] = t;
  if (done_event) {
    st = rw4_xfer_wait(ring->xfer, t, ring->signal);
    if (st) return st;
    st = rw4::cuda_status(cudaEventRecord(static_cast<cudaEvent_t>(done_event), ring->signal),
                          "rw4_ring_submit: done event");
  }
  return st;
}

extern "C" int rw4_ring_wait_compute(rw4_ring* ring, void* stream) {
  if (!ring) return fail(RW4_EINVAL, "rw4_ring_wait_compute: null ring");
  std::lock_guard<std::mutex> lock(ring->mu);
  for (size_t s = 0; s < ring->ticket.size(); ++s) {
    if (!ring->ticket[s]) continue;
    const int st = rw4_xfer_wait(ring->xfer, ring->ticket[s], stream);
    if (st) return st;
  }
  return RW4_OK;
}

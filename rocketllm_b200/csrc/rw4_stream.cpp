// Streaming: pinned host staging pool and the host->device transfer engine (C ABI in rw4.h).
//
// Pool (replaces rocketllm/streaming/staging.py:80-273 HostStagingPool): pinned buffers allocated
// once per power-of-two size class (>= 64 KiB, staging.py:112-117) and reused; a lease hands out the
// smallest free buffer that fits (staging.py:229-233), so a big buffer stays for big layers; a
// lease that does not fit the budget fails (the caller falls back to a transient buffer, as
// staging.py:218-227 does).
//
// Transfer engine (replaces rocketllm/streaming/transfer.py:124-292 WeightTransfer): the reference
// issues one host.to(device) per layer on one copy stream.  Here a send is split into chunks that go
// round-robin onto several non-blocking copy streams, so the H2D DMA engines work on one layer in
// parallel, and its completion is one event per stream used; compute waits on those events on the
// device (cudaStreamWaitEvent), never on the host (transfer.py:222-240).  Before overwriting a
// device buffer that compute may still read, the copy streams can first wait for the compute
// stream (`after_stream`), which is what lets a double-buffered layer slot be refilled while the
// other slot is being computed on.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <deque>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

#include "rw4_common.cuh"

namespace {

struct PoolBuf {
  void* host = nullptr;
  size_t bytes = 0;
  bool leased = false;
};

size_t size_class(size_t bytes) {
  size_t c = size_t(1) << 16;
  while (c < bytes) c <<= 1;
  return c;
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

struct Ticket {
  std::vector<cudaEvent_t> events;
};

}  // namespace

struct rw4_pool {
  std::mutex mu;
  size_t budget = 0;
  size_t resident = 0;
  std::vector<PoolBuf> bufs;
  uint64_t hits = 0, misses = 0;
};

struct rw4_xfer {
  int device = 0;
  std::vector<cudaStream_t> streams;
  std::mutex mu;
  uint64_t next_ticket = 1;
  size_t rr = 0;
  std::unordered_map<uint64_t, Ticket> live;
  std::vector<cudaEvent_t> spare;
  cudaEvent_t order_event = nullptr;
  uint64_t sends = 0, bytes = 0, chunks = 0;
};

using rw4::fail;

extern "C" int rw4_pool_create(size_t budget_bytes, rw4_pool** out) {
  if (!out) return fail(RW4_EINVAL, "rw4_pool_create: null output");
  auto* p = new (std::nothrow) rw4_pool();
  if (!p) return fail(RW4_ENOMEM, "rw4_pool_create: out of host memory");
  p->budget = budget_bytes;
  *out = p;
  return RW4_OK;
}

extern "C" int rw4_pool_destroy(rw4_pool* pool) {
  if (!pool) return RW4_OK;
  for (auto& b : pool->bufs)
    if (b.host) cudaFreeHost(b.host);
  delete pool;
  return RW4_OK;
}

extern "C" int rw4_pool_lease(rw4_pool* pool, size_t bytes, int32_t* id, void** host) {
  if (!pool || !id || !host) return fail(RW4_EINVAL, "rw4_pool_lease: null argument");
  std::lock_guard<std::mutex> lock(pool->mu);
  int best = -1;
  for (int i = 0; i < (int)pool->bufs.size(); ++i) {
    const PoolBuf& b = pool->bufs[i];
    if (!b.leased && b.bytes >= bytes && (best < 0 || b.bytes < pool->bufs[best].bytes)) best = i;
  }
  if (best >= 0) {
    pool->bufs[best].leased = true;
    pool->hits++;
    *id = best;
    *host = pool->bufs[best].host;
    return RW4_OK;
  }
  const size_t cls = size_class(bytes);
  if (pool->resident + cls > pool->budget) {
    pool->misses++;
    return fail(RW4_EBUSY, "rw4_pool_lease: %zu bytes would exceed the pinned budget %zu", cls,
                pool->budget);
  }
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, cls, cudaHostAllocPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    pool->misses++;
    return fail(RW4_ENOMEM, "rw4_pool_lease: cudaHostAlloc(%zu): %s", cls, cudaGetErrorString(e));
  }
  PoolBuf b;
  b.host = h;
  b.bytes = cls;
  b.leased = true;
  pool->bufs.push_back(b);
  pool->resident += cls;
  pool->misses++;
  *id = (int32_t)pool->bufs.size() - 1;
  *host = h;
  return RW4_OK;
}

extern "C" int rw4_pool_release(rw4_pool* pool, int32_t id) {
  if (!pool) return fail(RW4_EINVAL, "rw4_pool_release: null pool");
  std::lock_guard<std::mutex> lock(pool->mu);
  if (id < 0 || id >= (int)pool->bufs.size()) return fail(RW4_EINVAL, "rw4_pool_release: bad id %d", id);
  pool->bufs[id].leased = false;
  return RW4_OK;
}

extern "C" int rw4_pool_stats(rw4_pool* pool, uint64_t* resident, int32_t* buffers,
                              int32_t* leased, uint64_t* hits, uint64_t* misses) {
  if (!pool) return fail(RW4_EINVAL, "rw4_pool_stats: null pool");
  std::lock_guard<std::mutex> lock(pool->mu);
  int n = 0;
  for (auto& b : pool->bufs) n += b.leased;
  if (resident) *resident = pool->resident;
  if (buffers) *buffers = (int32_t)pool->bufs.size();
  if (leased) *leased = n;
  if (hits) *hits = pool->hits;
  if (misses) *misses = pool->misses;
  return RW4_OK;
}

// ---- transfer engine ---------------------------------------------------------------------------

namespace {

cudaEvent_t take_event(rw4_xfer* x) {
  if (!x->spare.empty()) {
    cudaEvent_t e = x->spare.back();
    x->spare.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  return e;
}

bool ticket_done(const Ticket& t) {
  for (cudaEvent_t e : t.events) {
    cudaError_t r = cudaEventQuery(e);
    if (r == cudaErrorNotReady) return false;
    if (r != cudaSuccess) cudaGetLastError();
  }
  return true;
}

// Recycle the events of completed tickets (caller holds the lock).
void harvest(rw4_xfer* x, uint64_t keep = 0) {
  for (auto it = x->live.begin(); it != x->live.end();) {
    if (it->first != keep && ticket_done(it->second)) {
      for (cudaEvent_t e : it->second.events) x->spare.push_back(e);
      it = x->live.erase(it);
    } else {
      ++it;
    }
  }
}

}  // namespace

extern "C" int rw4_xfer_create(int32_t device, int32_t copy_streams, rw4_xfer** out) {
  if (!out) return fail(RW4_EINVAL, "rw4_xfer_create: null output");
  if (copy_streams < 1 || copy_streams > 8)
    return fail(RW4_EINVAL, "rw4_xfer_create: copy_streams %d not in 1..8", copy_streams);
  auto* x = new (std::nothrow) rw4_xfer();
  if (!x) return fail(RW4_ENOMEM, "rw4_xfer_create: out of host memory");
  x->device = device;
  DeviceGuard g(device);
  for (int i = 0; i < copy_streams; ++i) {
    cudaStream_t s = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      for (auto t : x->streams) cudaStreamDestroy(t);
      delete x;
      return rw4::cuda_status(e, "rw4_xfer_create: stream");
    }
    x->streams.push_back(s);
  }
  if (cudaEventCreateWithFlags(&x->order_event, cudaEventDisableTiming) != cudaSuccess) {
    for (auto t : x->streams) cudaStreamDestroy(t);
    delete x;
    return fail(RW4_ECUDA, "rw4_xfer_create: event");
  }
  *out = x;
  return RW4_OK;
}

extern "C" int rw4_xfer_destroy(rw4_xfer* x) {
  if (!x) return RW4_OK;
  DeviceGuard g(x->device);
  for (auto s : x->streams) cudaStreamSynchronize(s);
  for (auto& kv : x->live)
    for (cudaEvent_t e : kv.second.events) cudaEventDestroy(e);
  for (cudaEvent_t e : x->spare) cudaEventDestroy(e);
  if (x->order_event) cudaEventDestroy(x->order_event);
  for (auto s : x->streams) cudaStreamDestroy(s);
  delete x;
  return RW4_OK;
}

extern "C" int rw4_xfer_send(rw4_xfer* x, void* dst, const void* src, size_t n,
                             size_t chunk_bytes, void* after_stream, uint64_t* ticket) {
  if (!x || !ticket) return fail(RW4_EINVAL, "rw4_xfer_send: null argument");
  if (n && (!dst || !src)) return fail(RW4_EINVAL, "rw4_xfer_send: null buffer");
  std::lock_guard<std::mutex> lock(x->mu);
  DeviceGuard g(x->device);
  harvest(x);
  const int ns = (int)x->streams.size();
  if (after_stream) {
    int st = rw4::cuda_status(cudaEventRecord(x->order_event, rw4::as_stream(after_stream)),
                              "rw4_xfer_send: order event");
    if (st) return st;
    for (auto s : x->streams) {
      st = rw4::cuda_status(cudaStreamWaitEvent(s, x->order_event, 0), "rw4_xfer_send: wait");
      if (st) return st;
    }
  }
  const size_t chunk = chunk_bytes ? chunk_bytes : (n ? n : 1);
  std::vector<bool> used(ns, false);
  size_t off = 0;
  uint64_t nchunks = 0;
  while (off < n) {
    const size_t len = std::min(chunk, n - off);
    const int si = (int)(x->rr++ % ns);
    cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dst) + off,
                                    static_cast<const char*>(src) + off, len,
                                    cudaMemcpyHostToDevice, x->streams[si]);
    if (e != cudaSuccess) return rw4::cuda_status(e, "rw4_xfer_send: cudaMemcpyAsync");
    used[si] = true;
    off += len;
    nchunks++;
  }
  Ticket t;
  for (int si = 0; si < ns; ++si) {
    if (!used[si] && n) continue;
    if (!n && si) break;  // an empty send completes behind stream 0
    cudaEvent_t e = take_event(x);
    if (!e) return fail(RW4_ECUDA, "rw4_xfer_send: cannot create event");
    int st = rw4::cuda_status(cudaEventRecord(e, x->streams[si]), "rw4_xfer_send: record");
    if (st) {
      x->spare.push_back(e);
      return st;
    }
    t.events.push_back(e);
  }
  const uint64_t id = x->next_ticket++;
  x->live.emplace(id, std::move(t));
  x->sends++;
  x->bytes += n;
  x->chunks += nchunks;
  *ticket = id;
  return RW4_OK;
}

extern "C" int rw4_xfer_wait(rw4_xfer* x, uint64_t ticket, void* stream) {
  if (!x) return fail(RW4_EINVAL, "rw4_xfer_wait: null engine");
  std::lock_guard<std::mutex> lock(x->mu);
  auto it = x->live.find(ticket);
  if (it == x->live.end()) {
    if (ticket == 0 || ticket >= x->next_ticket)
      return fail(RW4_EINVAL, "rw4_xfer_wait: unknown ticket %llu", (unsigned long long)ticket);
    return RW4_OK;  // already completed and harvested
  }
  for (cudaEvent_t e : it->second.events) {
    int st = rw4::cuda_status(cudaStreamWaitEvent(rw4::as_stream(stream), e, 0),
                              "rw4_xfer_wait");
    if (st) return st;
  }
  return RW4_OK;
}

extern "C" int rw4_xfer_query(rw4_xfer* x, uint64_t ticket) {
  if (!x) return fail(RW4_EINVAL, "rw4_xfer_query: null engine");
  std::lock_guard<std::mutex> lock(x->mu);
  auto it = x->live.find(ticket);
  if (it == x->live.end()) {
    if (ticket == 0 || ticket >= x->next_ticket)
      return fail(RW4_EINVAL, "rw4_xfer_query: unknown ticket %llu", (unsigned long long)ticket);
    return 1;
  }
  if (!ticket_done(it->second)) return 0;
  for (cudaEvent_t e : it->second.events) x->spare.push_back(e);
  x->live.erase(it);
  return 1;
}

extern "C" int rw4_xfer_sync(rw4_xfer* x, uint64_t ticket, int64_t timeout_ms) {
  if (!x) return fail(RW4_EINVAL, "rw4_xfer_sync: null engine");
  const auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  while (true) {
    const int r = rw4_xfer_query(x, ticket);
    if (r != 0) return r < 0 ? r : RW4_OK;
    if (timeout_ms >= 0) {
      const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
      if (el > timeout_ms)
        return fail(RW4_ETIMEOUT, "rw4_xfer_sync: ticket %llu not complete after %lld ms",
                    (unsigned long long)ticket, (long long)timeout_ms);
    }
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

extern "C" int rw4_xfer_stats(rw4_xfer* x, uint64_t* sends, uint64_t* bytes, uint64_t* chunks,
                              int32_t* in_flight) {
  if (!x) return fail(RW4_EINVAL, "rw4_xfer_stats: null engine");
  std::lock_guard<std::mutex> lock(x->mu);
  harvest(x);
  if (sends) *sends = x->sends;
  if (bytes) *bytes = x->bytes;
  if (chunks) *chunks = x->chunks;
  if (in_flight) *in_flight = (int32_t)x->live.size();
  return RW4_OK;
}

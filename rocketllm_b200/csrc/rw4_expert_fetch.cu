// Device-side routing into the expert cache: after the router, a residency kernel decides which
// routed experts are resident, assigns cache slots to the others (least recently used first, or by
// the reference's LFU with aging in the _lfu form; never a slot this layer's routed experts hold)
// and lists them; a copy kernel then moves exactly those
// experts' blobs from mapped pinned host memory into their slots over PCIe.  The grouped GEMV finds
// each expert through the slot index the residency kernel wrote (rw4_moe_grouped_slots), so no
// host step waits for the routing -- the reference reads the routed set back to the host once per
// MoE layer (rocketllm/moe/router.py:88-93, rocketllm/base.py:1375-1464) and issues the reads from
// there (rocketllm/moe/expert_cache.py:261-316).
//
// State (device, owned by the caller): where[L*E] (slot of layer l's expert e, or -1), owner[S]
// (key l*E + e held by a slot, or -1), stamp[S] (use clock), clock[1], counters[2] (hits,
// fetches); the LFU form keeps uses[L*E], admitted[L*E] and state[3] instead of stamp and clock
// (rw4_residency.cuh).
#include <cuda_runtime.h>

#include "rw4_common.cuh"
#include "rw4_residency.cuh"
#include "rw4_tma.cuh"

namespace {

using namespace rw4;

// One thread: the routed set is at most E (<= 4096) experts and the cache at most a few hundred
// slots; a single thread keeps the policy sequential and deterministic.
__global__ void expert_residency_kernel(const int32_t* __restrict__ offsets, int E, int layer,
                                        int32_t* __restrict__ where, int32_t* __restrict__ owner,
                                        int32_t* __restrict__ stamp, int S,
                                        int32_t* __restrict__ clock,
                                        int32_t* __restrict__ slot_of,
                                        int32_t* __restrict__ copy_expert,
                                        int32_t* __restrict__ copy_slot,
                                        int32_t* __restrict__ ncopy,
                                        unsigned long long* __restrict__ counters,
                                        unsigned int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int t = ++clock[0];
  const int base = layer * E;
  unsigned long long hits = 0, fetches = 0;
  // routed experts already resident: claim their slots for this call
  for (int e = 0; e < E; ++e) {
    slot_of[e] = -1;
    if (offsets[e + 1] <= offsets[e]) continue;
    const int s = where[base + e];
    if (s >= 0 && s < S && owner[s] == base + e) {
      slot_of[e] = s;
      stamp[s] = t;
      ++hits;
    }
  }
  // the others: a free slot, else the least recently used one not claimed by this call
  int n = 0;
  for (int e = 0; e < E; ++e) {
    if (offsets[e + 1] <= offsets[e] || slot_of[e] >= 0) continue;
    int best = -1;
    for (int s = 0; s < S; ++s) {
      if (owner[s] < 0) {
        best = s;
        break;
      }
      if (stamp[s] != t && (best < 0 || stamp[s] < stamp[best])) best = s;
    }
    if (best < 0) {  // fewer slots than this layer's routed experts
      atomicOr(status, RW4_DEVERR_SLOT);
      continue;
    }
    const int old = owner[best];
    if (old >= 0) where[old] = -1;
    owner[best] = base + e;
    where[base + e] = best;
    stamp[best] = t;
    slot_of[e] = best;
    copy_expert[n] = e;
    copy_slot[n] = best;
    ++n;
    ++fetches;
  }
  ncopy[0] = n;
  counters[0] += hits;
  counters[1] += fetches;
}

// The same step under the reference's LFU with aging (rw4_residency.cuh); one thread.
__global__ void expert_residency_lfu_kernel(const int32_t* __restrict__ offsets, int E, int layer,
                                            int keys, int32_t* __restrict__ where,
                                            int32_t* __restrict__ owner, int S,
                                            double* __restrict__ uses,
                                            int32_t* __restrict__ admitted,
                                            int64_t* __restrict__ state, int64_t aging_interval,
                                            int32_t* __restrict__ slot_of,
                                            int32_t* __restrict__ copy_expert,
                                            int32_t* __restrict__ copy_slot,
                                            int32_t* __restrict__ ncopy,
                                            uint64_t* __restrict__ counters,
                                            unsigned int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (lfu_residency_step(offsets, E, layer, keys, where, owner, S, uses, admitted, state,
                         aging_interval, slot_of, copy_expert, copy_slot, ncopy, counters))
    atomicOr(status, RW4_DEVERR_SLOT);
}

// grid (chunks, E): block (c, i) copies chunk c of the i-th listed expert (if there is one);
// 16-byte loads from the mapped host blob (four independent loads in flight per thread: PCIe
// latency is microseconds), 16-byte stores into the slot.
__global__ void __launch_bounds__(256)
    expert_copy_kernel(const int32_t* __restrict__ copy_expert,
                       const int32_t* __restrict__ copy_slot, const int32_t* __restrict__ ncopy,
                       int layer, int E, const unsigned long long* __restrict__ host_blobs,
                       int64_t blob_bytes, uint8_t* __restrict__ slots, int64_t slot_bytes,
                       int S) {
  const int i = blockIdx.y;
  if (i >= ncopy[0]) return;
  const int e = copy_expert[i];
  const int s = copy_slot[i];
  if (e < 0 || e >= E || s < 0 || s >= S) return;
  const uint4* src = reinterpret_cast<const uint4*>(host_blobs[(int64_t)layer * E + e]);
  uint4* dst = reinterpret_cast<uint4*>(slots + (int64_t)s * slot_bytes);
  const int64_t vecs = blob_bytes / 16;
  const int64_t per = (vecs + gridDim.x - 1) / gridDim.x;
  const int64_t beg = (int64_t)blockIdx.x * per;
  const int64_t end = beg + per < vecs ? beg + per : vecs;
  constexpr int kUnroll = 4;
  const int64_t step = blockDim.x;
  int64_t v = beg + threadIdx.x;
  for (; v + (kUnroll - 1) * step < end; v += kUnroll * step) {
    uint4 r[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) r[u] = ldg_stream_u4(src + v + u * step);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) dst[v + u * step] = r[u];
  }
  for (; v < end; v += step) dst[v] = ldg_stream_u4(src + v);
}

}  // namespace

extern "C" int rw4_host_ptr_device(const void* host, void** device_ptr) {
  if (!host || !device_ptr) return fail(RW4_EINVAL, "rw4_host_ptr_device: null pointer");
  *device_ptr = nullptr;
  cudaPointerAttributes attr;
  cudaError_t err = cudaPointerGetAttributes(&attr, host);
  if (err != cudaSuccess) return cuda_status(err, "rw4_host_ptr_device");
  if (attr.type != cudaMemoryTypeHost || !attr.devicePointer)
    return fail(RW4_EINVAL, "rw4_host_ptr_device: %p is not pinned host memory mapped into the "
                "device address space", host);
  *device_ptr = attr.devicePointer;
  return RW4_OK;
}

extern "C" int rw4_expert_residency(const int32_t* offsets, int32_t E, int32_t layer,
                                    int32_t* where, int32_t* owner, int32_t* stamp, int32_t S,
                                    int32_t* clock, int32_t* slot_of, int32_t* copy_expert,
                                    int32_t* copy_slot, int32_t* ncopy, uint64_t* counters,
                                    void* stream) {
  if (E < 1 || E > 4096 || S < 1 || layer < 0)
    return fail(RW4_EINVAL, "rw4_expert_residency: E=%d S=%d layer=%d", E, S, layer);
  if (!offsets || !where || !owner || !stamp || !clock || !slot_of || !copy_expert ||
      !copy_slot || !ncopy || !counters)
    return fail(RW4_EINVAL, "rw4_expert_residency: null pointer");
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "rw4_expert_residency: device status word unavailable");
  expert_residency_kernel<<<1, 32, 0, as_stream(stream)>>>(
      offsets, E, layer, where, owner, stamp, S, clock, slot_of, copy_expert, copy_slot, ncopy,
      reinterpret_cast<unsigned long long*>(counters), status);
  return launch_status("rw4_expert_residency launch");
}

namespace {

int check_lfu_args(const char* who, const int32_t* offsets, int32_t E, int32_t layer, int32_t keys,
                   const int32_t* where, const int32_t* owner, int32_t S, const double* uses,
                   const int32_t* admitted, const int64_t* state, int64_t aging_interval,
                   const int32_t* slot_of, const int32_t* copy_expert, const int32_t* copy_slot,
                   const int32_t* ncopy, const uint64_t* counters) {
  if (E < 1 || E > 4096 || S < 1 || layer < 0 || aging_interval < 1 ||
      (int64_t)(layer + 1) * E > keys)
    return fail(RW4_EINVAL, "%s: E=%d S=%d layer=%d keys=%d aging_interval=%lld", who, E, S, layer,
                keys, (long long)aging_interval);
  if (!offsets || !where || !owner || !uses || !admitted || !state || !slot_of || !copy_expert ||
      !copy_slot || !ncopy || !counters)
    return fail(RW4_EINVAL, "%s: null pointer", who);
  return RW4_OK;
}

}  // namespace

extern "C" int rw4_expert_residency_lfu(const int32_t* offsets, int32_t E, int32_t layer,
                                        int32_t keys, int32_t* where, int32_t* owner, int32_t S,
                                        double* uses, int32_t* admitted, int64_t* state,
                                        int64_t aging_interval, int32_t* slot_of,
                                        int32_t* copy_expert, int32_t* copy_slot, int32_t* ncopy,
                                        uint64_t* counters, void* stream) {
  const int st = check_lfu_args("rw4_expert_residency_lfu", offsets, E, layer, keys, where, owner,
                                S, uses, admitted, state, aging_interval, slot_of, copy_expert,
                                copy_slot, ncopy, counters);
  if (st) return st;
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "rw4_expert_residency_lfu: device status word unavailable");
  expert_residency_lfu_kernel<<<1, 32, 0, as_stream(stream)>>>(
      offsets, E, layer, keys, where, owner, S, uses, admitted, state, aging_interval, slot_of,
      copy_expert, copy_slot, ncopy, counters, status);
  return launch_status("rw4_expert_residency_lfu launch");
}

extern "C" int rw4_expert_residency_lfu_host(const int32_t* offsets, int32_t E, int32_t layer,
                                             int32_t keys, int32_t* where, int32_t* owner,
                                             int32_t S, double* uses, int32_t* admitted,
                                             int64_t* state, int64_t aging_interval,
                                             int32_t* slot_of, int32_t* copy_expert,
                                             int32_t* copy_slot, int32_t* ncopy,
                                             uint64_t* counters) {
  const int st = check_lfu_args("rw4_expert_residency_lfu_host", offsets, E, layer, keys, where,
                                owner, S, uses, admitted, state, aging_interval, slot_of,
                                copy_expert, copy_slot, ncopy, counters);
  if (st) return st;
  const int unplaced = lfu_residency_step(offsets, E, layer, keys, where, owner, S, uses, admitted,
                                          state, aging_interval, slot_of, copy_expert, copy_slot,
                                          ncopy, counters);
  if (unplaced)
    return fail(RW4_EINVAL, "rw4_expert_residency_lfu_host: %d routed experts of layer %d found no "
                "slot (%d slots, all held by the layer's routed experts)", unplaced, layer, S);
  return RW4_OK;
}

extern "C" int rw4_expert_copy(const int32_t* copy_expert, const int32_t* copy_slot,
                               const int32_t* ncopy, int32_t layer, int32_t E,
                               const uint64_t* host_blobs, int64_t blob_bytes, uint8_t* slots,
                               int64_t slot_bytes, int32_t S, int32_t ctas_per_expert,
                               void* stream) {
  if (E < 1 || E > 65535 || S < 1 || layer < 0 || blob_bytes <= 0 || blob_bytes % 16 ||
      blob_bytes > slot_bytes || slot_bytes % 16 || ctas_per_expert < 1)
    return fail(RW4_EINVAL, "rw4_expert_copy: E=%d S=%d blob=%lld slot=%lld", E, S,
                (long long)blob_bytes, (long long)slot_bytes);
  if (!copy_expert || !copy_slot || !ncopy || !host_blobs || !slots || !aligned(slots, 16))
    return fail(RW4_EINVAL, "rw4_expert_copy: null or misaligned pointer");
  dim3 grid(ctas_per_expert, E);
  expert_copy_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      copy_expert, copy_slot, ncopy, layer, E,
      reinterpret_cast<const unsigned long long*>(host_blobs), blob_bytes, slots, slot_bytes, S);
  return launch_status("rw4_expert_copy launch");
}

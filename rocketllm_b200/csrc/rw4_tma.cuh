// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a, with bounded waits.
//
// Every wait on an mbarrier gives up after kWaitLimitNs of %globaltimer time, records
// RW4_DEVERR_TIMEOUT in the library's device status word (passed to kernels as a pointer) and
// lets the kernel unwind, so a protocol error can never hang the GPU; rw4_device_status() reads
// (and optionally clears) that word.
// Every CTA fetches its own tiles with plain (per-CTA) TMA loads.
#pragma once

#include <cuda.h>

#include "rw4_common.cuh"

#define RW4_DEVERR_TIMEOUT 1u
#define RW4_DEVERR_TMEM 2u
#define RW4_DEVERR_ROWS 4u  // a grouped launch saw an expert with more rows than max_rows
#define RW4_DEVERR_SLOT 8u  // a routed expert had no expert-cache slot (device-side residency)

namespace rw4 {

// Device address of the status word (bit set) on the current device; resolved once per device.
unsigned int* device_status_ptr();

constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// try_wait with a suspend-time hint: a thread whose phase has not completed is suspended by the
// hardware (resumed when the phase completes or after at most kSuspendHintNs) instead of spinning,
// so waiting producer / MMA / consumer warps do not take issue slots from working warps.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait for the phase with parity `parity` to complete; false (and the status bit set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(status, RW4_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// 2-D tiled TMA load into shared memory, completion signalled on `bar` (complete_tx bytes).
// x is the innermost coordinate in elements; x * elemsize must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Same with an L2 eviction-priority hint (createpolicy) for data read exactly once.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// Prefetch a 2-D tile into L2 only (no shared-memory write, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// For data many CTAs re-read over the kernel's life (an activation matrix that every weight tile
// streams against): kept in L2 ahead of evict-first / normal lines.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- host side -------------------------------------------------------------------------------

// Encode a 2-D row-major tensor map: `rows` x `cols` elements of `elem_bytes`, row pitch
// `row_bytes`, box `box_rows` x `box_cols`.  Returns RW4_OK or an error (message recorded).
int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                       int elem_bytes, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                       uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle);

}  // namespace rw4

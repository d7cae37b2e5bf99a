// One residency step of the expert cache under the reference's expert policy, LFU with aging
// (rocketllm/memory/cache.py: _touch 434-441, _age 443-453, _expert_victims 484-493, acquire
// 201-250).  Compiled for the device (the one-thread residency kernel) and for the host (the
// host-table entry point), from this one definition, so both make the same decisions bit for bit.
//
// For MoE layer `layer`, over its routed experts in ascending order (routed: offsets[e+1] >
// offsets[e]):
//   * resident (owner[where[key]] == key): a hit;
//   * else it takes the first free slot, else the slot of the resident expert with the smallest
//     aged use count, ties to the one admitted first, skipping every slot that holds one of this
//     layer's routed experts (one grouped launch reads them all); the victim is chosen before the
//     incoming use is counted, as acquire makes room before it touches; the expert is listed for
//     a copy (copy_expert / copy_slot) and, on its first admission ever, gets the next ordinal;
//   * then its use is counted: uses[key] += 1, and every aging_interval-th use halves every count.
// Counts and admission ordinals outlive an eviction (the expert's pinned host blob stays, as an
// entry demoted to the reference's host tier keeps them).  Counts are doubles, as the reference's
// Python floats, so the halving sequence matches it exactly.
//
// Tables (key = layer * E + e, keys = layers * E): where int32 [keys] (slot or -1), owner int32 [S]
// (key or -1), uses double [keys], admitted int32 [keys] (-1 until admitted), state int64 [3]
// (uses counted, experts admitted, agings), counters uint64 [2] (hits, fetches).  Returns how many
// routed experts found no slot (every slot holds one of this layer's routed experts); those keep
// slot_of[e] = -1 and are neither listed nor counted.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define RW4_HOST_DEVICE __host__ __device__
#else
#define RW4_HOST_DEVICE
#endif

namespace rw4 {

RW4_HOST_DEVICE inline int lfu_residency_step(const int32_t* offsets, int E, int layer, int keys,
                                              int32_t* where, int32_t* owner, int S, double* uses,
                                              int32_t* admitted, int64_t* state,
                                              int64_t aging_interval, int32_t* slot_of,
                                              int32_t* copy_expert, int32_t* copy_slot,
                                              int32_t* ncopy, uint64_t* counters) {
  const int base = layer * E;
  uint64_t hits = 0, fetches = 0;
  int n = 0, unplaced = 0;
  for (int e = 0; e < E; ++e) {
    slot_of[e] = -1;
    if (offsets[e + 1] <= offsets[e]) continue;
    const int key = base + e;
    int s = where[key];
    if (s >= 0 && s < S && owner[s] == key) {
      ++hits;
    } else {
      s = -1;
      for (int i = 0; i < S; ++i) {
        if (owner[i] < 0) {
          s = i;
          break;
        }
      }
      if (s < 0) {
        for (int i = 0; i < S; ++i) {
          const int k = owner[i];
          if (k < 0 || k >= keys) continue;
          if (k >= base && k < base + E && offsets[k - base + 1] > offsets[k - base]) continue;
          if (s >= 0) {
            const int b = owner[s];
            if (uses[k] > uses[b] || (uses[k] == uses[b] && admitted[k] >= admitted[b])) continue;
          }
          s = i;
        }
      }
      if (s < 0) {
        ++unplaced;
        continue;
      }
      const int old = owner[s];
      if (old >= 0 && old < keys) where[old] = -1;
      if (admitted[key] < 0) admitted[key] = static_cast<int32_t>(state[1]++);
      owner[s] = key;
      where[key] = s;
      copy_expert[n] = e;
      copy_slot[n] = s;
      ++n;
      ++fetches;
    }
    slot_of[e] = s;
    uses[key] += 1.0;
    if (++state[0] % aging_interval == 0) {
      for (int k = 0; k < keys; ++k) uses[k] *= 0.5;
      ++state[2];
    }
  }
  ncopy[0] = n;
  counters[0] += hits;
  counters[1] += fetches;
  return unplaced;
}

}  // namespace rw4

// Routed-expert (MoE) kernels: token->expert permutation, row gather, grouped RW4 GEMV over only the
// routed experts (optionally with the SwiGLU epilogue fused), and the weighted combine.
//
// They replace the per-expert Python loop of the model's experts forward (transformers
// models/mixtral/modeling_mixtral.py:62-98: one_hot -> where -> F.linear(gate_up) -> act * up ->
// F.linear(down) -> * weight -> index_add_) and the reference's full-width expert-row assembly
// (rocketllm/base.py:1435-1464), which builds a zero tensor for every expert even when a token
// routes to two.  Here an expert with no routed rows costs one CTA that reads two offsets and exits:
// its weights are never read.
#include <atomic>
#include <new>

#include "rw4_gemv_tma_body.cuh"

namespace {

using namespace rw4;

// ---- permute -----------------------------------------------------------------------------------

// One CTA.  Histogram with shared atomics, exclusive scan, then one warp scatters the slots in
// flat (t*k + j) order 32 at a time: __match_any_sync groups lanes with the same expert, the rank
// inside the group is the popcount of lower lanes, so the result is a stable counting sort.
__global__ void __launch_bounds__(1024)
    moe_permute_kernel(const int64_t* __restrict__ idx, int n, int E, int32_t* __restrict__ perm,
                       int32_t* __restrict__ inv, int32_t* __restrict__ offsets) {
  extern __shared__ int sh[];
  int* count = sh;          // [E]
  int* cursor = sh + E;     // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) count[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t e = idx[i];
    if (e >= 0 && e < E) atomicAdd(&count[e], 1);
    if (inv) inv[i] = -1;
    perm[i] = -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = run;
      cursor[e] = run;
      run += count[e];
    }
    offsets[E] = run;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const unsigned lane = threadIdx.x;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const bool live = i < n;
      int e = live ? (int)idx[i] : -1;
      const bool ok = live && e >= 0 && e < E;
      if (!ok) e = -1 - (int)lane;  // unique key: never groups with a real expert
      const unsigned grp = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(grp & ((1u << lane) - 1u));
      int pos = 0;
      if (ok) pos = cursor[e] + rank;
      __syncwarp();
      if (ok && rank == __popc(grp) - 1) cursor[e] += __popc(grp);  // last lane of the group
      if (ok) {
        perm[pos] = i;
        if (inv) inv[i] = pos;
      }
      __syncwarp();
    }
  }
}

// ---- gather ------------------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
    moe_gather_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ perm, int64_t rows,
                      int k, int64_t vecs, uint4* __restrict__ out) {
  const int64_t total = rows * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vecs, v = i - r * vecs;
    const int32_t slot = perm[r];
    out[i] = slot >= 0 ? x[(int64_t)(slot / k) * vecs + v] : make_uint4(0, 0, 0, 0);
  }
}

// ---- grouped GEMV ------------------------------------------------------------------------------

constexpr int kMaxExperts = 32;  // experts per launch (tensor maps travel as kernel parameters)

struct ExpertMaps {
  CUtensorMap codes[kMaxExperts];
  CUtensorMap scale[kMaxExperts];
  CUtensorMap zero[kMaxExperts];
};

// Every routed row count runs the same bf16 body (one-token steps included), so an expert's output
// for a token does not depend on how many other tokens it serves.
template <int NT, int R, int S, bool SWIGLU>
__global__ void __launch_bounds__(gemv_tma::kThreads)
    moe_grouped_kernel(const __grid_constant__ ExpertMaps maps, int e0,
                       const int32_t* __restrict__ offsets, const __nv_bfloat16* __restrict__ x,
                       int K, int n_out, int up_offset, __nv_bfloat16* __restrict__ y,
                       int64_t ldy, int max_rows, unsigned int* status) {
  const int z = blockIdx.z;
  const int beg = offsets[e0 + z];
  const int rows = offsets[e0 + z + 1] - beg;
  const int m0 = blockIdx.y * 16;
  // more rows than the launch's max_rows: flag it (those rows get no output)
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && rows > max_rows)
    atomicOr(status, RW4_DEVERR_ROWS);
  if (m0 >= rows) return;  // unrouted expert (or past its rows): no weight is read
  constexpr int kRowsPerCta = SWIGLU ? 8 * R : 16 * R;
  gemv_tma::body<NT, R, S, SWIGLU, 1, false>(&maps.codes[z], &maps.scale[z], &maps.zero[z],
                                             nullptr, nullptr, nullptr, x, beg + m0, 16,
                                             min(16, rows - m0), K,
                                   y + (int64_t)(beg + m0) * ldy, ldy, blockIdx.x * kRowsPerCta,
                                   n_out, up_offset, status);
}

template <int NT, int R, int S, bool SWIGLU>
int launch_grouped(const void* x, const int32_t* offsets, int E, int64_t max_rows,
                   const uint8_t* const* packed_e, const void* const* scale_e,
                   const void* const* zero_e, int K, int N, void* y, cudaStream_t stream) {
  using L = gemv_tma::Layout<R, S>;
  static_assert(L::kBars >= gemv_tma::kConsumers * L::BR * (16 * NT + 1) * 4,
                "the epilogue's reduction buffer must fit in the ring below the barriers");
  const int box_rows = SWIGLU ? L::BR / 2 : L::BR;
  const int n_out = SWIGLU ? N / 2 : N;
  const int rows_per_cta = SWIGLU ? L::BR / 2 : L::BR;
  const int G = K / 64;
  auto kern = moe_grouped_kernel<NT, R, S, SWIGLU>;
  const int smem = L::kX + 1024;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "moe_grouped: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "moe_grouped: device status word unavailable");
  ExpertMaps maps;
  for (int e0 = 0; e0 < E; e0 += kMaxExperts) {
    const int ne = E - e0 < kMaxExperts ? E - e0 : kMaxExperts;
    for (int z = 0; z < ne; ++z) {
      const int e = e0 + z;
      if (!packed_e[e] || !scale_e[e] || !zero_e[e])
        return fail(RW4_EINVAL, "rw4_moe_grouped: null weight pointer for expert %d", e);
      int st = make_tensor_map_2d(&maps.codes[z], packed_e[e], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1,
                                  N, K / 2, K / 2, box_rows, 128, CU_TENSOR_MAP_SWIZZLE_128B);
      if (st == RW4_OK)
        st = make_tensor_map_2d(&maps.scale[z], scale_e[e], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N,
                                G, (uint64_t)G * 2, box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (st == RW4_OK)
        st = make_tensor_map_2d(&maps.zero[z], zero_e[e], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N,
                                G, (uint64_t)G * 2, box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (st != RW4_OK) return st;
    }
    dim3 grid((n_out + rows_per_cta - 1) / rows_per_cta, (unsigned)((max_rows + 15) / 16), ne);
    kern<<<grid, gemv_tma::kThreads, smem, stream>>>(
        maps, e0, offsets, static_cast<const __nv_bfloat16*>(x), K, n_out, n_out,
        static_cast<__nv_bfloat16*>(y), n_out,
        (int)max_rows, status);
    int st = launch_status("rw4_moe_grouped launch");
    if (st) return st;
  }
  return RW4_OK;
}

// ---- grouped GEMV over an expert cache (device-side routing) -----------------------------------

// One tensor-map set per SLOT of a device expert cache, encoded once when the slots are allocated;
// the kernel finds expert e's weights through a device slot index (slot_of[e]) that a residency
// kernel wrote after the router, so no host step depends on the routing.  80 slots x 3 maps x 128
// bytes = 30 KB of kernel parameters (the limit is 32,764 bytes).
constexpr int kMaxSlots = 80;

struct SlotMaps {
  CUtensorMap codes[kMaxSlots];
  CUtensorMap scale[kMaxSlots];
  CUtensorMap zero[kMaxSlots];
};

template <int NT, int R, int S, bool SWIGLU>
__global__ void __launch_bounds__(gemv_tma::kThreads)
    moe_grouped_slots_kernel(const __grid_constant__ SlotMaps maps, int nslots,
                             const int32_t* __restrict__ slot_of,
                             const int32_t* __restrict__ offsets,
                             const __nv_bfloat16* __restrict__ x, int K, int n_out, int up_offset,
                             __nv_bfloat16* __restrict__ y, int64_t ldy, int max_rows,
                             unsigned int* status) {
  const int z = blockIdx.z;
  const int beg = offsets[z];
  const int rows = offsets[z + 1] - beg;
  const int m0 = blockIdx.y * 16;
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && rows > max_rows)
    atomicOr(status, RW4_DEVERR_ROWS);
  if (m0 >= rows) return;  // unrouted expert: neither its slot index nor its weights are read
  const int slot = slot_of[z];
  if (slot < 0 || slot >= nslots) {  // a routed expert without a slot: no output, flagged
    if (threadIdx.x == 0) atomicOr(status, RW4_DEVERR_SLOT);
    return;
  }
  constexpr int kRowsPerCta = SWIGLU ? 8 * R : 16 * R;
  gemv_tma::body<NT, R, S, SWIGLU, 1, false>(
      &maps.codes[slot], &maps.scale[slot], &maps.zero[slot], nullptr, nullptr, nullptr, x,
      beg + m0, 16,
      min(16, rows - m0), K, y + (int64_t)(beg + m0) * ldy, ldy, blockIdx.x * kRowsPerCta, n_out,
      up_offset, status);
}

}  // namespace

struct rw4_slot_maps {
  SlotMaps maps;
  int nslots;
  int K, N, act;
};

namespace {

template <int NT, int R, int S, bool SWIGLU>
int launch_grouped_slots(const rw4_slot_maps* sm, const int32_t* slot_of, const void* x,
                         const int32_t* offsets, int E, int64_t max_rows, void* y,
                         cudaStream_t stream) {
  using L = gemv_tma::Layout<R, S>;
  static_assert(L::kBars >= gemv_tma::kConsumers * L::BR * (16 * NT + 1) * 4,
                "the epilogue's reduction buffer must fit in the ring below the barriers");
  const int K = sm->K, N = sm->N;
  const int n_out = SWIGLU ? N / 2 : N;
  const int rows_per_cta = SWIGLU ? L::BR / 2 : L::BR;
  auto kern = moe_grouped_slots_kernel<NT, R, S, SWIGLU>;
  const int smem = L::kX + 1024;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "moe_grouped_slots: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "moe_grouped_slots: device status word unavailable");
  dim3 grid((n_out + rows_per_cta - 1) / rows_per_cta, (unsigned)((max_rows + 15) / 16), E);
  kern<<<grid, gemv_tma::kThreads, smem, stream>>>(
      sm->maps, sm->nslots, slot_of, offsets, static_cast<const __nv_bfloat16*>(x), K, n_out,
      n_out, static_cast<__nv_bfloat16*>(y), n_out, (int)max_rows, status);
  return launch_status("rw4_moe_grouped_slots launch");
}

// ---- combine -----------------------------------------------------------------------------------

// One thread per (token, 8 hidden values).  The k contributions are visited in ascending expert
// order and accumulated with a bf16 rounding after every product and every add -- the order and
// rounding of the reference loop (index_add_ into a bf16 tensor, expert by expert).
template <typename WT>
__global__ void __launch_bounds__(256)
    moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ inv,
                       const int64_t* __restrict__ topk_idx, const WT* __restrict__ w, int64_t T,
                       int k, int64_t H, __nv_bfloat16* __restrict__ out) {
  const int64_t vecs = H / 8;
  const int64_t total = T * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vecs, v = i - t * vecs;
    int order[8];
    int cnt = 0;
    for (int j = 0; j < k && j < 8; ++j) {
      int p = cnt++;
      const int64_t ej = topk_idx ? topk_idx[t * k + j] : j;
      while (p > 0 && (topk_idx ? topk_idx[t * k + order[p - 1]] : order[p - 1]) > ej) {
        order[p] = order[p - 1];
        --p;
      }
      order[p] = j;
    }
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int c = 0; c < cnt; ++c) {
      const int j = order[c];
      const int32_t row = inv[t * k + j];
      if (row < 0) continue;
      const float wj = (float)w[t * k + j];
      const uint4 raw = reinterpret_cast<const uint4*>(y + row * H)[v];
      const __nv_bfloat16* yv = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float prod = __bfloat162float(__float2bfloat16_rn(__bfloat162float(yv[e]) * wj));
        acc[e] = __bfloat162float(__float2bfloat16_rn(acc[e] + prod));
      }
    }
    uint4 o;
    __nv_bfloat16* ov = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int e = 0; e < 8; ++e) ov[e] = __float2bfloat16_rn(acc[e]);
    reinterpret_cast<uint4*>(out + t * H)[v] = o;
  }
}

int grid_for(int64_t items, int threads) {
  int64_t b = (items + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" int rw4_moe_permute(const int64_t* topk_idx, int64_t T, int32_t k, int32_t E,
                               int32_t* perm, int32_t* inv, int32_t* offsets, void* stream) {
  if (T < 0 || k < 1 || E < 1 || E > 4096)
    return fail(RW4_EINVAL, "rw4_moe_permute: bad T=%lld k=%d E=%d", (long long)T, k, E);
  if (T * k > (1ll << 30)) return fail(RW4_EINVAL, "rw4_moe_permute: T*k too large");
  if (!offsets || (T && (!topk_idx || !perm)))
    return fail(RW4_EINVAL, "rw4_moe_permute: null pointer");
  moe_permute_kernel<<<1, 1024, 2 * E * sizeof(int), rw4::as_stream(stream)>>>(
      topk_idx, (int)(T * k), E, perm, inv, offsets);
  return launch_status("rw4_moe_permute launch");
}

extern "C" int rw4_moe_gather(const void* x_bf16, const int32_t* perm, int64_t T, int32_t k,
                              int64_t H, void* x_perm_bf16, void* stream) {
  if (T < 0 || k < 1 || H <= 0 || H % 8)
    return fail(RW4_EINVAL, "rw4_moe_gather: bad T=%lld k=%d H=%lld (H %% 8 == 0)",
                (long long)T, k, (long long)H);
  if (T == 0) return RW4_OK;
  if (!x_bf16 || !perm || !x_perm_bf16) return fail(RW4_EINVAL, "rw4_moe_gather: null pointer");
  if (!aligned(x_bf16, 16) || !aligned(x_perm_bf16, 16))
    return fail(RW4_EINVAL, "rw4_moe_gather: buffers must be 16-byte aligned");
  const int64_t rows = T * k, vecs = H / 8;
  moe_gather_kernel<<<grid_for(rows * vecs, 256), 256, 0, rw4::as_stream(stream)>>>(
      static_cast<const uint4*>(x_bf16), perm, rows, k, vecs, static_cast<uint4*>(x_perm_bf16));
  return launch_status("rw4_moe_gather launch");
}

extern "C" int rw4_moe_grouped(const void* x_perm_bf16, const int32_t* offsets, int32_t E,
                               int64_t max_rows, const uint8_t* const* packed_e,
                               const void* const* scale_e, const void* const* zero_e, int64_t K,
                               int64_t N, int32_t group, int32_t act, void* y_perm_bf16,
                               void* stream) {
  if (E < 1 || max_rows < 0 || K <= 0 || N <= 0)
    return fail(RW4_EINVAL, "rw4_moe_grouped: bad E=%d max_rows=%lld K=%lld N=%lld", E,
                (long long)max_rows, (long long)K, (long long)N);
  if (group != 64 || K % 512)
    return fail(RW4_EINVAL, "rw4_moe_grouped: needs group 64 and K %% 512 == 0 (K=%lld)",
                (long long)K);
  if (act != 0 && act != 1) return fail(RW4_EINVAL, "rw4_moe_grouped: act %d", act);
  if (act == 1 && (N % 2 || (N / 2) % 8))
    return fail(RW4_EINVAL, "rw4_moe_grouped: SwiGLU needs N = 2*I with I %% 8 == 0");
  if (N > (1 << 30) || K > (1 << 30) || max_rows > (1 << 30))
    return fail(RW4_EINVAL, "rw4_moe_grouped: too large");
  if (max_rows == 0) return RW4_OK;
  if (!x_perm_bf16 || !offsets || !packed_e || !scale_e || !zero_e || !y_perm_bf16)
    return fail(RW4_EINVAL, "rw4_moe_grouped: null pointer");
  if (!aligned(x_perm_bf16, 16) || !aligned(y_perm_bf16, 16))
    return fail(RW4_EINVAL, "rw4_moe_grouped: activations must be 16-byte aligned");
  cudaStream_t s = rw4::as_stream(stream);
  const bool wide = max_rows > 8;
  if (act == 1) {
    if (wide)
      return launch_grouped<2, 4, 4, true>(x_perm_bf16, offsets, E, max_rows, packed_e, scale_e,
                                           zero_e, (int)K, (int)N, y_perm_bf16, s);
    return launch_grouped<1, 4, 4, true>(x_perm_bf16, offsets, E, max_rows, packed_e, scale_e,
                                         zero_e, (int)K, (int)N, y_perm_bf16, s);
  }
  if (wide)
    return launch_grouped<2, 4, 4, false>(x_perm_bf16, offsets, E, max_rows, packed_e, scale_e,
                                          zero_e, (int)K, (int)N, y_perm_bf16, s);
  return launch_grouped<1, 2, 6, false>(x_perm_bf16, offsets, E, max_rows, packed_e, scale_e,
                                        zero_e, (int)K, (int)N, y_perm_bf16, s);
}

extern "C" int rw4_moe_combine(const void* y_perm_bf16, const int32_t* inv,
                               const int64_t* topk_idx, const void* topk_w, int32_t w_dtype,
                               int64_t T, int32_t k, int64_t H, void* out_bf16, void* stream) {
  if (T < 0 || k < 1 || k > 8 || H <= 0 || H % 8)
    return fail(RW4_EINVAL, "rw4_moe_combine: bad T=%lld k=%d H=%lld (k <= 8, H %% 8 == 0)",
                (long long)T, k, (long long)H);
  if (T == 0) return RW4_OK;
  if (!y_perm_bf16 || !inv || !topk_w || !out_bf16)
    return fail(RW4_EINVAL, "rw4_moe_combine: null pointer");
  if (!aligned(y_perm_bf16, 16) || !aligned(out_bf16, 16))
    return fail(RW4_EINVAL, "rw4_moe_combine: buffers must be 16-byte aligned");
  cudaStream_t s = rw4::as_stream(stream);
  const int blocks = grid_for(T * (H / 8), 256);
  auto* y = static_cast<const __nv_bfloat16*>(y_perm_bf16);
  auto* o = static_cast<__nv_bfloat16*>(out_bf16);
  if (w_dtype == RW4_F32)
    moe_combine_kernel<float><<<blocks, 256, 0, s>>>(y, inv, topk_idx,
                                                     static_cast<const float*>(topk_w), T, k, H, o);
  else if (w_dtype == RW4_BF16)
    moe_combine_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        y, inv, topk_idx, static_cast<const __nv_bfloat16*>(topk_w), T, k, H, o);
  else
    return fail(RW4_EINVAL, "rw4_moe_combine: w_dtype %d", w_dtype);
  return launch_status("rw4_moe_combine launch");
}

extern "C" int rw4_slot_maps_create(const uint8_t* const* slot_packed, const void* const* slot_scale,
                                    const void* const* slot_zero, int32_t nslots, int64_t K,
                                    int64_t N, int32_t act, rw4_slot_maps** out) {
  if (!out) return fail(RW4_EINVAL, "rw4_slot_maps_create: null output");
  *out = nullptr;
  if (nslots < 1 || nslots > kMaxSlots)
    return fail(RW4_EINVAL, "rw4_slot_maps_create: %d slots (1..%d)", nslots, kMaxSlots);
  if (K <= 0 || K % 512 || N <= 0 || N > (1 << 30) || K > (1 << 30))
    return fail(RW4_EINVAL, "rw4_slot_maps_create: K=%lld N=%lld (K %% 512 == 0)", (long long)K,
                (long long)N);
  if (act != 0 && act != 1) return fail(RW4_EINVAL, "rw4_slot_maps_create: act %d", act);
  if (act == 1 && (N % 2 || (N / 2) % 8))
    return fail(RW4_EINVAL, "rw4_slot_maps_create: SwiGLU needs N = 2*I with I %% 8 == 0");
  if (!slot_packed || !slot_scale || !slot_zero)
    return fail(RW4_EINVAL, "rw4_slot_maps_create: null pointer array");
  auto* sm = new (std::nothrow) rw4_slot_maps();
  if (!sm) return fail(RW4_ENOMEM, "rw4_slot_maps_create: out of host memory");
  using L = gemv_tma::Layout<2, 6>;  // the only ring every grouped instantiation uses
  const int box_rows = act == 1 ? 16 : L::BR;
  const int G = (int)(K / 64);
  for (int s = 0; s < nslots; ++s) {
    if (!slot_packed[s] || !slot_scale[s] || !slot_zero[s]) {
      delete sm;
      return fail(RW4_EINVAL, "rw4_slot_maps_create: null pointer for slot %d", s);
    }
    int st = make_tensor_map_2d(&sm->maps.codes[s], slot_packed[s], CU_TENSOR_MAP_DATA_TYPE_UINT8,
                                1, N, K / 2, K / 2, box_rows, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st == RW4_OK)
      st = make_tensor_map_2d(&sm->maps.scale[s], slot_scale[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              2, N, G, (uint64_t)G * 2, box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st == RW4_OK)
      st = make_tensor_map_2d(&sm->maps.zero[s], slot_zero[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                              N, G, (uint64_t)G * 2, box_rows, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != RW4_OK) {
      delete sm;
      return st;
    }
  }
  sm->nslots = nslots;
  sm->K = (int)K;
  sm->N = (int)N;
  sm->act = act;
  *out = sm;
  return RW4_OK;
}

extern "C" int rw4_slot_maps_destroy(rw4_slot_maps* maps) {
  delete maps;
  return RW4_OK;
}

extern "C" int rw4_moe_grouped_slots(const void* x_perm_bf16, const int32_t* offsets, int32_t E,
                                     int64_t max_rows, const rw4_slot_maps* maps,
                                     const int32_t* slot_of, void* y_perm_bf16, void* stream) {
  if (!maps) return fail(RW4_EINVAL, "rw4_moe_grouped_slots: null slot maps");
  if (E < 1 || E > 65535 || max_rows < 0 || max_rows > (1 << 30))
    return fail(RW4_EINVAL, "rw4_moe_grouped_slots: bad E=%d max_rows=%lld", E,
                (long long)max_rows);
  if (max_rows == 0) return RW4_OK;
  if (!x_perm_bf16 || !offsets || !slot_of || !y_perm_bf16)
    return fail(RW4_EINVAL, "rw4_moe_grouped_slots: null pointer");
  if (!aligned(x_perm_bf16, 16) || !aligned(y_perm_bf16, 16))
    return fail(RW4_EINVAL, "rw4_moe_grouped_slots: activations must be 16-byte aligned");
  cudaStream_t s = rw4::as_stream(stream);
  const bool wide = max_rows > 8;
  const int a = maps->act;
  if (a == 1)
    return wide ? launch_grouped_slots<2, 2, 6, true>(maps, slot_of, x_perm_bf16, offsets, E,
                                                      max_rows, y_perm_bf16, s)
                : launch_grouped_slots<1, 2, 6, true>(maps, slot_of, x_perm_bf16, offsets, E,
                                                      max_rows, y_perm_bf16, s);
  return wide ? launch_grouped_slots<2, 2, 6, false>(maps, slot_of, x_perm_bf16, offsets, E,
                                                     max_rows, y_perm_bf16, s)
              : launch_grouped_slots<1, 2, 6, false>(maps, slot_of, x_perm_bf16, offsets, E,
                                                     max_rows, y_perm_bf16, s);
}

// Decode attention over a bf16 static KV cache: one query token per sequence, every query head,
// over the cache's first L positions, L read from device memory (the decode step's position + 1),
// so a CUDA graph replays it unchanged from step to step.  It stands for the model's attention of
// a decode step -- transformers' sdpa_attention_forward over a StaticCache with grouped-query heads
// and a causal mask ending at the position (models/llama/modeling_llama.py) -- in the decode step
// that rocketllm_b200.fused_decode runs, with programmatic dependent launch on both sides.
//
// Cache layout: k_cache / v_cache [B, KVH, T, D] bf16 (the StaticCache tensors), q [B, H, D],
// out [B, H, D]; G = H / KVH <= 8 query heads per kv head, D = 64 or 128.
//
// Work: a (batch, kv head) slot is one thread-block cluster of S <= 16 CTAs (S by batch: about two
// CTAs per SM); CTA c of the cluster takes the 64-token blocks c, c + S, ...; its four warps take 16
// tokens of each block.  Blocks arrive by 2-D TMA (128-byte swizzle: [64 tokens x 64 channels]
// boxes of K and of V) through a three-stage ring, every wait bounded.  Math on mma.sync
// m16n8k16 with the query heads as the n8 columns (no padding rows at GQA 4-8):
//   S^T[t, h] = sum_c K[t, c] q[h, c]              A = K rows (ldmatrix), B = q (registers)
//   O^T[c, h] += sum_t V[t, c] P[t, h]             A = V^T (ldmatrix.trans), B = P^T (movmatrix)
// with an online softmax per warp in the log2 domain (scores scaled in fp32; P rounded to bf16 for
// the second product, as flash attention does).  Warps combine in shared memory, CTAs through
// distributed shared memory, each CTA writing a share of bf16(O / l).
#include <cooperative_groups.h>

#include <atomic>

#include "rw4_common.cuh"
#include "rw4_tma.cuh"

namespace cg = cooperative_groups;

namespace {

using namespace rw4;

constexpr int kTok = 64;      // tokens per ring stage
constexpr int kWarps = 4;     // 16 tokens of a stage each
constexpr int kThreads = 32 * kWarps;
constexpr int kStages = 3;
constexpr int kHeads = 8;     // MMA columns: query heads of one kv head
constexpr int kMaxCluster = 16;   // CTAs per slot (a non-portable cluster size above 8)
constexpr float kNegBig = -1.0e30f;

template <int D>
struct DaLayout {
  static constexpr int kBox = kTok * 128;           // one [64 tokens x 64 channels] bf16 box
  static constexpr int kBlk = kBox * (D / 64);      // K (or V) of one stage
  static constexpr int kStage = 2 * kBlk;           // K boxes, then V boxes
  static constexpr int kRing = kStages * kStage;
  static constexpr int kBars = kRing;               // full[kStages], empty[kStages]
  static constexpr int kSmem = kBars + 2 * kStages * 8 + 1024;   // + alignment slack
  // partials after the loop (over the ring): per warp O[8][D], m[8], l[8]; then the CTA's
  static constexpr int kPart = kHeads * (D + 2);
  static_assert((kWarps + 1) * kPart * 4 <= kRing, "partials fit over the ring");
};

struct DaArgs {
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  const int64_t* pos;
  int64_t T;
  int KVH, G;
  float scale_log2;   // softmax scaling * log2(e)
  unsigned int* status;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory address of the 16-byte chunk holding channels [8 c8, 8 c8 + 8) of token row r
// (0..63) of a K or V block: box c8 / 8, chunk c8 % 8 swizzled with the row (128-byte swizzle).
__device__ __forceinline__ uint32_t chunk_addr(uint32_t blk, int r, int c8) {
  return blk + (c8 >> 3) * (kTok * 128) + r * 128 + (((c8 & 7) ^ (r & 7)) << 4);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 2)
    rw4_decode_attn_kernel(const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const DaArgs a) {
  using L = DaLayout<D>;
  constexpr int KC = D / 16;   // 16-channel steps of Q K^T, and 16-channel row tiles of O^T
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sb = smem_addr(smem);
  const uint32_t full0 = sb + L::kBars, empty0 = full0 + 8 * kStages;

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int csize = static_cast<int>(cluster.num_blocks());
  const int hs = blockIdx.y;                 // (batch, kv head) slot
  const int b = hs / a.KVH, kvh = hs % a.KVH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // q, the cache entries of this step and the position come from the kernels before this one
  asm volatile("griddepcontrol.wait;" ::: "memory");

  int64_t len = *a.pos + 1;   // the step's own token (written at pos) included
  if (len < 1) len = 1;
  if (len > a.T) len = a.T;
  const int nblk = static_cast<int>((len + kTok - 1) / kTok);
  const int mine = crank < nblk ? (nblk - 1 - crank) / csize + 1 : 0;   // blocks of this CTA
  const int row0 = hs * static_cast<int>(a.T);                           // the slot's first row

  auto issue = [&](int j) {   // thread 0: this CTA's j-th block into stage j % kStages
    const int s = j % kStages;
    const int blk = crank + j * csize;
    const uint32_t dst = sb + s * L::kStage;
    mbar_arrive_expect_tx(full0 + 8 * s, L::kStage);
#pragma unroll
    for (int bx = 0; bx < D / 64; ++bx) {
      tma_load_2d(dst + bx * L::kBox, &tm_k, 64 * bx, row0 + blk * kTok, full0 + 8 * s);
      tma_load_2d(dst + L::kBlk + bx * L::kBox, &tm_v, 64 * bx, row0 + blk * kTok,
                  full0 + 8 * s);
    }
  };
  int issued = 0;   // thread 0: blocks whose copies were started
  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    for (; issued < kStages && issued < mine; ++issued) issue(issued);
  }

  // q as B fragments: column n = head g of this kv head (zero beyond G), rows = channels
  uint32_t qb[KC][2];
  {
    const bool live = g < a.G;
    const __nv_bfloat16* qr =
        a.q + (static_cast<int64_t>(b) * a.KVH * a.G + kvh * a.G + (live ? g : 0)) * D;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      qb[kc][0] = live ? *reinterpret_cast<const uint32_t*>(qr + 16 * kc + 2 * t) : 0u;
      qb[kc][1] = live ? *reinterpret_cast<const uint32_t*>(qr + 16 * kc + 2 * t + 8) : 0u;
    }
  }

  float m_run[2] = {kNegBig, kNegBig}, l_run[2] = {0.f, 0.f};
  float o[KC][4];
#pragma unroll
  for (int vm = 0; vm < KC; ++vm)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[vm][i] = 0.f;

  bool ok = true;
  int consumed = 0;
  for (int j = 0; j < mine; ++j) {
    const int s = j % kStages;
    const bool got = mbar_wait(full0 + 8 * s, static_cast<uint32_t>((j / kStages) & 1), a.status);
    if (!__all_sync(0xffffffffu, got)) {
      ok = false;
      break;
    }
    const uint32_t kb = sb + s * L::kStage, vb = kb + L::kBlk;
    const int64_t tok0 = static_cast<int64_t>(crank + j * csize) * kTok + 16 * warp;

    // S^T for this warp's 16 tokens: rows = tokens, columns = heads
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int r = 16 * warp + (lane & 15);
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        uint32_t af[4];
        ldsm_x4(chunk_addr(kb, r, 2 * kc + (lane >> 4)), af);
        mma_bf16_16816(sc, af, qb[kc][0], qb[kc][1], sc);
      }
    }
    // scale, mask the positions at or past the length, online softmax per head column
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t tk = tok0 + g + 8 * (i >> 1);
      sc[i] = tk < len ? sc[i] * a.scale_log2 : -INFINITY;
    }
    float p[4];
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
      float mx = fmaxf(sc[jh], sc[jh + 2]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mnew = fmaxf(m_run[jh], mx);
      const float alpha = ex2(m_run[jh] - mnew);
      m_run[jh] = mnew;
      p[jh] = ex2(sc[jh] - mnew);
      p[jh + 2] = ex2(sc[jh + 2] - mnew);
      l_run[jh] = l_run[jh] * alpha + p[jh] + p[jh + 2];
#pragma unroll
      for (int vm = 0; vm < KC; ++vm) {
        o[vm][jh] *= alpha;
        o[vm][jh + 2] *= alpha;
      }
    }
    // P^T as the B fragment (tokens x heads)
    const uint32_t pb0 = movtrans(pack_bf16(p[0], p[1]));
    const uint32_t pb1 = movtrans(pack_bf16(p[2], p[3]));
    // O^T += V^T P^T: A = V^T tiles (16 channels x 16 tokens) by transposing loads
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int r = 16 * warp + ((mi >> 1) << 3) + rr;   // token row of this lane's matrix
#pragma unroll
      for (int vm = 0; vm < KC; ++vm) {
        uint32_t af[4];
        ldsm_x4_t(chunk_addr(vb, r, 2 * vm + (mi & 1)), af);
        mma_bf16_16816(o[vm], af, pb0, pb1, o[vm]);
      }
    }
    // every lane's reads of the stage are ordered before the refill (async proxy)
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
    ++consumed;
    if (threadIdx.x == 0 && issued < mine && issued == j + kStages) {
      // the stage is free once all four warps have read it
      if (mbar_wait(empty0 + 8 * s, static_cast<uint32_t>((j / kStages) & 1), a.status)) {
        issue(issued);
        ++issued;
      }
    }
  }
  if (threadIdx.x == 0) {
    // give the copies still in flight a bounded chance to land before the ring is reused
    for (int j = consumed; j < issued; ++j)
      mbar_wait(full0 + 8 * (j % kStages), static_cast<uint32_t>((j / kStages) & 1), a.status);
  }
  if (!ok && lane == 0) atomicOr(a.status, RW4_DEVERR_TIMEOUT);
  // only now may the next kernel (the o_proj GEMV) start launching: its CTAs, resident early,
  // would otherwise take the shared memory that this grid's CTAs need while the cache streams
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---- per-warp partials: O[h][c], m[h], l[h] (the ring area is free once every warp is here)
#pragma unroll
  for (int jh = 0; jh < 2; ++jh) {
    float l = l_run[jh];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    l_run[jh] = l;
  }
  __syncthreads();
  float* part = reinterpret_cast<float*>(smem);
  float* pw = part + warp * L::kPart;
#pragma unroll
  for (int vm = 0; vm < KC; ++vm)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int h = 2 * t + (i & 1), c = 16 * vm + g + 8 * (i >> 1);
      pw[h * D + c] = o[vm][i];
    }
  if (g == 0) {
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
      pw[kHeads * D + 2 * t + jh] = m_run[jh];
      pw[kHeads * D + kHeads + 2 * t + jh] = l_run[jh];
    }
  }
  __syncthreads();
  float* cp = part + kWarps * L::kPart;   // this CTA's combination of its warps
  for (int i = threadIdx.x; i < kHeads * D; i += kThreads) {
    const int h = i / D;
    float mx = kNegBig;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, part[w * L::kPart + kHeads * D + h]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = ex2(part[w * L::kPart + kHeads * D + h] - mx);
      acc = fmaf(part[w * L::kPart + i], f, acc);
      l = fmaf(part[w * L::kPart + kHeads * D + kHeads + h], f, l);
    }
    cp[i] = acc;
    if (i % D == 0) {
      cp[kHeads * D + h] = mx;
      cp[kHeads * D + kHeads + h] = l;
    }
  }
  cluster.sync();
  // every CTA of the cluster finishes a share of the outputs: each thread loads all ranks'
  // partials of its output at once (one round of distributed-shared-memory latency)
  for (int i = crank * kThreads + threadIdx.x; i < a.G * D; i += csize * kThreads) {
    const int h = i / D, c = i % D;
    float mr[kMaxCluster], lr[kMaxCluster], orr[kMaxCluster];
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      mr[r] = kNegBig;
      lr[r] = 0.f;
      orr[r] = 0.f;
      if (r < csize) {
        const float* rp = cluster.map_shared_rank(cp, r);
        mr[r] = rp[kHeads * D + h];
        lr[r] = rp[kHeads * D + kHeads + h];
        orr[r] = rp[h * D + c];
      }
    }
    float mx = kNegBig;
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) mx = fmaxf(mx, mr[r]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      const float f = ex2(mr[r] - mx);
      acc = fmaf(orr[r], f, acc);
      l = fmaf(lr[r], f, l);
    }
    a.out[(static_cast<int64_t>(b) * a.KVH * a.G + kvh * a.G + h) * D + c] =
        __float2bfloat16(l > 0.f ? acc / l : 0.f);
  }
  cluster.sync();   // every CTA has read the partials it needed
}

template <int D>
int launch_da(const DaArgs& args, const CUtensorMap& tk, const CUtensorMap& tv, int slots, int S,
              cudaStream_t stream) {
  using L = DaLayout<D>;
  auto kern = rw4_decode_attn_kernel<D>;
  static std::atomic<uint32_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set.load() & (1u << dev))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess)
      return fail(RW4_ECUDA, "decode_attention: cannot set the kernel's launch attributes");
    attr_set.fetch_or(1u << dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, slots);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = getenv("RW4_NO_PDL") ? 0 : 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tk, tv, args);
  if (err != cudaSuccess) return cuda_status(err, "rw4 decode_attention launch");
  return launch_status("rw4 decode_attention launch");
}

}  // namespace

extern "C" int rw4_decode_attention(const void* q, int32_t batch, int32_t heads, int32_t kv_heads,
                                    int32_t head_dim, const void* k_cache, const void* v_cache,
                                    int64_t cache_cap, const int64_t* pos, float scaling,
                                    void* out, void* stream) {
  using namespace rw4;
  if (!q || !out || !k_cache || !v_cache || !pos)
    return fail(RW4_EINVAL, "decode_attention: null pointer");
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || cache_cap <= 0)
    return fail(RW4_EINVAL, "decode_attention: bad shape (%d x %d heads, %d kv heads, cap %lld)",
                batch, heads, kv_heads, (long long)cache_cap);
  const int G = heads / kv_heads;
  if (G > kHeads)
    return fail(RW4_EUNSUPPORTED, "decode_attention: %d query heads per kv head (at most 8)", G);
  if (head_dim != 64 && head_dim != 128)
    return fail(RW4_EUNSUPPORTED, "decode_attention: head_dim %d (64 or 128)", head_dim);
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(RW4_EINVAL, "decode_attention: q and the caches must be 16-byte aligned");
  const int64_t slots = static_cast<int64_t>(batch) * kv_heads;
  if (slots > 65535 || slots * cache_cap > (int64_t(1) << 31) - kTok)
    return fail(RW4_EINVAL, "decode_attention: cache of %lld rows too large",
                (long long)(slots * cache_cap));
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "decode_attention: device status word unavailable");
  CUtensorMap tk, tv;
  const uint64_t rows = static_cast<uint64_t>(slots * cache_cap);
  int st = make_tensor_map_2d(&tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows,
                              (uint64_t)head_dim, (uint64_t)head_dim * 2, kTok, 64,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows,
                            (uint64_t)head_dim, (uint64_t)head_dim * 2, kTok, 64,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != RW4_OK) return st;
  // CTAs per slot: about two per SM over the whole grid, a cluster of at most 16 (RW4_DA_CLUSTER
  // caps it lower, for measurements), and no more than the cache's 64-token blocks
  static const int cap_env = [] {
    const char* e = getenv("RW4_DA_CLUSTER");
    return e ? atoi(e) : 0;
  }();
  const int smax = (cap_env == 1 || cap_env == 2 || cap_env == 4 || cap_env == 8) ? cap_env
                                                                                 : kMaxCluster;
  const int64_t blocks = (cache_cap + kTok - 1) / kTok;
  int S = 1;
  while (S < smax && slots * (2 * S) <= 2 * static_cast<int64_t>(sm_count()) && 2 * S <= blocks)
    S *= 2;
  DaArgs args;
  args.q = static_cast<const __nv_bfloat16*>(q);
  args.out = static_cast<__nv_bfloat16*>(out);
  args.pos = pos;
  args.T = cache_cap;
  args.KVH = kv_heads;
  args.G = G;
  args.scale_log2 = scaling * 1.4426950408889634f;
  args.status = status;
  cudaStream_t s = as_stream(stream);
  return head_dim == 128 ? launch_da<128>(args, tk, tv, (int)slots, S, s)
                         : launch_da<64>(args, tk, tv, (int)slots, S, s);
}

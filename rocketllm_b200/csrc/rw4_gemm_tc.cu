// RW4 tensor-core GEMM for prefill and batched decode: y[M, N] = x[M, K] . W[N, K]^T, with W in
// RW4 and x, y bf16.  sm_100a: TMA -> shared memory -> tcgen05.mma (accumulator in TMEM) ->
// tcgen05.ld epilogue.
//
// Tile: 128 weight rows (UMMA M) x BN = 256 tokens (UMMA N) per CTA, K in blocks of 64 (= one RW4
// group = one 128-byte swizzle atom of bf16).  Roles (6 warps):
//   warp 0  TMA producer: per k-block, the raw codes [128 rows x 32 B] and the activation tile
//           [256 rows x 64 bf16] (128-byte swizzle) into stage s;
//   warp 1  allocates 256 TMEM columns, then one lane issues 4 tcgen05.mma (K = 16 each) per
//           k-block and tcgen05.commit's the stage back to the producer; a final commit signals the
//           epilogue;
//   warps 2-5  dequantize: thread r expands row r's 64 codes of the k-block to the exact bf16
//           weight the reference materialises, bf16(fp32(code) * scale + zero)
//           (rocketllm/quant/kv_cache.py:249-257), and writes them into the A tile in the canonical
//           K-major 128-byte-swizzled layout (16-byte chunk c of row r at c ^ (r % 8)); then, after
//           the last k-block, they read the accumulator out of TMEM (warp w reads lanes
//           32 (w % 4) .. +31) and store bf16 y.
// The product therefore equals a bf16 GEMM over the reference's dequantized weight, up to fp32
// accumulation order.
//
// Shared memory per stage: codes 4 KB + activations 32 KB + A tile 16 KB; 4 stages.  No TMA load
// uses multicast.  Every mbarrier wait is bounded (rw4_tma.cuh); on a timeout the CTA stops
// issuing, waits (bounded) for the MMAs it issued, frees its TMEM and writes nothing.
#include <atomic>

#include "rw4_tma.cuh"

namespace {

using namespace rw4;

constexpr int BM = 128;          // weight rows per CTA (UMMA M)
constexpr int BN = 256;          // tokens per CTA (UMMA N)
constexpr int BK = 64;           // K per stage (one group, one 128-byte bf16 swizzle atom)
constexpr int S = 4;             // pipeline stages
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;

constexpr int kCodeBytes = BM * (BK / 2);      // 4096
constexpr int kXBytes = BN * BK * 2;           // 32768
constexpr int kABytes = BM * BK * 2;           // 16384
// Layout (offsets from a 1024-byte aligned base): X stages, A stages, code stages, barriers.
constexpr int kOffX = 0;
constexpr int kOffA = kOffX + S * kXBytes;
constexpr int kOffCodes = kOffA + S * kABytes;
constexpr int kOffBars = kOffCodes + S * kCodeBytes;
constexpr int kNumBars = 3 * S + 1;            // full[S], aready[S], empty[S], accum
constexpr int kOffTmemSlot = kOffBars + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16;
constexpr int kDynSmem = kSmemBytes + 1024;
static_assert(kDynSmem <= 227 * 1024, "shared memory budget");
static_assert(kOffA % 1024 == 0 && kXBytes % 1024 == 0 && kABytes % 1024 == 0, "swizzle atoms");

// UMMA instruction descriptor, kind::f16: D f32, A bf16, B bf16, both K-major, M = 128, N = BN.
constexpr uint32_t kIdesc = (1u << 4)                    // D format: f32
                            | (1u << 7)                  // A format: bf16
                            | (1u << 10)                 // B format: bf16
                            | ((uint32_t)(BN >> 3) << 17)  // N / 8
                            | ((uint32_t)(BM >> 4) << 24); // M / 16

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                       // leading byte offset (unused for K-major SW128)
  d |= (uint64_t)(1024 >> 4) << 32;             // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                       // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 columns of 32-bit accumulator -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Exact fp32 of a 4-bit code: 2^23 + c as a float bit pattern, minus 2^23.
__device__ __forceinline__ float code_f32(uint32_t c) {
  return __uint_as_float(0x4B000000u | c) - 8388608.0f;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    rw4_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_codes,
                       const __grid_constant__ CUtensorMap tm_x,
                       const __half* __restrict__ scale, const __half* __restrict__ zero, int M,
                       int K, int N, __nv_bfloat16* __restrict__ y, unsigned int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  const uint32_t sb = smem_addr(smem);
  const uint32_t full0 = sb + kOffBars;            // TMA landed (codes + x)
  const uint32_t aready0 = full0 + 8 * S;          // A tile written by the dequant warps
  const uint32_t empty0 = aready0 + 8 * S;         // MMAs of the stage finished
  const uint32_t accum = empty0 + 8 * S;           // all MMAs finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BN;   // token tile (fastest: CTAs sharing a weight tile run together)
  const int n0 = blockIdx.y * BM;   // weight-row tile
  const int nkb = K / BK;
  const int G = K / 64;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(aready0 + 8 * s, 4);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_codes);
      prefetch_tensormap(&tm_x);
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(empty0 + 8 * s, ((kb / S) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        mbar_arrive_expect_tx(full0 + 8 * s, kCodeBytes + kXBytes);
        tma_load_2d(sb + kOffCodes + s * kCodeBytes, &tm_codes, kb * (BK / 2), n0, full0 + 8 * s);
        tma_load_2d(sb + kOffX + s * kXBytes, &tm_x, kb * BK, m0, full0 + 8 * s);
        issued = kb + 1;
      }
      // Drain: never leave the CTA with copies still landing in its shared memory.
      for (int kb = max(0, issued - S); kb < issued; ++kb)
        mbar_wait(full0 + 8 * (kb % S), (kb / S) & 1, status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t par = (kb / S) & 1;
        if (!mbar_wait(full0 + 8 * s, par, status) || !mbar_wait(aready0 + 8 * s, par, status)) {
          aborted = 1;
          break;
        }
        tc_fence_after();
        const uint64_t da = smem_desc(sb + kOffA + s * kABytes);
        const uint64_t db = smem_desc(sb + kOffX + s * kXBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // +32 bytes per 16 bf16 along K inside the swizzle atom (descriptor address >> 4).
          umma_bf16(tmem, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk),
                    (kb > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(empty0 + 8 * s);
      }
      umma_commit(accum);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------- dequant warps, then epilogue ----------------
    const int r = threadIdx.x - 64;           // 0..127: A-tile row
    const int n = min(n0 + r, N - 1);         // clamped for the scale loads; row >= N never stored
    const __half* srow = scale + (int64_t)n * G;
    const __half* zrow = zero + (int64_t)n * G;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      const float sc = __half2float(srow[kb]);
      const float zr = __half2float(zrow[kb]);
      if (!mbar_wait(full0 + 8 * s, (kb / S) & 1, status)) {
        aborted = 1;
        break;
      }
      const uint4* src = reinterpret_cast<const uint4*>(smem + kOffCodes + s * kCodeBytes + r * 32);
      const uint4 c0 = src[0], c1 = src[1];
      const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      uint8_t* arow = smem + kOffA + s * kABytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = k 8c .. 8c+7 = word c (8 nibbles)
        const uint32_t w = words[c];
        uint4 out;
        out.x = pack_bf16x2(fmaf(code_f32(w & 0xF), sc, zr), fmaf(code_f32((w >> 4) & 0xF), sc, zr));
        out.y = pack_bf16x2(fmaf(code_f32((w >> 8) & 0xF), sc, zr),
                            fmaf(code_f32((w >> 12) & 0xF), sc, zr));
        out.z = pack_bf16x2(fmaf(code_f32((w >> 16) & 0xF), sc, zr),
                            fmaf(code_f32((w >> 20) & 0xF), sc, zr));
        out.w = pack_bf16x2(fmaf(code_f32((w >> 24) & 0xF), sc, zr),
                            fmaf(code_f32(w >> 28), sc, zr));
        *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = out;
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(aready0 + 8 * s);
    }
    // epilogue: wait for every MMA, then TMEM -> registers -> bf16 y
    if (!aborted && mbar_wait(accum, 0, status)) {
      tc_fence_after();
      const int q = warp & 3;                 // TMEM lane quarter this warp may access
      const int row = 32 * q + lane;          // accumulator row = weight row n0 + row
      const int nrow = n0 + row;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
        if (nrow < N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            if (m < M) y[(int64_t)m * N + nrow] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
        }
      }
    } else {
      aborted = 1;
    }
  }

  // ---- teardown: every MMA this CTA issued has completed before TMEM is released -------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (aborted) {
      // the accumulator commit may still be pending on an error path: bounded wait, then free
      if (lane == 0) mbar_wait(accum, 0, status);
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

namespace rw4 {

bool gemm_tc_supported(int64_t M, int64_t K, int64_t N) {
  static const bool off = getenv("RW4_GEMM_TC_OFF") != nullptr;
  return !off && M > 16 && K % 64 == 0 && K >= 64 && N >= 1;
}

int gemm_tc_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                   const void* zr, int64_t N, void* y, cudaStream_t stream) {
  CUtensorMap tc, tx;
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, BM,
                              BK / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, (uint64_t)K * 2,
                            BN, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != RW4_OK) return st;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(rw4_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kDynSmem) != cudaSuccess)
      return fail(RW4_ECUDA, "gemm_tc: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemm_tc: device status word unavailable");
  dim3 grid((unsigned)((M + BN - 1) / BN), (unsigned)((N + BM - 1) / BM));
  rw4_gemm_tc_kernel<<<grid, kThreads, kDynSmem, stream>>>(
      tc, tx, static_cast<const __half*>(sc), static_cast<const __half*>(zr), (int)M, (int)K,
      (int)N, static_cast<__nv_bfloat16*>(y), status);
  return launch_status("rw4 gemm_tc launch");
}

}  // namespace rw4

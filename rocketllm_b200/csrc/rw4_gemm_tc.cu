// RW4 tensor-core GEMM for prefill and batched decode: y[M, N] = x[M, K] . W[N, K]^T, with W in
// RW4 and x, y bf16.  sm_100a: TMA -> shared memory -> tcgen05.mma (accumulator in TMEM) ->
// tcgen05.ld epilogue.
//
// Tile: 128 weight rows (UMMA M) x BN tokens (UMMA N; 64, 128 or 256 by batch size) per CTA, K in
// blocks of 64 (= one RW4 group = one 128-byte swizzle atom of bf16).  Roles (11 warps):
//   warp 0     codes producer: TMA of the raw codes [128 rows x 32 B] of each k-block into a deep
//              ring (12-16 stages, L2 evict-first), so that enough HBM reads are in flight per SM;
//   warp 10    activation producer: TMA of the activation tile [BN rows x 64 bf16] (128-byte
//              swizzle) into a shallow ring shared with the dequantized A tiles;
//   warp 1     allocates BN TMEM columns, then one lane issues 4 tcgen05.mma (K = 16 each) per
//              k-block and tcgen05.commit's the stage back to the producer; a final commit
//              signals the epilogue;
//   warps 2-9  dequantize: two threads per weight row (adjacent lanes, 16 code bytes each) expand
//              the k-block to the exact bf16 weight the reference materialises,
//              bf16(fp32(code) * scale + zero) (rocketllm/quant/kv_cache.py:249-257), and write it
//              into the A tile in the canonical K-major 128-byte-swizzled layout (16-byte chunk c of
//              row r at c ^ (r % 8)); scales and zeros are prefetched 8 groups at a time.  After the
//              last k-block the same warps read the accumulator out of TMEM (warp w reads lanes
//              32 (w % 4) .. +31, the two warps of a quarter split the columns) and store bf16 y.
// The product equals a bf16 GEMM over the reference's dequantized weight up to fp32 accumulation
// order.  CTAs sharing a weight tile are adjacent in the grid (tokens fastest), so a weight tile
// is read from HBM about once; the activations are loaded evict-last and stay in L2 across the
// waves of weight tiles.
//
// Every TMA load is a plain per-CTA load.  Every mbarrier wait is bounded (rw4_tma.cuh); on a timeout the CTA
// stops issuing, waits (bounded) for its own copies and MMAs, frees its TMEM and writes nothing.
#include <atomic>

#include "rw4_tcgen05.cuh"

namespace {

using namespace rw4;

constexpr int BM = 128;          // weight rows per CTA (UMMA M)
constexpr int BK = 64;           // K per stage (one group, one 128-byte bf16 swizzle atom)
constexpr int kDequantWarps = 8;
constexpr int kThreads = 32 * (3 + kDequantWarps);  // codes, MMA, dequant x8, activations
// A codes stage covers 4 k-blocks: 128 rows x 128 bytes (256 k), one 128-byte-swizzled TMA box.
// (Measured with device timestamps: a 128 x 32-byte box -- one k-block -- took ~2.7 us from
// issue to landing, and with one box per k-block the ring, not the tensor core or the dequant,
// set the pace: ~0.55 us per k-block.)
constexpr int kKbPerCodeStage = 4;
constexpr int kCodeBytes = BM * (BK / 2) * kKbPerCodeStage;  // 16384
constexpr int kABytes = BM * BK * 2;           // 16384

template <int BN>
struct Cfg {
  // Two rings.  An x / A stage is freed only when the MMAs that read it complete, and refilling it
  // takes an L2 -> shared-memory TMA plus the dequant, a round trip of roughly 2 us; that ring is
  // therefore as deep as shared memory allows (4 / 6 / 8 stages for BN = 256 / 128 / 64).  The raw
  // codes (4 KB a k-block) are released as soon as the dequant warps have them in registers, so a
  // shorter ring keeps enough HBM reads in flight.
  static constexpr int S1 = BN == 256 ? 2 : 3;                  // codes stages (4 k-blocks each)
  static constexpr int S2 = BN == 256 ? 4 : BN == 128 ? 5 : 7;  // x / A stages
  static constexpr int kXBytes = BN * BK * 2;
  static constexpr int kOffX = 0;
  static constexpr int kOffA = kOffX + S2 * kXBytes;
  static constexpr int kOffCodes = kOffA + S2 * kABytes;
  static constexpr int kOffBars = kOffCodes + S1 * kCodeBytes;
  // codes_full[S1], codes_empty[S1], x_full[S2], a_ready[S2], stage_empty[S2], accum
  static constexpr int kNumBars = 2 * S1 + 3 * S2 + 1;
  static constexpr int kOffTmemSlot = kOffBars + kNumBars * 8;  // + 8: the dequant scratch word
  static constexpr int kDynSmem = kOffTmemSlot + 16 + 1024;
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  // UMMA instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M = 128, N = BN.
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                     ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  static_assert(kDynSmem <= 227 * 1024, "shared memory budget");
  static_assert(kOffA % 1024 == 0 && kXBytes % 1024 == 0 && kOffCodes % 1024 == 0,
                "swizzle atoms stay 1024-aligned");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Exact fp32 code without moving the nibble: nibble i of a half-word, masked in place under the
// 2^23 bit pattern, is the float 2^23 + c * 2^(4i) (the code sits in mantissa bits 4i..4i+3);
// minus 2^23 that is c * 2^(4i) exactly, and the caller multiplies by s * 2^(-4i) (exact: a power
// of two times an fp16 value), so fma gives RN(c * s + z) -- the reference's value -- with one LOP3
// and one FADD per code and no per-nibble shift.
__device__ __forceinline__ float code_at(uint32_t half_word, uint32_t mask) {
  return __uint_as_float((half_word & mask) | 0x4B000000u) - 8388608.0f;
}

// 8 codes of one 32-bit word -> 8 exact bf16 weights (one 16-byte A-tile chunk).
// s4[i] = scale * 2^(-4i); the upper half-word is moved down once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, const float (&s4)[4], float zr) {
  const uint32_t lo = w, hi = w >> 16;  // the masks below only select bits 0..15
  uint4 o;
  o.x = pack_bf16x2(fmaf(code_at(lo, 0x000Fu), s4[0], zr), fmaf(code_at(lo, 0x00F0u), s4[1], zr));
  o.y = pack_bf16x2(fmaf(code_at(lo, 0x0F00u), s4[2], zr), fmaf(code_at(lo, 0xF000u), s4[3], zr));
  o.z = pack_bf16x2(fmaf(code_at(hi, 0x000Fu), s4[0], zr), fmaf(code_at(hi, 0x00F0u), s4[1], zr));
  o.w = pack_bf16x2(fmaf(code_at(hi, 0x0F00u), s4[2], zr), fmaf(code_at(hi, 0xF000u), s4[3], zr));
  return o;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    rw4_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_codes,
                       const __grid_constant__ CUtensorMap tm_x,
                       const __half* __restrict__ scale, const __half* __restrict__ zero, int M,
                       int K, int N, __nv_bfloat16* __restrict__ y, unsigned int* status) {
  using C = Cfg<BN>;
  constexpr int S1 = C::S1, S2 = C::S2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  const uint32_t sb = smem_addr(smem);
  const uint32_t cfull0 = sb + C::kOffBars;        // codes landed
  const uint32_t cempty0 = cfull0 + 8 * S1;        // codes read by all dequant warps
  const uint32_t xfull0 = cempty0 + 8 * S1;        // activation tile landed
  const uint32_t aready0 = xfull0 + 8 * S2;        // A tile written by the dequant warps
  const uint32_t sempty0 = aready0 + 8 * S2;       // MMAs of the x / A stage finished
  const uint32_t accum = sempty0 + 8 * S2;         // all MMAs finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BN;   // token tile (fastest: CTAs sharing a weight tile run together)
  const int n0 = blockIdx.y * BM;   // weight-row tile
  const int nkb = K / BK;
  const int G = K / 64;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < S1; ++s) {
      mbar_init(cfull0 + 8 * s, 1);
      mbar_init(cempty0 + 8 * s, kDequantWarps);
    }
    for (int s = 0; s < S2; ++s) {
      mbar_init(xfull0 + 8 * s, 1);  // unused: the activation tile completes on a_ready
      // a_ready: the 8 dequant warps' arrivals plus the activation producer's arrive.expect_tx,
      // completed by its TMA bytes -- the MMA thread waits on this one barrier per k-block
      mbar_init(aready0 + 8 * s, kDequantWarps + 1);
      mbar_init(sempty0 + 8 * s, 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- codes producer (deep ring) ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_codes);
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      const int ncs = (nkb + kKbPerCodeStage - 1) / kKbPerCodeStage;
      for (int cs = 0; cs < ncs; ++cs) {
        const int s = cs % S1;
        if (!mbar_wait(cempty0 + 8 * s, ((cs / S1) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        mbar_arrive_expect_tx(cfull0 + 8 * s, kCodeBytes);
        tma_load_2d_hint(sb + C::kOffCodes + s * kCodeBytes, &tm_codes,
                         cs * (BK / 2) * kKbPerCodeStage, n0, cfull0 + 8 * s, pol);
        issued = cs + 1;
      }
      for (int cs = max(0, issued - S1); cs < issued; ++cs)  // drain own copies
        mbar_wait(cfull0 + 8 * (cs % S1), (cs / S1) & 1, status);
    }
  } else if (warp == kThreads / 32 - 1) {
    // ---------------- activation producer (shallow ring) ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      // every weight-row tile streams against the same activations: keep them in L2 (evict-last)
      // so that each wave of weight tiles finds them there
      const uint64_t pol = policy_evict_last();
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S2;
        if (!mbar_wait(sempty0 + 8 * s, ((kb / S2) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        mbar_arrive_expect_tx(aready0 + 8 * s, C::kXBytes);
        tma_load_2d_hint(sb + C::kOffX + s * C::kXBytes, &tm_x, kb * BK, m0, aready0 + 8 * s,
                         pol);
        issued = kb + 1;
      }
      for (int kb = max(0, issued - S2); kb < issued; ++kb)  // drain own copies
        mbar_wait(aready0 + 8 * (kb % S2), (kb / S2) & 1, status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S2;
        const uint32_t par = (kb / S2) & 1;
        if (!mbar_wait(aready0 + 8 * s, par, status)) {
          aborted = 1;
          break;
        }
        tc_fence_after();
        const uint64_t da = smem_desc(sb + C::kOffA + s * kABytes);
        const uint64_t db = smem_desc(sb + C::kOffX + s * C::kXBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // +32 bytes per 16 bf16 along K inside the swizzle atom (descriptor address >> 4).
          umma_f16(tmem, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), C::kIdesc,
                    (kb > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(sempty0 + 8 * s);
      }
      umma_commit(accum);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------- dequant warps (2 .. 2+kDequantWarps-1), then epilogue ----------------
    const int d = threadIdx.x - 64;           // 0..255
    const int r = d >> 1;                     // A-tile row
    const int h = d & 1;                      // which 16 code bytes (32 k) of the row
    const int n = min(n0 + r, N - 1);         // clamped for the scale loads; rows >= N not stored
    const __half* srow = scale + (int64_t)n * G;
    const __half* zrow = zero + (int64_t)n * G;
    const bool vec8 = (G & 7) == 0;
    // scales / zeros of 8 consecutive groups, loaded one block ahead
    uint4 sc_cur = make_uint4(0, 0, 0, 0), zr_cur = sc_cur, sc_nxt = sc_cur, zr_nxt = sc_cur;
    auto load8 = [&](int g0, uint4& sv, uint4& zv) {
      if (g0 >= G) return;
      if (vec8) {
        sv = __ldg(reinterpret_cast<const uint4*>(srow + g0));
        zv = __ldg(reinterpret_cast<const uint4*>(zrow + g0));
      } else {
        unsigned short sa[8], za[8];
        for (int i = 0; i < 8; ++i) {
          const int gi = min(g0 + i, G - 1);
          sa[i] = __half_as_ushort(srow[gi]);
          za[i] = __half_as_ushort(zrow[gi]);
        }
        sv = make_uint4(sa[0] | (sa[1] << 16), sa[2] | (sa[3] << 16), sa[4] | (sa[5] << 16),
                        sa[6] | (sa[7] << 16));
        zv = make_uint4(za[0] | (za[1] << 16), za[2] | (za[3] << 16), za[4] | (za[5] << 16),
                        za[6] | (za[7] << 16));
      }
    };
    load8(0, sc_cur, zr_cur);
    load8(8, sc_nxt, zr_nxt);
    const int ncs = (nkb + kKbPerCodeStage - 1) / kKbPerCodeStage;
    for (int cs = 0; cs < ncs && !aborted; ++cs) {
      // this thread's 16 code bytes of each of the stage's k-blocks, then release the stage
      const int s1 = cs % S1;
      if (!mbar_wait(cfull0 + 8 * s1, (cs / S1) & 1, status)) {
        aborted = 1;
        break;
      }
      uint4 cw[kKbPerCodeStage];
      const uint8_t* crow = smem + C::kOffCodes + s1 * kCodeBytes + r * 128;
#pragma unroll
      for (int j = 0; j < kKbPerCodeStage; ++j)   // 128-byte swizzle: chunk c at c ^ (r % 8)
        cw[j] = *reinterpret_cast<const uint4*>(crow + (((2 * j + h) ^ (r & 7)) << 4));
      // The TMA refill of this slot (async proxy) must not overtake these shared-memory reads
      // (released right after them, outputs varied from run to run at some shapes): every thread
      // stores a value computed from all 16 words it read into a scratch word, which it cannot
      // issue before those reads have returned, and only then is the slot released.  (A
      // fence.proxy.async here does the same but also waits for the scale prefetch in flight.)
      {
        const uint32_t v = cw[0].x ^ cw[0].y ^ cw[0].z ^ cw[0].w ^ cw[1].x ^ cw[1].y ^ cw[1].z ^
                           cw[1].w ^ cw[2].x ^ cw[2].y ^ cw[2].z ^ cw[2].w ^ cw[3].x ^ cw[3].y ^
                           cw[3].z ^ cw[3].w;
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(sb + C::kOffTmemSlot + 8), "r"(v) : "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(cempty0 + 8 * s1);  // codes slot may be refilled
#pragma unroll
      for (int j = 0; j < kKbPerCodeStage; ++j) {
        const int kb = cs * kKbPerCodeStage + j;
        if (kb >= nkb) break;
        const int s2 = kb % S2;
        const int gi = kb & 7;
        if (gi == 0 && kb > 0) {
          sc_cur = sc_nxt;
          zr_cur = zr_nxt;
          load8(kb + 8, sc_nxt, zr_nxt);
        }
        const uint32_t sw = (gi < 4) ? ((gi < 2) ? sc_cur.x : sc_cur.y)
                                     : ((gi < 6) ? sc_cur.z : sc_cur.w);
        const uint32_t zw = (gi < 4) ? ((gi < 2) ? zr_cur.x : zr_cur.y)
                                     : ((gi < 6) ? zr_cur.z : zr_cur.w);
        const float sc = __half2float(__ushort_as_half((unsigned short)(sw >> (16 * (gi & 1)))));
        const float zr = __half2float(__ushort_as_half((unsigned short)(zw >> (16 * (gi & 1)))));
        const float s4[4] = {sc, sc * 0.0625f, sc * 0.00390625f, sc * 0.000244140625f};
        // the A slot is free once the MMAs of k-block kb - S2 have finished
        if (!mbar_wait(sempty0 + 8 * s2, ((kb / S2) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        uint8_t* arow = smem + C::kOffA + s2 * kABytes + r * 128;
        const uint32_t words[4] = {cw[j].x, cw[j].y, cw[j].z, cw[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // chunk 4h + c = k 8(4h+c) .. +7
          const int chunk = 4 * h + c;
          *reinterpret_cast<uint4*>(arow + ((chunk ^ (r & 7)) << 4)) = dequant8(words[c], s4, zr);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(aready0 + 8 * s2);
      }
    }
    // epilogue: wait for every MMA, then TMEM -> registers -> bf16 y
    if (!aborted && mbar_wait(accum, 0, status)) {
      tc_fence_after();
      const int q = warp & 3;                 // TMEM lane quarter this warp may access
      const int colhalf = (warp - 2) >> 2;    // the two warps of a quarter split the columns
      const int row = 32 * q + lane;          // accumulator row = weight row n0 + row
      const int nrow = n0 + row;
      constexpr int kCols = BN / 2;
#pragma unroll 1
      for (int c0 = colhalf * kCols; c0 < (colhalf + 1) * kCols; c0 += 32) {
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
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int BN>
int launch_bn(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
              const void* zr, int64_t N, void* y, cudaStream_t stream) {
  using C = Cfg<BN>;
  CUtensorMap tc, tx;
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, BM,
                              BK / 2 * kKbPerCodeStage, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, (uint64_t)K * 2,
                            BN, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != RW4_OK) return st;
  auto kern = rw4_gemm_tc_kernel<BN>;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmem) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "gemm_tc: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemm_tc: device status word unavailable");
  dim3 grid((unsigned)((M + BN - 1) / BN), (unsigned)((N + BM - 1) / BM));
  kern<<<grid, kThreads, C::kDynSmem, stream>>>(tc, tx, static_cast<const __half*>(sc),
                                                static_cast<const __half*>(zr), (int)M, (int)K,
                                                (int)N, static_cast<__nv_bfloat16*>(y), status);
  return launch_status("rw4 gemm_tc launch");
}

}  // namespace

namespace rw4 {

bool gemm_tc_supported(int64_t M, int64_t K, int64_t N) {
  static const bool off = getenv("RW4_GEMM_TC_OFF") != nullptr;
  return !off && M > 16 && K % 64 == 0 && K >= 64 && N >= 1;
}

int gemm_tc_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                   const void* zr, int64_t N, void* y, cudaStream_t stream) {
  static const int forced = [] {
    const char* e = getenv("RW4_GEMM_BN");
    return e ? atoi(e) : 0;
  }();
  const int bn = forced ? forced : (M <= 64 ? 64 : M <= 128 ? 128 : 256);
  if (bn == 64) return launch_bn<64>(x, M, K, wq, sc, zr, N, y, stream);
  if (bn == 128) return launch_bn<128>(x, M, K, wq, sc, zr, N, y, stream);
  return launch_bn<256>(x, M, K, wq, sc, zr, N, y, stream);
}

}  // namespace rw4

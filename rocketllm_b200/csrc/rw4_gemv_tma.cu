// RW4 dequant-GEMV, TMA-fed (K a multiple of 512): y[M, N] = x[M, K] . W[N, K]^T, M <= 16 per
// 16-row batch slice.
//
// Same arithmetic as rw4_gemv.cu (codes multiplied as bf16 (128 + c) on the tensor cores, per-group
// fp32 scale / zero epilogue, x sums from an all-ones MMA), but the codes and scales reach the SM
// through a multi-stage shared-memory pipeline instead of registers, so the bytes a CTA keeps in
// flight are bounded by shared memory (tens of KB per SM), not by the register file:
//
//   producer warp (one elected lane)      S-stage ring in shared memory          8 consumer warps
//   wait empty[s] ---------------------> codes  [2 boxes x 16R rows x 128 B]  --> wait full[s]
//   expect_tx(full[s]); 4 TMA loads      scales [16R rows x 8 fp16]              copy 2x8 B codes +
//   (cp.async.bulk.tensor.2d, L2        zeros  [16R rows x 8 fp16]              scales to registers
//    evict-first hint)                                                            arrive empty[s]
//                                                                                 MMA + epilogue
//
// A stage is 512 values of K (8 groups) of the CTA's 16R rows; consumer warp w always takes group w
// of the stage, accumulates over all stages, and the 8 partial sums are combined in shared memory
// at the end (deterministic, no atomics, no scratch memory).  The code boxes use the 128-byte TMA
// swizzle (16-byte chunk index XOR row % 8), which keeps the consumers' 8-byte shared loads free of
// bank conflicts beyond the two wavefronts 256 bytes need anyway.  Rows past N are zero-filled by
// the TMA unit and never stored.
//
// Every mbarrier wait is bounded (rw4_tma.cuh); on a timeout the CTA drains its own copies, writes
// nothing and sets the library's device status word.
#include <atomic>

#include "rw4_gemv_frag.cuh"
#include "rw4_tma.cuh"

namespace {

using namespace rw4;
using namespace rw4::frag;

constexpr int kConsumers = 8;                 // consumer warps = groups per stage
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kStageK = 64 * kConsumers;      // 512 values of K per stage

template <int R, int S>
struct Layout {
  static constexpr int BR = 16 * R;                   // rows per CTA
  static constexpr int kCodeBox = BR * 128;           // one box: BR rows x 128 bytes (256 k)
  static constexpr int kCodeStage = 2 * kCodeBox;
  static constexpr int kScaleStage = BR * 16;         // BR rows x 8 fp16
  static constexpr int kCodes = 0;
  static constexpr int kScales = S * kCodeStage;
  static constexpr int kZeros = kScales + S * kScaleStage;
  static constexpr int kBars = kZeros + S * kScaleStage;
  static constexpr int kBytes = kBars + 2 * S * 8;
  static constexpr int kStageTx = kCodeStage + 2 * kScaleStage;
  static constexpr int kDynSmem = kBytes + 1024;      // slack to align the ring to 1024 bytes
};

template <int NT, int R, int S>
__global__ void __launch_bounds__(kThreads)
    rw4_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_scale,
                        const __grid_constant__ CUtensorMap tm_zero,
                        const __nv_bfloat16* __restrict__ x, int M, int K, int N,
                        __nv_bfloat16* __restrict__ y, unsigned int* status) {
  using L = Layout<R, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  const uint32_t sbase = smem_addr(smem);
  const uint32_t full0 = sbase + L::kBars;
  const uint32_t empty0 = full0 + 8 * S;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nstages = K / kStageK;
  const int r0 = blockIdx.x * L::BR;
  const int m0 = blockIdx.y * 16;
  const int Ml = min(16, M - m0);
  x += (int64_t)m0 * K;
  y += (int64_t)m0 * N;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();

  float out[R][NT][4];
#pragma unroll
  for (int rt = 0; rt < R; ++rt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) out[rt][nt][e] = 0.f;

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_codes);
      prefetch_tensormap(&tm_scale);
      prefetch_tensormap(&tm_zero);
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int s = 0; s < nstages; ++s) {
        const int st = s % S;
        const uint32_t par = ((s / S) & 1) ^ 1;
        if (!mbar_wait(empty0 + 8 * st, par, status)) {
          aborted = 1;
          break;
        }
        const uint32_t fb = full0 + 8 * st;
        mbar_arrive_expect_tx(fb, L::kStageTx);
        const uint32_t cdst = sbase + L::kCodes + st * L::kCodeStage;
        tma_load_2d_hint(cdst, &tm_codes, s * (kStageK / 2), r0, fb, pol);
        tma_load_2d_hint(cdst + L::kCodeBox, &tm_codes, s * (kStageK / 2) + 128, r0, fb, pol);
        tma_load_2d_hint(sbase + L::kScales + st * L::kScaleStage, &tm_scale, s * kConsumers, r0,
                         fb, pol);
        tma_load_2d_hint(sbase + L::kZeros + st * L::kScaleStage, &tm_zero, s * kConsumers, r0, fb,
                         pol);
        issued = s + 1;
      }
      // Drain: never leave the CTA with copies still landing in its shared memory.
      for (int s = max(0, issued - S); s < issued; ++s)
        mbar_wait(full0 + 8 * (s % S), (s / S) & 1, status);
    }
  } else {
    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    const int w = warp;              // group of the stage this warp owns
    const int half = w >> 2, q = w & 3;
    const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nstages; ++s) {
      const int st = s % S;
      if (!mbar_wait(full0 + 8 * st, (s / S) & 1, status)) {
        aborted = 1;
        break;
      }
      const uint8_t* cbase = smem + L::kCodes + st * L::kCodeStage + half * L::kCodeBox;
      const __half* sc = reinterpret_cast<const __half*>(smem + L::kScales + st * L::kScaleStage);
      const __half* zr = reinterpret_cast<const __half*>(smem + L::kZeros + st * L::kScaleStage);
      uint2 wa[R], wb[R];
      float s_a[R], s_b[R], z_a[R], z_b[R];
#pragma unroll
      for (int rt = 0; rt < R; ++rt) {
        const int ra = 16 * rt + g, rb = ra + 8;
        const int chunk = 2 * q + (t >> 1);
        wa[rt] = *reinterpret_cast<const uint2*>(cbase + ra * 128 + ((chunk ^ (ra & 7)) << 4) +
                                                 8 * (t & 1));
        wb[rt] = *reinterpret_cast<const uint2*>(cbase + rb * 128 + ((chunk ^ (rb & 7)) << 4) +
                                                 8 * (t & 1));
        s_a[rt] = __half2float(sc[ra * 8 + w]);
        s_b[rt] = __half2float(sc[rb * 8 + w]);
        z_a[rt] = fmaf(-128.f, s_a[rt], __half2float(zr[ra * 8 + w]));
        z_b[rt] = fmaf(-128.f, s_b[rt], __half2float(zr[rb * 8 + w]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * st);

      // x fragment of group (s * 8 + w) and its sums over the group
      const int kofs = s * kStageK + 64 * w + 16 * t;
      uint32_t b[NT][4][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + g;
        load_x_frag(x + (int64_t)min(m, Ml - 1) * K + kofs, m < Ml, b[nt]);
      }
      float xs[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_bf16_16816(xs[nt], ones, b[nt][0][0], b[nt][0][1], zero4);
#pragma unroll
        for (int j = 1; j < 4; ++j) mma_bf16_16816(xs[nt], ones, b[nt][j][0], b[nt][j][1], xs[nt]);
      }
#pragma unroll
      for (int rt = 0; rt < R; ++rt) {
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          a_frag(wa[rt], wb[rt], j, a);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (j == 0)
              mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], zero4);
            else
              mma_bf16_16816(acc[nt], a, b[nt][j][0], b[nt][j][1], acc[nt]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          out[rt][nt][0] = fmaf(s_a[rt], acc[nt][0], fmaf(z_a[rt], xs[nt][0], out[rt][nt][0]));
          out[rt][nt][1] = fmaf(s_a[rt], acc[nt][1], fmaf(z_a[rt], xs[nt][1], out[rt][nt][1]));
          out[rt][nt][2] = fmaf(s_b[rt], acc[nt][2], fmaf(z_b[rt], xs[nt][2], out[rt][nt][2]));
          out[rt][nt][3] = fmaf(s_b[rt], acc[nt][3], fmaf(z_b[rt], xs[nt][3], out[rt][nt][3]));
        }
      }
    }
  }

  // ---- combine the consumer warps' partial sums (ring memory reused) and write bf16 -----------
  __syncthreads();
  if (aborted) return;
  constexpr int kCols = 16 * NT + 1;
  float* red = reinterpret_cast<float*>(smem);  // [kConsumers][BR][kCols]
  if (warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int rt = 0; rt < R; ++rt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* base = red + (warp * L::BR + 16 * rt + g) * kCols + nt * 8 + 2 * t;
        base[0] = out[rt][nt][0];
        base[1] = out[rt][nt][1];
        base[8 * kCols] = out[rt][nt][2];
        base[8 * kCols + 1] = out[rt][nt][3];
      }
  }
  __syncthreads();
  for (int o = threadIdx.x; o < L::BR * 16 * NT; o += kThreads) {
    const int r = o % L::BR;
    const int m = o / L::BR;
    const int n = r0 + r;
    if (n < N && m < Ml) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) v += red[(w * L::BR + r) * kCols + m];
      y[(int64_t)m * N + n] = __float2bfloat16_rn(v);
    }
  }
}

template <int NT, int R, int S>
int launch_tma(const void* x, int M, int K, const uint8_t* wq, const void* sc, const void* zr,
               int N, void* y, cudaStream_t stream) {
  using L = Layout<R, S>;
  static_assert(L::kCodeStage * S >= kConsumers * L::BR * (16 * NT + 1) * 4,
                "reduction buffer must fit in the ring");
  CUtensorMap tc, ts, tz;
  const int G = K / 64;
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, L::BR,
                              128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&ts, sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            L::BR, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tz, zr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            L::BR, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != RW4_OK) return st;
  auto kern = rw4_gemv_tma_kernel<NT, R, S>;
  // The dynamic shared memory limit is a per-device function attribute: set it once per device.
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kDynSmem) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "gemv_tma: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemv_tma: device status word unavailable");
  dim3 grid((N + L::BR - 1) / L::BR, (M + 15) / 16);
  kern<<<grid, kThreads, L::kDynSmem, stream>>>(tc, ts, tz,
                                                static_cast<const __nv_bfloat16*>(x), M, K, N,
                                                static_cast<__nv_bfloat16*>(y), status);
  return launch_status("rw4 gemv_tma launch");
}

}  // namespace

namespace rw4 {

bool gemv_tma_supported(int64_t K) { return K % kStageK == 0; }

int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles) {
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  if (M <= 8) {
    if (row_tiles == 4) return launch_tma<1, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (row_tiles == 2) return launch_tma<1, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    return launch_tma<1, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  }
  if (row_tiles >= 2) return launch_tma<2, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  return launch_tma<2, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
}

}  // namespace rw4

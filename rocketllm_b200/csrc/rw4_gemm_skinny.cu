// RW4 tcgen05 GEMM for batched decode (17-64 activation rows): y[M, N] = x[M, K] . W[N, K]^T with
// W in RW4 (exact fp32 weights c * s + z, as the dequant-GEMV multiplies them) and x, y bf16.
//
// Why a second tensor-core kernel.  The dequant-GEMV runs legacy mma.sync, whose issue rate caps it
// near half of HBM at 16 rows and a quarter at 32; the bf16 tcgen05 GEMM (rw4_gemm_tc.cu) spends
// ~3.5 instructions per weight materialising bf16(c * s + z), ~950 cycles per 64-wide k-block.
// Here each weight costs five eighths of an instruction: the codes enter the tensor cores as the
// fp16 bit patterns 1024 + c (low nibble) and 1024 + 16 c (high nibble, masked in place) -- one
// LOP3 per pair, the fragment order of rw4_gemv_frag.cuh -- and the activations as the x-prep
// pass's fp16 rows (x 2^e in low-nibble slots, x 2^(e-4) in high-nibble slots, the same order; one
// power of two per row, rw4_gemv_tma.cu).  A 64-wide k-block is one quantization group, so its
// four MMAs (K = 16 each) accumulate into their own TMEM buffer and the epilogue warps apply the
// group's scale and zero in fp32 registers:
//
//   D_g[n, m] = sum_k (1024 + c') x'          (the MMA result: 1024 sum x' + 2^e sum c x)
//   y[m, n]   = 2^-e_m sum_g ( s[n,g] (D_g[n,m] + off[g,m]) + z[n,g] xs[g,m] )
//
// with off = -1024 sum fp16 x' and xs = 2^e sum x the x-prep side pairs.  The per-group epilogue is
// 3 fp32 instructions per (row, column, group): cheaper than dequantizing for up to ~32 columns.
//
// Tile: 128 weight rows (UMMA M) x BN activation rows (UMMA N = 32 or 64: the whole batch), all of
// K per CTA.  Warp roles (11 warps):
//   warp 0      codes producer: TMA of [128 rows x 128 B] (four k-blocks, 128-byte swizzle, L2
//               evict-first) into an S1-stage ring;
//   warp 1      activation producer: TMA of the x-prep rows [BN x 64 fp16] (128-byte swizzle) and
//               the group's side pairs [2 BN fp32] per k-block into an S3-stage ring;
//   warp 2      allocates the TMEM (all 512 columns: accumulator buffers, then A stages), then one
//               lane issues the 4 MMAs of a k-block (A from TMEM, B from shared memory) into buffer
//               kb % NB and commits the A stage, the x slot and the buffer;
//   warps 3-6   expansion: one thread per weight row (= TMEM lane) writes the k-block's 64 codes as
//               fp16 patterns into its lane of an A stage with tcgen05.st (32 columns, two values
//               per column) -- the A operand never touches shared memory;
//   warps 7-10  epilogue: one thread per TMEM lane (weight row) reads the buffer (tcgen05.ld), frees
//               it, and folds it into BN fp32 accumulators; at the end 2^-e, bf16, store.
// Every mbarrier wait is bounded (rw4_tma.cuh); on a timeout the CTA stops, waits (bounded) for its
// MMAs, frees its TMEM and writes nothing.  Every TMA load is a plain per-CTA load.
#include <atomic>

#include "rw4_gemv_frag.cuh"
#include "rw4_tcgen05.cuh"
#include "rw4_xprep.cuh"

namespace {

using namespace rw4;

constexpr int kRows = 128;                       // weight rows per CTA (UMMA M)
constexpr int kCodeStageBytes = kRows * 128;     // four k-blocks of codes
constexpr int kExpandWarps = 4;
constexpr int kEpilogueWarps = 4;
constexpr int kSkThreads = 32 * (3 + kExpandWarps + kEpilogueWarps);

// Ring depths: a tcgen05.commit reaches its mbarrier long after the MMAs were issued (with a
// 4-deep ring handed back and forth per k-block the MMA issue rate halved in a probe), so eight
// k-blocks of A stages and activations are kept in flight.  With the A operand in shared memory
// (written by the expansion warps, read by the tensor core: 32 KB of traffic per k-block beside
// the codes and activations) the MMA thread spent ~650 of every ~1,040 cycles per k-block issuing;
// in TMEM it costs shared memory nothing.
template <int BN>
struct SkCfg {
  static constexpr int S1 = 4;                    // codes stages (4 k-blocks each)
  static constexpr int S2 = 8;                    // A stages (in TMEM, 32 columns each)
  static constexpr int S3 = 8;                    // activation stages
  static constexpr int NB = BN == 32 ? 8 : 4;     // TMEM accumulator buffers
  static constexpr int kXBytes = BN * 128;
  static constexpr int kSideBytes = BN * 8;
  static constexpr int kXStage = (kXBytes + kSideBytes + 1023) / 1024 * 1024;
  static constexpr int kOffCodes = 0;
  static constexpr int kOffX = kOffCodes + S1 * kCodeStageBytes;
  static constexpr int kOffBars = kOffX + S3 * kXStage;
  // cfull/cempty [S1], afull/aempty [S2], xfull/xempty [S3], accfull/accempty [NB], done
  static constexpr int kNumBars = 2 * S1 + 2 * S2 + 2 * S3 + 2 * NB + 1;
  static constexpr int kOffSlot = kOffBars + kNumBars * 8;
  static constexpr int kDynSmem = kOffSlot + 16 + 1024;
  static constexpr uint32_t kAccCols = NB * BN;        // accumulators: columns [0, kAccCols)
  static constexpr uint32_t kTmemCols = kAccCols + S2 * 32;   // then the A stages: 512
  // kind::f16 instruction descriptor: D f32, A and B f16 (type 0), both K-major, M = 128, N = BN
  static constexpr uint32_t kIdesc =
      (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
  static_assert(kDynSmem <= 227 * 1024, "shared memory budget");
  static_assert(kOffX % 1024 == 0 && kXStage % 1024 == 0, "swizzle atoms 1024-aligned");
  static_assert(kTmemCols == 512, "TMEM allocation: all 512 columns");
};

template <int BN>
__global__ void __launch_bounds__(kSkThreads, 1)
    rw4_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_codes,
                           const __grid_constant__ CUtensorMap tm_x,
                           const __grid_constant__ CUtensorMap tm_side,
                           const __half* __restrict__ scale, const __half* __restrict__ zero,
                           const int* __restrict__ row_exp, int M, int K, int N,
                           __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ res,
                           unsigned int* status) {
  using C = SkCfg<BN>;
  constexpr int S1 = C::S1, S2 = C::S2, S3 = C::S3, NB = C::NB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int aborted;
  const uint32_t sb = smem_addr(smem);
  const uint32_t cfull0 = sb + C::kOffBars;
  const uint32_t cempty0 = cfull0 + 8 * S1;
  const uint32_t afull0 = cempty0 + 8 * S1;
  const uint32_t aempty0 = afull0 + 8 * S2;
  const uint32_t xfull0 = aempty0 + 8 * S2;
  const uint32_t xempty0 = xfull0 + 8 * S3;
  const uint32_t accfull0 = xempty0 + 8 * S3;
  const uint32_t accempty0 = accfull0 + 8 * NB;
  const uint32_t done = accempty0 + 8 * NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kRows;
  const int nkb = K / 64;
  const int ncs = nkb / 4;
  const int G = K / 64;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < S1; ++s) {
      mbar_init(cfull0 + 8 * s, 1);
      mbar_init(cempty0 + 8 * s, kExpandWarps);
    }
    for (int s = 0; s < S2; ++s) {
      mbar_init(afull0 + 8 * s, kExpandWarps);
      mbar_init(aempty0 + 8 * s, 1);
    }
    for (int s = 0; s < S3; ++s) {
      mbar_init(xfull0 + 8 * s, 1);
      mbar_init(xempty0 + 8 * s, 1 + kEpilogueWarps);   // the MMA commit + the side readers
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(accfull0 + 8 * b, 1);
      mbar_init(accempty0 + 8 * b, kEpilogueWarps);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(smem_addr(tmem_slot), C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the activations come from the x-prep pass launched just before (programmatic launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---------------- codes producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_codes);
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int cs = 0; cs < ncs; ++cs) {
        const int s = cs % S1;
        if (!mbar_wait(cempty0 + 8 * s, ((cs / S1) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        mbar_arrive_expect_tx(cfull0 + 8 * s, kCodeStageBytes);
        tma_load_2d_hint(sb + C::kOffCodes + s * kCodeStageBytes, &tm_codes, cs * 128, n0,
                         cfull0 + 8 * s, pol);
        issued = cs + 1;
      }
      for (int cs = max(0, issued - S1); cs < issued; ++cs)   // drain own copies
        mbar_wait(cfull0 + 8 * (cs % S1), (cs / S1) & 1, status);
    }
  } else if (warp == 1) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      prefetch_tensormap(&tm_side);
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S3;
        if (!mbar_wait(xempty0 + 8 * s, ((kb / S3) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        const uint32_t dst = sb + C::kOffX + s * C::kXStage;
        mbar_arrive_expect_tx(xfull0 + 8 * s, C::kXBytes + C::kSideBytes);
        tma_load_2d(dst, &tm_x, kb * 64, 0, xfull0 + 8 * s);
        tma_load_2d(dst + C::kXBytes, &tm_side, 0, kb, xfull0 + 8 * s);
        issued = kb + 1;
      }
      for (int kb = max(0, issued - S3); kb < issued; ++kb)
        mbar_wait(xfull0 + 8 * (kb % S3), (kb / S3) & 1, status);
    }
  } else if (warp == 2) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int sa = kb % S2, sx = kb % S3, b = kb % NB;
        if (!mbar_wait(afull0 + 8 * sa, (kb / S2) & 1, status) ||
            !mbar_wait(xfull0 + 8 * sx, (kb / S3) & 1, status) ||
            !mbar_wait(accempty0 + 8 * b, ((kb / NB) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        tc_fence_after();
        const uint32_t ta = tmem + C::kAccCols + (uint32_t)(sa * 32);
        const uint64_t db = smem_desc(sb + C::kOffX + sx * C::kXStage);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // 16 values along K: 8 TMEM columns of A, 32 bytes of B
          umma_f16_ta(tmem + (uint32_t)(b * BN), ta + (uint32_t)(8 * kk), db + (uint64_t)(2 * kk),
                      C::kIdesc, kk > 0 ? 1u : 0u);
        umma_commit(aempty0 + 8 * sa);
        umma_commit(xempty0 + 8 * sx);
        umma_commit(accfull0 + 8 * b);
      }
      umma_commit(done);   // every MMA issued above has completed when this arrives
    }
  } else if (warp < 3 + kExpandWarps) {
    // ---------------- expansion: codes -> fp16 patterns in TMEM ----------------
    // a warp may store only to its own TMEM lane quarter (warp % 4): weight row = TMEM lane
    const int r = 32 * (warp & 3) + lane;
    for (int cs = 0; cs < ncs && !aborted; ++cs) {
      const int s1 = cs % S1;
      if (!mbar_wait(cfull0 + 8 * s1, (cs / S1) & 1, status)) {
        aborted = 1;
        break;
      }
      uint4 c[8];
      const uint32_t crow = sb + C::kOffCodes + s1 * kCodeStageBytes + r * 128;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t a = crow + ((q ^ (r & 7)) << 4);
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(c[q].x), "=r"(c[q].y), "=r"(c[q].z), "=r"(c[q].w)
                     : "r"(a));
      }
      // the TMA refill (async proxy) must not overtake these reads
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(cempty0 + 8 * s1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kb = cs * 4 + j;
        const int sa = kb % S2;
        if (!mbar_wait(aempty0 + 8 * sa, ((kb / S2) & 1) ^ 1, status)) {
          aborted = 1;
          break;
        }
        tc_fence_after();   // the MMAs that read this A stage have completed
        // the k-block's 8 code words (chunks 2j, 2j+1 of the row) -> the row's 32 A columns
        const uint32_t w[8] = {c[2 * j].x,     c[2 * j].y,     c[2 * j].z,     c[2 * j].w,
                               c[2 * j + 1].x, c[2 * j + 1].y, c[2 * j + 1].z, c[2 * j + 1].w};
        uint32_t a[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t v = w[q], v8 = w[q] >> 8;
          a[4 * q + 0] = frag::nib_lo_f16(v);
          a[4 * q + 1] = frag::nib_hi_f16(v);
          a[4 * q + 2] = frag::nib_lo_f16(v8);
          a[4 * q + 3] = frag::nib_hi_f16(v8);
        }
        tmem_st32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + C::kAccCols + (uint32_t)(sa * 32),
                  a);
        tc_fence_before();   // the stores, before the MMA thread's wait
        __syncwarp();
        if (lane == 0) mbar_arrive(afull0 + 8 * sa);
      }
    }
  } else {
    // ---------------- epilogue: per-group scale and zero, then the store ----------------
    const int q4 = warp & 3;                 // TMEM lane quarter this warp may access
    const int rl = 32 * q4 + lane;           // accumulator row = weight row n0 + rl
    const int n = n0 + rl;
    const int nc = min(n, N - 1);            // clamped for the scale loads; rows >= N not stored
    const __half* srow = scale + (int64_t)nc * G;
    const __half* zrow = zero + (int64_t)nc * G;
    float acc[BN];
#pragma unroll
    for (int m = 0; m < BN; ++m) acc[m] = 0.f;
    uint4 sc8 = make_uint4(0, 0, 0, 0), zr8 = sc8;
    for (int kb = 0; kb < nkb; ++kb) {
      const int b = kb % NB, sx = kb % S3, gi = kb & 7;
      if (gi == 0) {   // the scales and zeros of the next 8 groups (G is a multiple of 8)
        sc8 = __ldg(reinterpret_cast<const uint4*>(srow + kb));
        zr8 = __ldg(reinterpret_cast<const uint4*>(zrow + kb));
      }
      if (!mbar_wait(accfull0 + 8 * b, (kb / NB) & 1, status) ||
          !mbar_wait(xfull0 + 8 * sx, (kb / S3) & 1, status)) {
        aborted = 1;
        break;
      }
      tc_fence_after();
      uint32_t v[BN];
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32)
        tmem_ld32(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(b * BN + c0),
                  *reinterpret_cast<uint32_t(*)[32]>(&v[c0]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty0 + 8 * b);   // the buffer may take the next group
      const uint32_t sw = (gi < 4) ? ((gi < 2) ? sc8.x : sc8.y) : ((gi < 6) ? sc8.z : sc8.w);
      const uint32_t zw = (gi < 4) ? ((gi < 2) ? zr8.x : zr8.y) : ((gi < 6) ? zr8.z : zr8.w);
      const float s = __half2float(__ushort_as_half((unsigned short)(sw >> (16 * (gi & 1)))));
      const float z = __half2float(__ushort_as_half((unsigned short)(zw >> (16 * (gi & 1)))));
      const uint32_t side = sb + C::kOffX + sx * C::kXStage + C::kXBytes;
#pragma unroll
      for (int m = 0; m < BN; m += 2) {   // (xs, off) of columns m and m + 1
        float4 p;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(p.x), "=f"(p.y), "=f"(p.z), "=f"(p.w)
                     : "r"(side + 8 * m));
        acc[m] = fmaf(s, __uint_as_float(v[m]) + p.y, fmaf(z, p.x, acc[m]));
        acc[m + 1] = fmaf(s, __uint_as_float(v[m + 1]) + p.w, fmaf(z, p.z, acc[m + 1]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(xempty0 + 8 * sx);   // side pairs read
    }
    if (!aborted && n < N) {
#pragma unroll
      for (int m = 0; m < BN; ++m) {
        if (m < M) {
          float o = ldexpf(acc[m], -row_exp[m]);
          if (res) o = __bfloat162float(__float2bfloat16_rn(o)) +
                       __bfloat162float(res[(int64_t)m * N + n]);
          y[(int64_t)m * N + n] = __float2bfloat16_rn(o);
        }
      }
    }
  }

  // ---- teardown: every MMA this CTA issued has completed before TMEM is released -------------
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    if (lane == 0) mbar_wait(done, 0, status);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int BN>
int launch_bn(const void* x, int M, int K, const uint8_t* wq, const void* sc, const void* zr,
              int N, void* y, const XPrepLayout& l, uint8_t* ws, const void* res,
              cudaStream_t stream) {
  using C = SkCfg<BN>;
  const int G = K / 64;
  CUtensorMap tc, tx, tside;
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, kRows,
                              128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tx, ws + l.xf, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, M, K,
                            (uint64_t)K * 2, BN, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tside, ws + l.side, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, G,
                            2 * l.Mpad, (uint64_t)l.Mpad * 8, 1, 2 * BN,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != RW4_OK) return st;
  auto kern = rw4_gemm_skinny_kernel<BN>;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> dev) & 1)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmem) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "gemm_skinny: cannot set dynamic shared memory size");
    attr_set.fetch_or(1ull << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemm_skinny: device status word unavailable");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + kRows - 1) / kRows));
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = C::kDynSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = getenv("RW4_NO_PDL") ? 0 : 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(
      &cfg, kern, tc, tx, tside, static_cast<const __half*>(sc), static_cast<const __half*>(zr),
      reinterpret_cast<const int*>(ws + l.row_exp), M, K, N, static_cast<__nv_bfloat16*>(y),
      static_cast<const __nv_bfloat16*>(res), status);
  if (err != cudaSuccess) return cuda_status(err, "rw4 gemm_skinny launch");
  return launch_status("rw4 gemm_skinny launch");
}

}  // namespace

namespace rw4 {

// Rows 17-64, K a multiple of 512 (the x-prep layout and whole groups of 8 scales), and enough
// weight-row tiles to give most SMs one (no K split here).
bool gemm_skinny_supported(int64_t M, int64_t K, int64_t N) {
  static const bool off = getenv("RW4_SKINNY_OFF") != nullptr;
  return !off && M > 16 && M <= 64 && K % 512 == 0 && K <= (1 << 20) && N >= 96 * kRows &&
         N <= (1 << 30);
}

// The x-prep workspace of the same rows (xprep_layout(M, K).bytes) must be passed in `ws`.
int gemm_skinny_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                       const void* zr, int64_t N, void* y, cudaStream_t s, void* ws,
                       size_t ws_bytes, const void* res, const XNorm* norm) {
  const XPrepLayout l = xprep_layout(M, K);
  if (!ws || ws_bytes < l.bytes)
    return fail(RW4_EINVAL, "rw4_linear: the decode GEMM needs a %zu-byte workspace (got %zu)",
                l.bytes, ws_bytes);
  if (!aligned(ws, 256)) return fail(RW4_EINVAL, "rw4_linear: workspace must be 256-byte aligned");
  if (!aligned(sc, 16) || !aligned(zr, 16))
    return fail(RW4_EINVAL, "rw4_linear: scales and zeros must be 16-byte aligned");
  uint8_t* w = static_cast<uint8_t*>(ws);
  int st = xprep_launch(x, (int)M, (int)K, l, w, s, norm);
  if (st != RW4_OK) return st;
  if (M <= 32) return launch_bn<32>(x, (int)M, (int)K, wq, sc, zr, (int)N, y, l, w, res, s);
  return launch_bn<64>(x, (int)M, (int)K, wq, sc, zr, (int)N, y, l, w, res, s);
}

}  // namespace rw4

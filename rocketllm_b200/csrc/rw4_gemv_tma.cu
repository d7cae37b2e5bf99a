// RW4 dequant-GEMV, TMA-fed (K a multiple of 512): y[M, N] = x[M, K] . W[N, K]^T for decode
// batches, one 16-row batch slice per grid row.  The pipeline itself lives in
// rw4_gemv_tma_body.cuh; this file encodes the tensor maps and launches it.
#include <atomic>

#include "rw4_gemv_tma_body.cuh"

namespace {

using namespace rw4;
using namespace rw4::gemv_tma;

// Two CTAs per SM: the register cap this implies (<= 113 per thread) measurably improves the
// schedule (16 consumer warps per SM sharing the ALU pipe with the producers).  KS > 1 splits K
// over a (1, 1, KS) thread-block cluster (grid.z = KS) reduced through distributed shared memory.
// XT: activations through the TMA ring (default); otherwise the consumers load them from global
// memory (RW4_GEMV_X_GLOBAL=1, kept for comparison).  M1: one activation row.  XF: one row, in
// fp16 from shared memory (rw4_gemv_frag.cuh), the default for M = 1 when the CTA's K range fits
// 32 KB of shared memory (RW4_GEMV_NO_F16=1 keeps bf16).
template <int NT, int R, int S, int KS, bool XT, bool M1, bool XF = false>
__global__ void __cluster_dims__(1, 1, KS) __launch_bounds__(kThreads, 2)
    rw4_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_scale,
                        const __grid_constant__ CUtensorMap tm_zero,
                        const __grid_constant__ CUtensorMap tm_x,
                        const __nv_bfloat16* __restrict__ x, int bm, int M, int K, int N,
                        __nv_bfloat16* __restrict__ y, unsigned int* status) {
  // batch slices are the fastest grid dimension: the CTAs of all slices of one row tile run
  // together, so the slices after the first find the tile's weights in L2
  const int m0 = blockIdx.x * 16;
  body<NT, R, S, false, KS, XT, M1, XF>(&tm_codes, &tm_scale, &tm_zero, &tm_x, x, m0, bm,
                                        min(16, M - m0), K, y + (int64_t)m0 * N, N,
                                        blockIdx.y * Layout<R, S>::BR, N, 0, status);
}

bool pdl_enabled() {
  static const bool off = getenv("RW4_NO_PDL") != nullptr;
  return !off;
}

// Smallest dynamic shared memory request that keeps a third CTA off an SM (228 KB per SM, 1 KB
// reserved per CTA).
constexpr int kTwoPerSmSmem = 228 * 1024 / 3 + 1024;

constexpr int kF16MaxStages = 32;  // fp16 activation row in shared memory: 1 KB per stage

bool no_f16() {
  static const bool on = getenv("RW4_GEMV_NO_F16") != nullptr;
  return on;
}

bool x_global() {
  static const bool on = getenv("RW4_GEMV_X_GLOBAL") != nullptr;
  return on;
}

template <int NT, int R, int S, int KS = 1>
int launch_tma(const void* x, int M, int K, const uint8_t* wq, const void* sc, const void* zr,
               int N, void* y, cudaStream_t stream) {
  using L = Layout<R, S>;
  static_assert(L::kBars >= kConsumers * L::BR * (16 * NT + 1) * 4,
                "reduction buffer must fit in the ring below the barriers");
  CUtensorMap tc, ts, tz, tx;
  const int G = K / 64;
  // activation rows per slice: the whole batch for M <= 8 (NT = 1), 16-row slices above
  const int bm = M < 16 ? M : 16;
  if (bm > 8 * NT) return fail(RW4_EINVAL, "gemv_tma: %d activation rows for NT=%d", M, NT);
  int st = make_tensor_map_2d(&tc, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K / 2, K / 2, L::BR,
                              128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&ts, sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            L::BR, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tz, zr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, N, G, (uint64_t)G * 2,
                            L::BR, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == RW4_OK)
    st = make_tensor_map_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, (uint64_t)K * 2,
                            bm, 256, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != RW4_OK) return st;
  const bool xt = !x_global();
  const bool m1 = NT == 1 && M == 1;
  const int cta_stages = ((K / kStageK) + KS - 1) / KS;
  const bool xf = m1 && xt && !no_f16() && cta_stages <= kF16MaxStages;
  const int variant = xf ? 4 : (xt ? 0 : 1) + (m1 ? 2 : 0);
  auto kern = xf ? rw4_gemv_tma_kernel<NT, R, S, KS, false, NT == 1, NT == 1>
              : xt ? (m1 ? rw4_gemv_tma_kernel<NT, R, S, KS, true, NT == 1>
                         : rw4_gemv_tma_kernel<NT, R, S, KS, true, false>)
                   : (m1 ? rw4_gemv_tma_kernel<NT, R, S, KS, false, NT == 1>
                         : rw4_gemv_tma_kernel<NT, R, S, KS, false, false>);
  // The dynamic shared memory limit is a per-device function attribute: set it once per device
  // and kernel variant.
  static std::atomic<uint32_t> attr_set[5];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set[variant].load() & (1u << dev))) {
    const int need = xf ? L::kX + kF16MaxStages * 1024 + 1024 : L::dyn_smem(8 * NT);
    const int most = need > kTwoPerSmSmem ? need : kTwoPerSmSmem;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, most) !=
        cudaSuccess)
      return fail(RW4_ECUDA, "gemv_tma: cannot set dynamic shared memory size");
    attr_set[variant].fetch_or(1u << dev);
  }
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "gemv_tma: device status word unavailable");
  const int64_t tiles = (N + L::BR - 1) / L::BR;
  if (tiles > 65535) return fail(RW4_EINVAL, "gemv_tma: N=%d needs more than 65535 row tiles", N);
  dim3 grid((M + 15) / 16, (unsigned)tiles, KS);
  // Programmatic dependent launch: this grid may start while the previous kernel on the stream
  // drains; it streams its weights at once and waits (griddepcontrol.wait) only before it reads x.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  // At most two CTAs per SM: with smaller rings the block scheduler may stack three or four CTAs
  // of a one-wave grid on some SMs and leave others idle (measured: M=1 slower than M=8 on the
  // 4096-row shapes until the shared-memory request made a third CTA impossible).
  const int smem_need = xf ? L::kX + cta_stages * 1024 + 1024
                        : xt ? L::dyn_smem(bm) : L::kX + 1024;
  cfg.dynamicSmemBytes = smem_need > kTwoPerSmSmem ? smem_need : kTwoPerSmSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tc, ts, tz, tx,
                                       static_cast<const __nv_bfloat16*>(x), bm, M, K, N,
                                       static_cast<__nv_bfloat16*>(y), status);
  if (err != cudaSuccess) return cuda_status(err, "rw4 gemv_tma launch");
  return launch_status("rw4 gemv_tma launch");
}

}  // namespace

namespace rw4 {

bool gemv_tma_supported(int64_t K) { return K % kStageK == 0; }

// Launch shape policy (measured on the isolated sweep and the Llama / Mixtral projection shapes,
// decode M = 1 and 16).  Wider CTAs amortise the per-stage work (x fragment, barrier, all-ones
// MMA) over more weight rows and win whenever they still give about 1.5 CTAs per SM (>= 222 of
// the 296 two-per-SM slots): 64-row CTAs (M <= 8 only) from N >= 14208, then 32-row CTAs, then
// 16-row CTAs, each with K split over a cluster of up to 4 CTAs (keeping >= 2 stages per CTA) to
// reach that count.  9..16 activation rows always use 32-row CTAs; their K loops are twice as
// costly, so long-K weights (>= 64 stages) also split K in two.
void gemv_tma_policy(int64_t M, int64_t K, int64_t N, int* row_tiles, int* ksplit) {
  constexpr int64_t kTarget = 222;
  const int64_t slices = (M + 15) / 16;
  const int64_t nst = K / kStageK;
  auto ctas = [&](int r) { return (N + 16 * r - 1) / (16 * r) * slices; };
  auto split_for = [&](int r) {
    int ks = 1;
    while (ks < 4 && ctas(r) * ks < kTarget && nst / (ks * 2) >= 2) ks *= 2;
    return ks;
  };
  if (M > 8) {
    *row_tiles = 2;
    int ks = split_for(2);
    if (ks == 1 && nst >= 64 && ctas(2) * 2 <= 1200) ks = 2;
    *ksplit = ks;
    return;
  }
  if (ctas(4) >= kTarget) {
    *row_tiles = 4;
    *ksplit = 1;
    return;
  }
  for (int r : {2, 1}) {
    const int ks = split_for(r);
    if (ctas(r) * ks >= kTarget || r == 1) {
      *row_tiles = r;
      *ksplit = ks;
      return;
    }
  }
}

int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles) {
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  static const int forced_ks = [] {
    const char* e = getenv("RW4_GEMV_KSPLIT");
    return e ? atoi(e) : 0;
  }();
  int policy_rt = 1, ks = 1;
  gemv_tma_policy(M, K, N, &policy_rt, &ks);
  if (row_tiles != 1 && row_tiles != 2 && row_tiles != 4) row_tiles = policy_rt;
  if (row_tiles == 4 && M > 8) row_tiles = 2;
  if (forced_ks == 1 || forced_ks == 2 || forced_ks == 4) ks = forced_ks;
  if (row_tiles >= 4) ks = 1;
  if (M == 1 && !no_f16()) {
    // the fp16 one-row path holds the CTA's activation row in shared memory (<= 32 stages):
    // split a longer K over a cluster, 64-row CTAs included
    int need = 1;
    while (need < 4 && (K / kStageK + need - 1) / need > kF16MaxStages) need *= 2;
    if (need > ks) ks = need;
  }
  if (M <= 8) {
    if (row_tiles == 4) {
      if (ks == 4) return launch_tma<1, 4, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      if (ks == 2) return launch_tma<1, 4, 4, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      return launch_tma<1, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    }
    if (row_tiles == 2) {
      if (ks == 4) return launch_tma<1, 2, 6, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      if (ks == 2) return launch_tma<1, 2, 6, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      return launch_tma<1, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    }
    if (ks == 4) return launch_tma<1, 1, 8, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (ks == 2) return launch_tma<1, 1, 8, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    return launch_tma<1, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  }
  // 9..16 activation rows: 16 KB of x per stage, so shallower rings keep two CTAs per SM
  if (row_tiles >= 2) {
    if (ks == 4) return launch_tma<2, 2, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (ks == 2) return launch_tma<2, 2, 4, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    return launch_tma<2, 2, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  }
  if (ks == 4) return launch_tma<2, 1, 5, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  if (ks == 2) return launch_tma<2, 1, 5, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  return launch_tma<2, 1, 5>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
}

}  // namespace rw4

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
template <int NT, int R, int S, int KS>
__global__ void __cluster_dims__(1, 1, KS) __launch_bounds__(kThreads, 2)
    rw4_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_scale,
                        const __grid_constant__ CUtensorMap tm_zero,
                        const __nv_bfloat16* __restrict__ x, int M, int K, int N,
                        __nv_bfloat16* __restrict__ y, unsigned int* status) {
  const int m0 = blockIdx.y * 16;
  body<NT, R, S, false, KS>(&tm_codes, &tm_scale, &tm_zero, x + (int64_t)m0 * K,
                            min(16, M - m0), K, y + (int64_t)m0 * N, N,
                            blockIdx.x * Layout<R, S>::BR, N, 0, status);
}

bool pdl_enabled() {
  static const bool off = getenv("RW4_NO_PDL") != nullptr;
  return !off;
}

template <int NT, int R, int S, int KS = 1>
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
  auto kern = rw4_gemv_tma_kernel<NT, R, S, KS>;
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
  dim3 grid((N + L::BR - 1) / L::BR, (M + 15) / 16, KS);
  // Programmatic dependent launch: this grid may start while the previous kernel on the stream
  // drains; it streams its weights at once and waits (griddepcontrol.wait) only before it reads x.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kDynSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tc, ts, tz,
                                       static_cast<const __nv_bfloat16*>(x), M, K, N,
                                       static_cast<__nv_bfloat16*>(y), status);
  if (err != cudaSuccess) return cuda_status(err, "rw4 gemv_tma launch");
  return launch_status("rw4 gemv_tma launch");
}

}  // namespace

namespace rw4 {

bool gemv_tma_supported(int64_t K) { return K % kStageK == 0; }

int gemv_tma_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                    const void* zr, int64_t N, void* y, cudaStream_t s, int row_tiles) {
  const int Mi = (int)M, Ki = (int)K, Ni = (int)N;
  // K split over a cluster only when the row tiles alone leave SMs idle (< 148 CTAs; measured: with
  // 256+ CTAs the cluster barrier costs more than the shorter K loop saves), keeping >= 2 stages
  // (1024 of K) per CTA.
  static const int forced_ks = [] {
    const char* e = getenv("RW4_GEMV_KSPLIT");
    return e ? atoi(e) : 0;
  }();
  const int64_t ctas = ((N + 16 * row_tiles - 1) / (16 * row_tiles)) * ((M + 15) / 16);
  const int64_t nst = K / kStageK;
  int ks = 1;
  while (ks < 4 && ctas * ks < 148 && nst / (ks * 2) >= 2) ks *= 2;
  if (forced_ks == 1 || forced_ks == 2 || forced_ks == 4) ks = forced_ks;
  if (row_tiles >= 4) ks = 1;
  if (M <= 8) {
    if (row_tiles == 4) return launch_tma<1, 4, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (row_tiles == 2) {
      if (ks == 4) return launch_tma<1, 2, 6, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      if (ks == 2) return launch_tma<1, 2, 6, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
      return launch_tma<1, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    }
    if (ks == 4) return launch_tma<1, 1, 8, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (ks == 2) return launch_tma<1, 1, 8, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    return launch_tma<1, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  }
  if (row_tiles >= 2) {
    if (ks == 4) return launch_tma<2, 2, 6, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    if (ks == 2) return launch_tma<2, 2, 6, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
    return launch_tma<2, 2, 6>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  }
  if (ks == 4) return launch_tma<2, 1, 8, 4>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  if (ks == 2) return launch_tma<2, 1, 8, 2>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
  return launch_tma<2, 1, 8>(x, Mi, Ki, wq, sc, zr, Ni, y, s);
}

}  // namespace rw4

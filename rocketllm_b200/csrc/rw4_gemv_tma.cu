// RW4 dequant-GEMV, TMA-fed (K a multiple of 512): y[M, N] = x[M, K] . W[N, K]^T for decode
// batches, one 16-row batch slice per grid row.  The pipeline itself lives in
// rw4_gemv_tma_body.cuh; this file encodes the tensor maps and launches it.
#include <atomic>

#include "rw4_gemv_tma_body.cuh"

namespace {

using namespace rw4;
using namespace rw4::gemv_tma;

// Two CTAs per SM: the register cap this implies (<= 113 per thread) measurably improves the
// schedule (16 consumer warps per SM sharing the ALU pipe with the producers).
template <int NT, int R, int S>
__global__ void __launch_bounds__(kThreads, 2)
    rw4_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_scale,
                        const __grid_constant__ CUtensorMap tm_zero,
                        const __nv_bfloat16* __restrict__ x, int M, int K, int N,
                        __nv_bfloat16* __restrict__ y, unsigned int* status) {
  const int m0 = blockIdx.y * 16;
  body<NT, R, S, false>(&tm_codes, &tm_scale, &tm_zero, x + (int64_t)m0 * K, min(16, M - m0), K,
                        y + (int64_t)m0 * N, N, blockIdx.x * Layout<R, S>::BR, N, 0, status);
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

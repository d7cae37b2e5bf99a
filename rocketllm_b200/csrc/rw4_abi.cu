// Entry points of the RW4 C ABI that are not tied to one kernel file: version, error reporting,
// device queries and the rw4_linear dispatcher.
#include <mutex>
#include <string>
#include <vector>

#include "rw4_common.cuh"
#include "rw4_tma.cuh"
#include "rw4_xprep.cuh"

namespace rw4 {

namespace {
thread_local std::string g_last_error;
}

void set_error_message(const char* msg) { g_last_error = msg ? msg : ""; }

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int gemv_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                const void* zr, int64_t N, void* y, cudaStream_t s, void* ws, size_t ws_bytes);
size_t gemv_workspace(int64_t M, int64_t K, int64_t N);
int gemm_tc_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                   const void* zr, int64_t N, void* y, cudaStream_t s);
bool gemm_tc_supported(int64_t M, int64_t K, int64_t N);
bool gemm_skinny_supported(int64_t M, int64_t K, int64_t N);
int gemm_skinny_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                       const void* zr, int64_t N, void* y, cudaStream_t s, void* ws,
                       size_t ws_bytes, const void* res, const XNorm* norm = nullptr);

// Shape / pointer validation shared by every RW4 matmul entry point.
int check_linear_args(const char* who, const void* x, int64_t M, int64_t K, const uint8_t* wq,
                      const void* sc, const void* zr, int64_t N, int32_t group, const void* y) {
  if (M < 0 || K <= 0 || N < 0)
    return fail(RW4_EINVAL, "%s: bad shape M=%lld K=%lld N=%lld", who, (long long)M,
                (long long)K, (long long)N);
  if (group != 64) return fail(RW4_EINVAL, "%s: group %d unsupported (64 only)", who, group);
  if (K % 64) return fail(RW4_EINVAL, "%s: K=%lld is not a multiple of 64", who, (long long)K);
  if (K > (1ll << 30) || N > (1ll << 30) || M > (1ll << 30))
    return fail(RW4_EINVAL, "%s: dimension beyond 2^30", who);
  if (M == 0 || N == 0) return RW4_OK;
  if (!x || !wq || !sc || !zr || !y) return fail(RW4_EINVAL, "%s: null pointer", who);
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(wq, 16) || !aligned(sc, 8) || !aligned(zr, 8))
    return fail(RW4_EINVAL, "%s: x/y/packed must be 16-byte and scale/zero 8-byte aligned", who);
  if ((N * 2) % 16)
    return fail(RW4_EINVAL, "%s: N=%lld must be a multiple of 8 (16-byte output rows)", who,
                (long long)N);
  return RW4_OK;
}

}  // namespace rw4

extern "C" int rw4_version(void) { return 100; }

extern "C" int rw4_last_error(char* buf, size_t n) {
  const std::string& e = rw4::g_last_error;
  if (buf && n) {
    const size_t c = e.size() < n - 1 ? e.size() : n - 1;
    memcpy(buf, e.data(), c);
    buf[c] = 0;
  }
  return (int)e.size();
}

// Paths: 1 the dequant-GEMV (up to 16 rows); 3 the GEMV in 16-row batch slices (17-64 rows);
// 4 the tcgen05 decode GEMM (17-64 rows, K % 512 == 0, N >= 12288), chosen for 49-64 rows, where it
// measured faster than the slices (below that the slices win: its k-blocks advance at ~1,000 cycles
// whatever the row count); 2 the bf16 tcgen05 GEMM (more rows).  Paths 1, 3 and 4 multiply by the
// exact fp32 weight; the GEMV gives a row the same bits at every M <= 16 (and in every 16-row
// slice), so decode steps and speculative verify passes round like a one-token step; the decode
// GEMM gives a row the same bits at every M in 17-32 and in 33-64.  Path 2 (prefill-sized M)
// multiplies by the reference's bf16-rounded dequantized weight, as the reference's F.linear over
// dequantize().to(bf16) does.
constexpr int64_t kGemvMaxRows = 64;
constexpr int64_t kDecodeGemmMinRows = 49;

extern "C" int rw4_linear_path(int64_t M, int64_t K, int64_t N) {
  if (M < 0 || K <= 0 || N < 0 || K % 64) return RW4_EINVAL;
  if (M <= 16) return 1;
  if (M >= kDecodeGemmMinRows && M <= kGemvMaxRows && rw4::gemm_skinny_supported(M, K, N))
    return 4;
  if (M > kGemvMaxRows && rw4::gemm_tc_supported(M, K, N)) return 2;
  return 3;
}

extern "C" int rw4_linear_workspace_size(int64_t M, int64_t K, int64_t N, int32_t path,
                                         size_t* bytes) {
  using namespace rw4;
  if (!bytes) return fail(RW4_EINVAL, "rw4_linear_workspace_size: null output");
  *bytes = 0;
  if (M < 0 || K <= 0 || N < 0 || K % 64)
    return fail(RW4_EINVAL, "rw4_linear_workspace_size: bad shape M=%lld K=%lld N=%lld",
                (long long)M, (long long)K, (long long)N);
  if (path == 0) path = rw4_linear_path(M, K, N);
  if (M > 0 && N > 0 && (path == 1 || path == 3 || path == 4)) *bytes = gemv_workspace(M, K, N);
  return RW4_OK;
}

extern "C" int rw4_linear_ws(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                             const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                             void* y_bf16, int32_t path, void* workspace, size_t workspace_bytes,
                             void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear", x_bf16, M, K, packed, scale_f16, zero_f16, N, group,
                             y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  if (path == 0) path = rw4_linear_path(M, K, N);
  if (path == 2 && !gemm_tc_supported(M, K, N))
    return fail(RW4_EINVAL, "rw4_linear: the tensor-core GEMM needs M > 16 (M=%lld)",
                (long long)M);
  if (path == 4 && !gemm_skinny_supported(M, K, N))
    return fail(RW4_EINVAL, "rw4_linear: the decode GEMM needs 17-64 rows, K %% 512 == 0 and "
                "N >= 12288 (M=%lld K=%lld N=%lld)", (long long)M, (long long)K, (long long)N);
  cudaStream_t s = as_stream(stream);
  switch (path) {
    case 1:
    case 3:
      return gemv_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s, workspace,
                         workspace_bytes);
    case 2:
      return gemm_tc_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s);
    case 4:
      return gemm_skinny_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, s,
                                workspace, workspace_bytes, nullptr);
    default:
      return fail(RW4_EINVAL, "rw4_linear: no path %d for M=%lld K=%lld N=%lld", path,
                  (long long)M, (long long)K, (long long)N);
  }
}

// The entry points without a workspace argument take one, when the call needs one, from the
// device's stream-ordered pool (cudaMallocAsync / cudaFreeAsync on the caller's stream).
extern "C" int rw4_linear_on_path(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                                  const void* scale_f16, const void* zero_f16, int64_t N,
                                  int32_t group, void* y_bf16, int32_t path, void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear", x_bf16, M, K, packed, scale_f16, zero_f16, N, group,
                             y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  size_t bytes = 0;
  st = rw4_linear_workspace_size(M, K, N, path, &bytes);
  if (st != RW4_OK) return st;
  cudaStream_t s = as_stream(stream);
  void* ws = nullptr;
  if (bytes) {
    st = cuda_status(cudaMallocAsync(&ws, bytes, s), "rw4_linear workspace");
    if (st != RW4_OK) return st;
  }
  st = rw4_linear_ws(x_bf16, M, K, packed, scale_f16, zero_f16, N, group, y_bf16, path, ws,
                     bytes, stream);
  if (ws) {
    const int fst = cuda_status(cudaFreeAsync(ws, s), "rw4_linear workspace release");
    if (st == RW4_OK) st = fst;
  }
  return st;
}

extern "C" int rw4_linear(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                          const void* scale_f16, const void* zero_f16, int64_t N, int32_t group,
                          void* y_bf16, void* stream) {
  return rw4_linear_on_path(x_bf16, M, K, packed, scale_f16, zero_f16, N, group, y_bf16, 0,
                            stream);
}

// ---- device status word and TMA descriptors ---------------------------------------------------

namespace {
__device__ unsigned int g_device_status_word = 0;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

namespace rw4 {

unsigned int* device_status_ptr() {
  static std::mutex mu;
  static std::vector<unsigned int*> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, nullptr);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status_word) == cudaSuccess)
      cache[dev] = static_cast<unsigned int*>(p);
  }
  return cache[dev];
}

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                       int elem_bytes, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                       uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(RW4_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned(base, 16) || row_bytes % 16 || (box_cols * elem_bytes) % 16)
    return fail(RW4_EINVAL, "tensor map: base/pitch/box not 16-byte aligned");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(RW4_ECUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u",
                (int)r, (unsigned long long)rows, (unsigned long long)cols, box_rows, box_cols);
  return RW4_OK;
}

}  // namespace rw4

extern "C" int rw4_device_status(uint32_t* word, int32_t clear, void* stream) {
  using namespace rw4;
  if (!word) return fail(RW4_EINVAL, "rw4_device_status: null output");
  unsigned int* p = device_status_ptr();
  if (!p) return fail(RW4_ECUDA, "rw4_device_status: no device status word");
  cudaStream_t s = as_stream(stream);
  unsigned int v = 0;
  int st = cuda_status(cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, s),
                       "rw4_device_status read");
  if (st == RW4_OK && clear) st = cuda_status(cudaMemsetAsync(p, 0, sizeof(v), s), "clear");
  if (st == RW4_OK) st = cuda_status(cudaStreamSynchronize(s), "rw4_device_status sync");
  *word = v;
  return st;
}

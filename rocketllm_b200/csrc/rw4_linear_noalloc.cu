// rw4_linear_noalloc: the decode GEMV for callers that cannot allocate device memory per call.
//
// rw4_linear needs a few megabytes of device scratch for the converted activations and takes it
// from the stream-ordered pool; rw4_linear_ws takes it from the caller.  Some callers can do
// neither: a host that budgets every byte of VRAM up front (a streaming engine that sizes its
// layer slots from the free memory it measured at start-up, a serving process with a fixed memory
// plan) must not have a library allocate behind its back, and a C caller may have no allocator to
// hand a workspace from at all.  This entry point runs the same GEMV with its scratch in a
// fixed-size array that is part of the library's device image: nothing is allocated or freed per
// call.
//
// The array (kScratchBytes) is reserved on every GPU that loads the library, until the process
// exits.  Its device address is looked up once per device (cudaGetSymbolAddress, with that device
// current) on the first call on that device.  Every call shares it, so calls whose work can
// overlap on the GPU -- several streams, several host threads -- race on it and must be serialised
// by the caller.  It keeps the last call's contents; nothing in it has to start at zero, because
// the activation-conversion pass rewrites every byte the GEMV then reads.
#include <mutex>

#include "rw4_common.cuh"

namespace rw4 {
int check_linear_args(const char* who, const void* x, int64_t M, int64_t K, const uint8_t* wq,
                      const void* sc, const void* zr, int64_t N, int32_t group, const void* y);
int gemv_launch(const void* x, int64_t M, int64_t K, const uint8_t* wq, const void* sc,
                const void* zr, int64_t N, void* y, cudaStream_t s, void* ws, size_t ws_bytes);
size_t gemv_workspace(int64_t M, int64_t K, int64_t N);
}  // namespace rw4

namespace {

// 4 MiB: the converted activations of up to about 2 M values (e.g. 64 rows of K = 16384, or 16
// rows of K = 53248), plus their per-group sums.
constexpr size_t kScratchBytes = size_t(4) << 20;
constexpr int kMaxRows = 64;  // the GEMV's row limit (16-row slices above 16 rows)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

// Device address of g_scratch on the current device.  In host code the name g_scratch is only a
// host-side stand-in for the symbol, never a device address, so it is never passed to a kernel.
int scratch_address(uint8_t** out) {
  static std::mutex mu;
  static uint8_t* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return rw4::cuda_status(err, "rw4_linear_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return rw4::fail(RW4_EUNSUPPORTED, "rw4_linear_noalloc: device %d beyond %d", dev,
                     kMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_scratch);
    if (err != cudaSuccess || !p)
      return rw4::cuda_status(err != cudaSuccess ? err : cudaErrorInvalidSymbol,
                              "rw4_linear_noalloc: cudaGetSymbolAddress of its scratch");
    addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = addr[dev];
  return RW4_OK;
}

}  // namespace

extern "C" int rw4_linear_noalloc(const void* x_bf16, int64_t M, int64_t K, const uint8_t* packed,
                                  const void* scale_f16, const void* zero_f16, int64_t N,
                                  int32_t group, void* y_bf16, void* stream) {
  using namespace rw4;
  int st = check_linear_args("rw4_linear_noalloc", x_bf16, M, K, packed, scale_f16, zero_f16, N,
                             group, y_bf16);
  if (st != RW4_OK || M == 0 || N == 0) return st;
  if (M > kMaxRows)
    return fail(RW4_EINVAL,
                "rw4_linear_noalloc: M=%lld rows; this entry point runs the GEMV, at most %d rows "
                "(rw4_linear runs larger M on the tensor-core GEMM, which needs no scratch)",
                (long long)M, kMaxRows);
  const size_t need = gemv_workspace(M, K, N);
  if (need > kScratchBytes)
    return fail(RW4_EINVAL,
                "rw4_linear_noalloc: M=%lld x K=%lld needs %zu bytes of scratch; its fixed "
                "scratch holds %zu (about M*K <= 2M values)",
                (long long)M, (long long)K, need, kScratchBytes);
  uint8_t* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != RW4_OK) return st;
  return gemv_launch(x_bf16, M, K, packed, scale_f16, zero_f16, N, y_bf16, as_stream(stream),
                     scratch, kScratchBytes);
}

// RW4 tensor-core GEMM for prefill and batched decode (M > 16).  Placeholder until the tcgen05
// kernel lands: reports itself unsupported so rw4_linear routes to the GEMV slices.
#include "rw4_common.cuh"

namespace rw4 {
bool gemm_tc_supported(int64_t, int64_t, int64_t) { return false; }
int gemm_tc_launch(const void*, int64_t, int64_t, const uint8_t*, const void*, const void*,
                   int64_t, void*, cudaStream_t) {
  return fail(RW4_EUNSUPPORTED, "tcgen05 GEMM not built");
}
}  // namespace rw4

// Diagnostic: the bounded mbarrier wait every kernel of this library uses (rw4_tma.cuh), run on a
// barrier whose phase either completes (arrive != 0: thread 0 arrives first) or never does
// (arrive == 0: nobody arrives).  In the second case every thread's wait gives up after the
// library's limit (1 s of %globaltimer), sets RW4_DEVERR_TIMEOUT in the device status word and the
// kernel returns normally -- the path a kernel takes when a copy it waits for never lands, checked
// without faulting or hanging anything.
#include "rw4_common.cuh"
#include "rw4_tma.cuh"

namespace {

using namespace rw4;

__global__ void wait_selftest_kernel(int arrive, unsigned int* status) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) mbar_arrive(b);
  mbar_wait(b, 0, status);
}

}  // namespace

extern "C" int rw4_wait_selftest(int32_t arrive, void* stream) {
  unsigned int* status = device_status_ptr();
  if (!status) return fail(RW4_ECUDA, "rw4_wait_selftest: device status word unavailable");
  wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(arrive ? 1 : 0, status);
  return launch_status("rw4_wait_selftest launch");
}

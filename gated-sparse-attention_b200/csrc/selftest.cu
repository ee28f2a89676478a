// Diagnostic kernel of the failure-handling path: one CTA waits, through the same bounded
// mbarrier wait every pipelined kernel uses, on a barrier that nothing ever arrives on.  The
// wait gives up after ``limit`` polls, records GSA_ERR_TIMEOUT in the device error word and the
// kernel returns -- no trap, no unbounded spin -- so that a host can check the whole route
// (bounded wait -> error word -> gsa_get_device_error) without a real fault.
#include "kernels.cuh"

namespace gsa {
namespace {

__global__ void wait_selftest_kernel(uint32_t limit, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // phase 0 of a fresh barrier completes only when one arrival is made; none is
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, err, limit);
  __syncthreads();
}

}  // namespace

int launch_wait_selftest(uint32_t limit, int* err, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit, err);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa

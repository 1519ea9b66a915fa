// Self-test of the bounded-wait error path that every kernel of the library
// shares: one CTA waits on an mbarrier phase that nothing completes.  The
// wait gives up after its time limit (common.cuh, 1 s of %globaltimer) and
// records kDeviceErrWaitTimeout in the device error word, and the kernel
// returns normally, so the context stays usable.  Nothing faults or hangs.
#include "common.cuh"
#include "kernels.h"

namespace qsa {
namespace {

__global__ void wait_timeout_selftest_kernel(int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival would complete phase 0; none comes
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0)) record_error(err, kDeviceErrWaitTimeout);
}

}  // namespace

cudaError_t launch_wait_timeout_selftest(int* err, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(err);
  return count_launches(cudaGetLastError());
}

}  // namespace qsa

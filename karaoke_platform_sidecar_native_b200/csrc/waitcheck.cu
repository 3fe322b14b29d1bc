// Failure-path check of the kernels' bounded waits.
//
// One CTA arms an mbarrier for a transfer that is never issued and waits on it
// with the same wait loop the tcgen05 kernels use (mbar_wait_limit), under a
// caller-given limit.  Nothing is in flight (no TMA, no MMA), so when the wait
// runs out the kernel records its error code and simply returns: the host then
// takes the path every kernel wait timeout takes.  Used only by the test of
// that path; the production kernels wait with the fixed kWaitLimitNs.
#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {
namespace {

__global__ void wait_check_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // Completes only when 1024 bytes arrive; no copy is ever issued.
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar, 1024u);
  __syncthreads();
  mbar_wait_limit(&bar, 0, &abort_flag, err, kErrWaitTma, limit_ns);
}

}  // namespace

cudaError_t launch_wait_check(int* err, unsigned long long limit_ns, cudaStream_t stream) {
  wait_check_kernel<<<1, 128, 0, stream>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace vab

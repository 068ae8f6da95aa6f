// sfa_selftest.cu — the failure path of the kernels' bounded waits, exercised
// without a fault: one warp waits on an mbarrier that nothing ever arrives on,
// with a short limit, through the same wait (mbar_wait) and status word
// (record_status) every tensor-core kernel uses.  The wait gives up, the code
// lands in the device status word, the kernel returns and the context stays
// usable.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"

namespace sfa {
using namespace tc;

constexpr int32_t kSelftestCode = SFA_SELFTEST_STATUS;   // kernel 15 (self-test), site 1

__global__ void __launch_bounds__(32) wait_probe_kernel(uint64_t limit_ns, int32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  // phase 0 needs one arrival, and no thread arrives: the wait runs out
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, limit_ns)) record_status(status, kSelftestCode);
}

cudaError_t launch_wait_probe(uint32_t limit_us, int32_t* status, cudaStream_t st) {
  wait_probe_kernel<<<1, 32, 0, st>>>((uint64_t)limit_us * 1000ull, status);
  return cudaGetLastError();
}

}  // namespace sfa

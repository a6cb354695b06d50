// selftest.cu -- exercises the bounded-wait machinery on the device.
//
// One warp initialises an mbarrier that nothing ever arrives on and waits on
// it with the same bounded wait the GEMM roles use, but with a short limit.
// The wait expires, records DEV_TIMEOUT_SELFTEST in the context's status word
// and the kernel returns, so orda_context_check reports ORDA_ERR_TIMEOUT and
// the context stays usable. No fault, trap or unbounded spin is involved.
#include <cuda_runtime.h>

#include "../../include/orda.h"
#include "host_logic.h"
#include "ptx.cuh"

namespace orda {
namespace {

__global__ void bounded_wait_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  // phase 0 never completes: the bounded wait gives up after limit_ns
  mbar_wait(&bar, 0, status, DEV_TIMEOUT_SELFTEST, limit_ns);
}

}  // namespace

cudaError_t launch_bounded_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
  return cudaGetLastError();
}

}  // namespace orda

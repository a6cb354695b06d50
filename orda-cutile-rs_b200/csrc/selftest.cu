// selftest.cu -- device self-tests: the bounded-wait machinery, and the two
// exp2 implementations the kernels use (for accuracy tests against float64).
//
// One warp initialises an mbarrier that nothing ever arrives on and waits on
// it with the same bounded wait the GEMM roles use, but with a short limit.
// The wait expires, records DEV_TIMEOUT_SELFTEST in the context's status word
// and the kernel returns, so orda_context_check reports ORDA_ERR_TIMEOUT and
// the context stays usable. No fault, trap or unbounded spin is involved.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/orda.h"
#include "fastmath.cuh"
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

// y_fma[i] = exp2_fma(x[i]) (FMA pipe), y_sfu[i] = ex2.approx.ftz (SFU).
__global__ void exp2_selftest_kernel(const float* x, float* y_fma, float* y_sfu, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    float s;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(s) : "f"(v));
    y_fma[i] = exp2_fma(v);
    y_sfu[i] = s;
  }
}

}  // namespace

cudaError_t launch_bounded_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
  return cudaGetLastError();
}

}  // namespace orda

extern "C" int orda_selftest_exp2(const float* x, float* y_fma, float* y_sfu, size_t n, void* stream, char* err,
                                  size_t err_len) {
  if (!x || !y_fma || !y_sfu) {
    orda::set_error(err, err_len, "null argument");
    return ORDA_ERR_INVALID;
  }
  if (n == 0) return ORDA_OK;
  const long long blocks = std::min<long long>((static_cast<long long>(n) + 255) / 256, 148 * 8);
  orda::exp2_selftest_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y_fma, y_sfu, static_cast<long long>(n));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    orda::set_error(err, err_len, "CUDA error in the exp2 self-test: %s", cudaGetErrorString(e));
    return ORDA_ERR_CUDA;
  }
  return ORDA_OK;
}

// noalloc.cu -- the allocation-free variant of the INT8 grad_W quantiser.
//
// Some callers cannot call cudaMalloc: code that runs inside a host
// allocator hook or an out-of-memory handler, callers whose device memory is
// fully carved out by their own pool, and runtimes that forbid new device
// allocations after start-up. The regular quantiser entry keeps its scratch
// (one flag byte per vocabulary row marking the rows that are kept exact) in
// a context workspace obtained with cudaMalloc. This entry keeps that scratch
// in the file-scope device array below instead, so it allocates nothing; the
// caller still passes grad_W, the labels and the optional outputs.
//
// Limits and sharing rules:
//   * V (rows of grad_W) must be at most ORDA_NOALLOC_MAX_V; larger V is
//     rejected with an error. The array occupies ORDA_NOALLOC_MAX_V bytes
//     (256 KiB) on every GPU that loads this library, until the process exits.
//   * All calls on a device share the one array. Each call clears the part it
//     uses before use, but calls whose work overlaps on the GPU (different
//     streams without ordering between them) race on it: order them.
//   * Every call looks up the array's device address for the current device
//     with cudaGetSymbolAddress (cheap, allocates nothing), so the address is
//     never stale, also after cudaDeviceReset or a re-created primary
//     context. The first call on a device also makes CUDA load this
//     library's device code for that device: make that first call before any
//     CUDA stream capture.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/orda.h"
#include "host_logic.h"
#include "kernels.h"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_target_flags[ORDA_NOALLOC_MAX_V];

// The host-side name of the array is only a stand-in: kernels must receive
// the device address, which cudaGetSymbolAddress returns for the current
// device.
cudaError_t noalloc_scratch(uint8_t** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_target_flags);
  if (e != cudaSuccess) return e;
  *out = static_cast<uint8_t*>(p);
  return cudaSuccess;
}

}  // namespace

extern "C" int orda_quantize_grad_w_device_noalloc(float* grad_w, size_t v, size_t h, size_t ld, const int64_t* labels,
                                                   size_t bt, int64_t ignore_index, int stochastic, uint64_t seed,
                                                   int8_t* q, float* scale, void* stream, char* err, size_t err_len) {
  if (!grad_w || (bt > 0 && !labels) || ld < h) {
    orda::set_error(err, err_len, "invalid argument");
    return ORDA_ERR_INVALID;
  }
  if (v > ORDA_NOALLOC_MAX_V) {
    orda::set_error(err, err_len, "V=%zu exceeds the no-allocation limit of %d rows (ORDA_NOALLOC_MAX_V)", v,
                    ORDA_NOALLOC_MAX_V);
    return ORDA_ERR_INVALID;
  }
  uint8_t* flags = nullptr;
  cudaError_t e = noalloc_scratch(&flags);
  if (e != cudaSuccess) {
    orda::set_error(err, err_len, "CUDA error looking up the no-allocation scratch: %s", cudaGetErrorString(e));
    return ORDA_ERR_CUDA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's flags: clear the rows this call uses
  e = cudaMemsetAsync(flags, 0, v, st);
  if (e != cudaSuccess) {
    orda::set_error(err, err_len, "CUDA error clearing the no-allocation scratch: %s", cudaGetErrorString(e));
    return ORDA_ERR_CUDA;
  }
  orda::launch_target_flags(labels, static_cast<long long>(bt), static_cast<long long>(v), ignore_index, flags, st);
  orda::launch_quant(grad_w, static_cast<long long>(v), static_cast<long long>(h), static_cast<long long>(ld), flags,
                     stochastic, seed, q, scale, st);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    orda::set_error(err, err_len, "CUDA error in the quantiser: %s", cudaGetErrorString(e));
    return ORDA_ERR_CUDA;
  }
  return ORDA_OK;
}

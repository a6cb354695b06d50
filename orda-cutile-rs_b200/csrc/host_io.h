// Host-side data movement of the host-Mat entry (host_io.cc): the fp32 ->
// bf16 rounding of the GEMM operands before they cross PCIe, the lossless
// narrowing of teacher logits that are bf16 values already, the
// dequantisation of a compressed grad_W download, and the worker pool that
// runs them.
#pragma once
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace orda {

// dst[i] = bf16(src[i]) (f32_bits_to_bf16), i < n.
void f32_to_bf16_host(const float* src, size_t n, uint16_t* dst);

// When every src[i] is a bf16 value (its low 16 bits are zero), writes
// dst[i] = its high 16 bits and returns true; otherwise returns false (dst
// then holds unspecified values).
bool f32_to_bf16_if_exact(const float* src, size_t n, uint16_t* dst);

// Rows [r0, r1) of out (ld = h): exact_rows[exact_pos[r]] where
// exact_pos[r] >= 0, else q[r, :] * scale[r] (float multiply).
void dequant_rows_host(const int8_t* q, const float* scale, const int32_t* exact_pos, const float* exact_rows,
                       size_t r0, size_t r1, size_t h, float* out);

// n workers: n - 1 threads plus the caller of run(). run(fn) calls fn(w, n)
// on every worker w < n and returns when all have returned. One run() at a
// time.
class HostPool {
 public:
  explicit HostPool(unsigned n);
  ~HostPool();
  HostPool(const HostPool&) = delete;
  HostPool& operator=(const HostPool&) = delete;
  unsigned size() const { return n_; }
  void run(const std::function<void(unsigned, unsigned)>& fn);

 private:
  void loop(unsigned w);
  unsigned n_;
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(unsigned, unsigned)>* fn_ = nullptr;
  uint64_t gen_ = 0;
  unsigned pending_ = 0;
  bool stop_ = false;
};

// Splits [0, n) into `parts` nearly equal pieces; piece w is [*a, *b).
inline void split_range(size_t n, unsigned parts, unsigned w, size_t* a, size_t* b) {
  const size_t per = n / parts, extra = n % parts;
  *a = w * per + (w < extra ? w : extra);
  *b = *a + per + (w < extra ? 1 : 0);
}

}  // namespace orda

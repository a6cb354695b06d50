// Host-side data movement of the host-Mat entry (declarations in host_io.h).
//
// PCIe, not the GPU, bounds the host-Mat call: at c4 it moves 6.58 GB of
// fp32 inputs and 2.28 GB of fp32 gradients at about 55 GB/s per direction.
// Three host passes, spread over the cores, cut those bytes without changing
// a bit of the result:
//  * the GEMM operands (hidden states, weights) are rounded to bf16 here with
//    the device's own rounding (bf16_bits.h) instead of after the copy;
//  * fp32 teacher logits that hold bf16 values (the logits of a bf16 teacher
//    model, upcast) cross as their high halves and are widened back on the
//    device, exactly; any other chunk crosses as fp32;
//  * with the INT8 round trip (src/api.rs:391-399, src/quant.rs:157-202)
//    grad_W comes back as its codes, row scales and exact target rows, and
//    the dequantised value q * s is formed here with the device's single IEEE
//    float multiply.
// Built by the host compiler (not nvcc). The loops have AVX-512 and AVX2
// versions chosen at run time and write with non-temporal stores, so the
// outputs cost one pass of memory writes.
#include "host_io.h"

#include <immintrin.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/orda.h"
#include "bf16_bits.h"

namespace orda {
namespace {

// ---------------------------------------------------------------- bf16

void to_bf16_scalar(const float* src, size_t n, uint16_t* dst) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t b;
    std::memcpy(&b, src + i, 4);
    dst[i] = f32_bits_to_bf16(b);
  }
}

bool exact_scalar(const float* src, size_t n, uint16_t* dst) {
  uint32_t low = 0;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b;
    std::memcpy(&b, src + i, 4);
    low |= b & 0xFFFFu;
    dst[i] = static_cast<uint16_t>(b >> 16);
  }
  return low == 0;
}

// elements before dst reaches an `align`-byte boundary (at most n)
size_t head_to_align(const uint16_t* dst, size_t n, size_t align) {
  const size_t mis = reinterpret_cast<uintptr_t>(dst) & (align - 1);
  if (mis & 1) return n;  // odd address: no vector path
  const size_t k = mis ? (align - mis) / 2 : 0;
  return k < n ? k : n;
}

__attribute__((target("avx512f"))) __m256i bf16x16_avx512(__m512i b) {
  const __m512i abs = _mm512_and_si512(b, _mm512_set1_epi32(0x7FFFFFFF));
  const __mmask16 nan = _mm512_cmpgt_epi32_mask(abs, _mm512_set1_epi32(0x7F800000));
  const __m512i hi = _mm512_srli_epi32(b, 16);
  const __m512i odd = _mm512_and_si512(hi, _mm512_set1_epi32(1));
  __m512i r = _mm512_srli_epi32(_mm512_add_epi32(b, _mm512_add_epi32(_mm512_set1_epi32(0x7FFF), odd)), 16);
  r = _mm512_mask_or_epi32(r, nan, hi, _mm512_set1_epi32(0x40));
  return _mm512_cvtepi32_epi16(r);
}

__attribute__((target("avx512f"))) void to_bf16_avx512(const float* src, size_t n, uint16_t* dst) {
  size_t i = head_to_align(dst, n, 32);
  to_bf16_scalar(src, i, dst);
  for (; i + 16 <= n; i += 16)
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), bf16x16_avx512(_mm512_loadu_si512(src + i)));
  to_bf16_scalar(src + i, n - i, dst + i);
}

__attribute__((target("avx512f"))) bool exact_avx512(const float* src, size_t n, uint16_t* dst) {
  size_t i = head_to_align(dst, n, 32);
  bool ok = exact_scalar(src, i, dst);
  __m512i low = _mm512_setzero_si512();
  const __m512i mask = _mm512_set1_epi32(0xFFFF);
  for (; i + 16 <= n; i += 16) {
    const __m512i b = _mm512_loadu_si512(src + i);
    low = _mm512_or_si512(low, _mm512_and_si512(b, mask));
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), _mm512_cvtepi32_epi16(_mm512_srli_epi32(b, 16)));
  }
  ok = exact_scalar(src + i, n - i, dst + i) && ok;
  return ok && _mm512_test_epi32_mask(low, low) == 0;
}

__attribute__((target("avx2"))) __m256i pack16_avx2(__m256i a, __m256i b) {
  // 8 + 8 values < 2^16 -> 16 uint16 in order
  return _mm256_permute4x64_epi64(_mm256_packus_epi32(a, b), 0xD8);
}

__attribute__((target("avx2"))) __m256i round8_avx2(__m256i b) {
  const __m256i abs = _mm256_and_si256(b, _mm256_set1_epi32(0x7FFFFFFF));
  const __m256i nan = _mm256_cmpgt_epi32(abs, _mm256_set1_epi32(0x7F800000));
  const __m256i hi = _mm256_srli_epi32(b, 16);
  const __m256i odd = _mm256_and_si256(hi, _mm256_set1_epi32(1));
  const __m256i r = _mm256_srli_epi32(_mm256_add_epi32(b, _mm256_add_epi32(_mm256_set1_epi32(0x7FFF), odd)), 16);
  return _mm256_blendv_epi8(r, _mm256_or_si256(hi, _mm256_set1_epi32(0x40)), nan);
}

__attribute__((target("avx2"))) void to_bf16_avx2(const float* src, size_t n, uint16_t* dst) {
  size_t i = head_to_align(dst, n, 32);
  to_bf16_scalar(src, i, dst);
  for (; i + 16 <= n; i += 16) {
    const __m256i a = round8_avx2(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i)));
    const __m256i b = round8_avx2(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 8)));
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i), pack16_avx2(a, b));
  }
  to_bf16_scalar(src + i, n - i, dst + i);
}

__attribute__((target("avx2"))) bool exact_avx2(const float* src, size_t n, uint16_t* dst) {
  size_t i = head_to_align(dst, n, 32);
  bool ok = exact_scalar(src, i, dst);
  __m256i low = _mm256_setzero_si256();
  const __m256i mask = _mm256_set1_epi32(0xFFFF);
  for (; i + 16 <= n; i += 16) {
    const __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i));
    const __m256i b = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(src + i + 8));
    low = _mm256_or_si256(low, _mm256_and_si256(_mm256_or_si256(a, b), mask));
    _mm256_stream_si256(reinterpret_cast<__m256i*>(dst + i),
                        pack16_avx2(_mm256_srli_epi32(a, 16), _mm256_srli_epi32(b, 16)));
  }
  ok = exact_scalar(src + i, n - i, dst + i) && ok;
  return ok && _mm256_testz_si256(low, low);
}

// ------------------------------------------------------------ dequant

void row_scalar(const int8_t* q, float s, size_t n, float* out) {
  for (size_t c = 0; c < n; ++c) out[c] = static_cast<float>(q[c]) * s;
}

__attribute__((target("avx2"))) void row_avx2(const int8_t* q, float s, size_t h, float* out) {
  size_t c = 0;
  while (c < h && (reinterpret_cast<uintptr_t>(out + c) & 31) != 0) {
    out[c] = static_cast<float>(q[c]) * s;
    ++c;
  }
  const __m256 vs = _mm256_set1_ps(s);
  for (; c + 8 <= h; c += 8) {
    const __m128i b = _mm_loadl_epi64(reinterpret_cast<const __m128i*>(q + c));
    const __m256 f = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b));
    _mm256_stream_ps(out + c, _mm256_mul_ps(f, vs));
  }
  row_scalar(q + c, s, h - c, out + c);
}

__attribute__((target("avx512f"))) void row_avx512(const int8_t* q, float s, size_t h, float* out) {
  size_t c = 0;
  while (c < h && (reinterpret_cast<uintptr_t>(out + c) & 63) != 0) {
    out[c] = static_cast<float>(q[c]) * s;
    ++c;
  }
  const __m512 vs = _mm512_set1_ps(s);
  for (; c + 16 <= h; c += 16) {
    const __m128i b = _mm_loadu_si128(reinterpret_cast<const __m128i*>(q + c));
    const __m512 f = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(b));
    _mm512_stream_ps(out + c, _mm512_mul_ps(f, vs));
  }
  row_scalar(q + c, s, h - c, out + c);
}

enum class Isa { kScalar, kAvx2, kAvx512 };

Isa pick_isa() {
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return Isa::kAvx512;
  if (__builtin_cpu_supports("avx2")) return Isa::kAvx2;
  return Isa::kScalar;
}

Isa isa() {
  static const Isa k = pick_isa();
  return k;
}

}  // namespace

namespace {

void to_bf16_isa(Isa k, const float* src, size_t n, uint16_t* dst) {
  switch (k) {
    case Isa::kAvx512: to_bf16_avx512(src, n, dst); break;
    case Isa::kAvx2: to_bf16_avx2(src, n, dst); break;
    default: to_bf16_scalar(src, n, dst);
  }
  _mm_sfence();  // the non-temporal stores are visible before the copy reads them
}

bool exact_isa(Isa k, const float* src, size_t n, uint16_t* dst) {
  bool ok;
  switch (k) {
    case Isa::kAvx512: ok = exact_avx512(src, n, dst); break;
    case Isa::kAvx2: ok = exact_avx2(src, n, dst); break;
    default: ok = exact_scalar(src, n, dst);
  }
  _mm_sfence();
  return ok;
}

void dequant_isa(Isa k, const int8_t* q, const float* scale, const int32_t* exact_pos, const float* exact_rows,
                 size_t r0, size_t r1, size_t h, float* out) {
  for (size_t r = r0; r < r1; ++r) {
    float* o = out + r * h;
    const int32_t e = exact_pos[r];
    if (e >= 0) std::memcpy(o, exact_rows + static_cast<size_t>(e) * h, h * sizeof(float));
    else if (k == Isa::kAvx512) row_avx512(q + r * h, scale[r], h, o);
    else if (k == Isa::kAvx2) row_avx2(q + r * h, scale[r], h, o);
    else row_scalar(q + r * h, scale[r], h, o);
  }
  _mm_sfence();
}

}  // namespace

void f32_to_bf16_host(const float* src, size_t n, uint16_t* dst) { to_bf16_isa(isa(), src, n, dst); }

bool f32_to_bf16_if_exact(const float* src, size_t n, uint16_t* dst) { return exact_isa(isa(), src, n, dst); }

void dequant_rows_host(const int8_t* q, const float* scale, const int32_t* exact_pos, const float* exact_rows,
                       size_t r0, size_t r1, size_t h, float* out) {
  dequant_isa(isa(), q, scale, exact_pos, exact_rows, r0, r1, h, out);
}

// ------------------------------------------------------------ self-test

namespace {

uint32_t lcg(uint64_t* st) {
  *st = *st * 6364136223846793005ull + 1442695040888963407ull;
  return static_cast<uint32_t>(*st >> 32);
}

float from_bits(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

const char* isa_name(Isa k) { return k == Isa::kAvx512 ? "avx512" : k == Isa::kAvx2 ? "avx2" : "scalar"; }

// Empty string when every check of ISA k agrees with the scalar definitions.
std::string check_isa(Isa k) {
  uint64_t st = 12345;
  // fp32 -> bf16: special bit patterns, then random ones
  std::vector<uint32_t> bits = {0x00000000u, 0x80000000u, 0x3F800000u, 0x3F808000u, 0x3F818000u, 0x3F807FFFu,
                                0x3F808001u, 0x7F7FFFFFu, 0x7F7F7FFFu, 0xFF7FFFFFu, 0x7F800000u, 0xFF800000u,
                                0x7FC00000u, 0x7F800001u, 0xFFC00001u, 0x7FFFFFFFu, 0x00000001u, 0x00008000u,
                                0x00018000u, 0x807F8000u, 0x00800000u, 0x3F80FFFFu};
  for (int i = 0; i < 70000; ++i) bits.push_back(lcg(&st));
  std::vector<float> src(bits.size());
  for (size_t i = 0; i < bits.size(); ++i) src[i] = from_bits(bits[i]);
  for (size_t off : {size_t{0}, size_t{1}, size_t{3}}) {
    for (size_t n : {bits.size() - off, size_t{33}, size_t{7}}) {
      std::vector<uint16_t> out(n + 8, 0xABCD);
      to_bf16_isa(k, src.data() + off, n, out.data() + off % 2);
      for (size_t i = 0; i < n; ++i)
        if (out[off % 2 + i] != f32_bits_to_bf16(bits[off + i])) return "f32->bf16 rounding differs";
    }
  }
  // exactness: bf16 values pass, one low bit anywhere fails
  std::vector<float> ex(1000);
  for (size_t i = 0; i < ex.size(); ++i) ex[i] = from_bits(lcg(&st) & 0xFFFF0000u);
  std::vector<uint16_t> hi(ex.size() + 8);
  for (size_t off : {size_t{0}, size_t{1}}) {
    if (!exact_isa(k, ex.data(), ex.size(), hi.data() + off)) return "bf16 values reported inexact";
    for (size_t i = 0; i < ex.size(); ++i) {
      uint32_t b;
      std::memcpy(&b, &ex[i], 4);
      if (hi[off + i] != static_cast<uint16_t>(b >> 16)) return "exact narrowing differs";
    }
    for (size_t pos : {size_t{0}, size_t{5}, size_t{500}, ex.size() - 1}) {
      std::vector<float> bad(ex);
      uint32_t b;
      std::memcpy(&b, &bad[pos], 4);
      bad[pos] = from_bits(b | 0x1u);
      if (exact_isa(k, bad.data(), bad.size(), hi.data() + off)) return "inexact value not detected";
    }
  }
  // dequantisation: q * s, exact rows copied, odd widths, misaligned output
  for (size_t h : {size_t{256}, size_t{250}, size_t{17}}) {
    const size_t rows = 40;
    std::vector<int8_t> q(rows * h);
    for (auto& x : q) x = static_cast<int8_t>(static_cast<int>(lcg(&st) % 255u) - 127);
    std::vector<float> s(rows), xr;
    std::vector<int32_t> pos(rows, -1);
    for (size_t r = 0; r < rows; ++r) s[r] = std::ldexp(1.0f + static_cast<float>(lcg(&st) % 1000u) / 999.0f,
                                                        -static_cast<int>(lcg(&st) % 60u));
    for (size_t r = 0; r < rows; r += 7) {
      pos[r] = static_cast<int32_t>(xr.size() / h);
      for (size_t c = 0; c < h; ++c) xr.push_back(from_bits(lcg(&st) & 0xBFFFFFFFu));
    }
    std::vector<float> out(rows * h + 16);
    float* o = out.data() + 1;
    dequant_isa(k, q.data(), s.data(), pos.data(), xr.data(), 0, rows, h, o);
    for (size_t r = 0; r < rows; ++r)
      for (size_t c = 0; c < h; ++c) {
        const float want = pos[r] >= 0 ? xr[static_cast<size_t>(pos[r]) * h + c] : static_cast<float>(q[r * h + c]) * s[r];
        if (std::memcmp(&want, &o[r * h + c], 4) != 0) return "dequantisation differs";
      }
  }
  return std::string();
}

}  // namespace

// ------------------------------------------------------------- pool

HostPool::HostPool(unsigned n) : n_(n ? n : 1) {
  try {
    for (unsigned w = 1; w < n_; ++w) threads_.emplace_back([this, w] { loop(w); });
  } catch (...) {
    // a thread could not be started: stop the ones that were, then report
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : threads_) t.join();
    throw;
  }
}

HostPool::~HostPool() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : threads_) t.join();
}

void HostPool::run(const std::function<void(unsigned, unsigned)>& fn) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    fn_ = &fn;
    pending_ = n_ - 1;
    ++gen_;
  }
  cv_.notify_all();
  fn(0, n_);
  std::unique_lock<std::mutex> lk(mu_);
  done_cv_.wait(lk, [this] { return pending_ == 0; });
  fn_ = nullptr;
}

void HostPool::loop(unsigned w) {
  uint64_t seen = 0;
  for (;;) {
    const std::function<void(unsigned, unsigned)>* f;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      f = fn_;
    }
    (*f)(w, n_);
    std::lock_guard<std::mutex> lk(mu_);
    if (--pending_ == 0) done_cv_.notify_one();
  }
}

}  // namespace orda

extern "C" ORDA_API int orda_selftest_host_io(char* err, size_t err_len) {
  using namespace orda;
  std::vector<Isa> isas = {Isa::kScalar};
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx2")) isas.push_back(Isa::kAvx2);
  if (__builtin_cpu_supports("avx512f")) isas.push_back(Isa::kAvx512);
  std::string names;
  for (Isa k : isas) {
    const std::string why = check_isa(k);
    if (!why.empty()) {
      if (err && err_len) std::snprintf(err, err_len, "%s: %s", isa_name(k), why.c_str());
      return ORDA_ERR_BACKEND;
    }
    names += (names.empty() ? "" : ",") + std::string(isa_name(k));
  }
  if (err && err_len) std::snprintf(err, err_len, "checked: %s", names.c_str());
  return ORDA_OK;
}

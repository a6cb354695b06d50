// quant.cu -- fused INT8 row-wise grad_W quantisation (absmax + quantise +
// dequantise in one kernel), bit-exact with src/quant.rs:
//   s = max(amax, 1e-12) / 127            (IEEE f32 divide, row_scale :91-94)
//   q = clamp(rne(x / s), -127, 127)      (IEEE divide; rne = round half even,
//                                          round_half_even :48-63)
//   stochastic: q = clamp(floor(x/s) + [frac > u_k], -127, 127) with u_k the
//   k-th draw (k = r*H + c, row-major) of the SplitMix64 stream :18-44,120-144;
//   draw k is computed directly from its index, so rows run in parallel.
//   dequantised = q * s, target rows (labels) restored exactly (:157-202).
// This file is compiled without fast-math, so '/' is the correctly rounded
// divide; __fdiv_rn makes that explicit.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace orda {

namespace {

constexpr int QT = 256;

__device__ __forceinline__ int8_t to_i8(float v) {
  if (isnan(v)) return 0;  // Rust `as i8` maps NaN to 0
  v = fminf(fmaxf(v, -127.0f), 127.0f);
  return static_cast<int8_t>(v);
}

// u_k of the reference's SplitMix64 Rng::new(seed): the k-th call sees
// state = seed + (k + 2) * golden (wrapping).
__device__ __forceinline__ float splitmix_uniform(uint64_t seed, uint64_t k) {
  const uint64_t golden = 0x9E3779B97F4A7C15ull;
  uint64_t z = seed + (k + 2) * golden;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(QT) quant_kernel(float* grad_w, long long h, long long ld,
                                                   const uint8_t* target_flags, int stochastic, uint64_t seed,
                                                   int8_t* q, float* scale, long long row_offset) {
  __shared__ float sh[QT / 32];
  const long long r = blockIdx.x;
  float* row = grad_w + r * ld;

  float amax = 0.0f;
  const bool vec = (h % 4 == 0) && (ld % 4 == 0);
  if (vec) {
    for (long long c = threadIdx.x * 4; c < h; c += QT * 4) {
      const float4 x = *reinterpret_cast<const float4*>(row + c);
      amax = fmaxf(amax, fabsf(x.x));
      amax = fmaxf(amax, fabsf(x.y));
      amax = fmaxf(amax, fabsf(x.z));
      amax = fmaxf(amax, fabsf(x.w));
    }
  } else {
    for (long long c = threadIdx.x; c < h; c += QT) amax = fmaxf(amax, fabsf(row[c]));
  }
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = sh[0];
#pragma unroll
  for (int w = 1; w < QT / 32; ++w) amax = fmaxf(amax, sh[w]);

  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 127.0f);
  if (scale && threadIdx.x == 0) scale[r] = s;
  const bool keep = target_flags && target_flags[r];
  int8_t* qrow = q ? q + r * h : nullptr;

  for (long long c = threadIdx.x; c < h; c += QT) {
    const float x = row[c];
    const float scaled = __fdiv_rn(x, s);
    int8_t qi;
    if (!stochastic) {
      qi = to_i8(rintf(scaled));
    } else {
      const float fl = floorf(scaled);
      const float frac = scaled - fl;
      const float u = splitmix_uniform(seed, static_cast<uint64_t>(r + row_offset) * static_cast<uint64_t>(h) +
                                                 static_cast<uint64_t>(c));
      qi = to_i8(fl + (frac > u ? 1.0f : 0.0f));
    }
    if (qrow) qrow[c] = qi;
    if (!keep) row[c] = static_cast<float>(qi) * s;
  }
}

// Sum of the world partial slices of a slot buffer, in rank order (the
// fixed order makes the reduced grad_W independent of arrival order).
// One CTA per row, 128-bit accesses when the row allows them.
__global__ void __launch_bounds__(QT) slot_reduce_kernel(const float* __restrict__ slots, int world,
                                                         long long slice, long long h, float* out, long long ld) {
  const long long r = blockIdx.x;
  const long long part = slice * h;
  float* orow = out + r * ld;
  const float* srow = slots + r * h;
  if (h % 4 == 0 && ld % 4 == 0) {
    for (long long c = threadIdx.x * 4; c < h; c += QT * 4) {
      float4 acc = *reinterpret_cast<const float4*>(srow + c);
      for (int k = 1; k < world; ++k) {
        const float4 x = *reinterpret_cast<const float4*>(srow + k * part + c);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      *reinterpret_cast<float4*>(orow + c) = acc;
    }
  } else {
    for (long long c = threadIdx.x; c < h; c += QT) {
      float acc = srow[c];
      for (int k = 1; k < world; ++k) acc += srow[k * part + c];
      orow[c] = acc;
    }
  }
}

// Rank-ordered sum of the world partials of one row fused with its INT8
// round trip: the summed row is kept in shared memory (h floats), so the
// slice is read once (the partials) and written once, and the values equal
// slot_reduce_kernel followed by quant_kernel bit for bit.
__global__ void __launch_bounds__(QT) slot_reduce_quant_kernel(const float* __restrict__ slots, int world,
                                                               long long slice, long long h, float* out,
                                                               long long ld, const uint8_t* target_flags,
                                                               int stochastic, uint64_t seed, int8_t* q,
                                                               float* scale, long long row_offset) {
  extern __shared__ __align__(16) float xs[];  // h floats
  __shared__ float sh[QT / 32];
  const long long r = blockIdx.x;
  const long long part = slice * h;
  const float* srow = slots + r * h;
  float amax = 0.0f;
  for (long long c = threadIdx.x * 4; c < h; c += QT * 4) {
    float4 acc = *reinterpret_cast<const float4*>(srow + c);
    for (int k = 1; k < world; ++k) {
      const float4 x = *reinterpret_cast<const float4*>(srow + k * part + c);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    *reinterpret_cast<float4*>(xs + c) = acc;
    amax = fmaxf(fmaxf(amax, fabsf(acc.x)), fmaxf(fabsf(acc.y), fmaxf(fabsf(acc.z), fabsf(acc.w))));
  }
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = sh[0];
#pragma unroll
  for (int w = 1; w < QT / 32; ++w) amax = fmaxf(amax, sh[w]);

  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 127.0f);
  if (scale && threadIdx.x == 0) scale[r] = s;
  const bool keep = target_flags && target_flags[r];
  int8_t* qrow = q ? q + r * h : nullptr;
  float* orow = out + r * ld;
  for (long long c = threadIdx.x; c < h; c += QT) {
    const float x = xs[c];
    const float scaled = __fdiv_rn(x, s);
    int8_t qi;
    if (!stochastic) {
      qi = to_i8(rintf(scaled));
    } else {
      const float fl = floorf(scaled);
      const float frac = scaled - fl;
      const float u = splitmix_uniform(seed, static_cast<uint64_t>(r + row_offset) * static_cast<uint64_t>(h) +
                                                 static_cast<uint64_t>(c));
      qi = to_i8(fl + (frac > u ? 1.0f : 0.0f));
    }
    if (qrow) qrow[c] = qi;
    orow[c] = keep ? x : static_cast<float>(qi) * s;
  }
}

// Absmax of one row (block reduction; every thread gets the result). vec:
// the row starts 16-byte aligned and h % 4 == 0 (float4 loads).
__device__ __forceinline__ float row_absmax(const float* row, long long h, bool vec, float* sh) {
  float amax = 0.0f;
  if (vec) {
    for (long long c = threadIdx.x * 4; c < h; c += QT * 4) {
      const float4 x = *reinterpret_cast<const float4*>(row + c);
      amax = fmaxf(fmaxf(amax, fabsf(x.x)), fmaxf(fabsf(x.y), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
  } else {
    for (long long c = threadIdx.x; c < h; c += QT) amax = fmaxf(amax, fabsf(row[c]));
  }
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = sh[0];
#pragma unroll
  for (int w = 1; w < QT / 32; ++w) amax = fmaxf(amax, sh[w]);
  return amax;
}

// INT8 wire format of the row-sharded grad_W exchange: row r of this rank's
// local fp32 partial goes to its owner o = r / slice as one INT8 row with one
// fp32 scale, by the row-wise rules of quantize_rowwise_int8 (src/quant.rs:
// 97-117: s = max(amax, 1e-12) / 127, q = clamp(rne(x / s), +-127)). The
// owner's buffer holds [world][slice][h] codes and [world][slice] scales;
// this rank writes partial index slot_rank (plain stores, over NVLink for
// other owners), 16 codes per store when h allows.
__global__ void __launch_bounds__(QT) quant_send_kernel(const float* __restrict__ gw, long long h, long long ld,
                                                        long long slice, int slot_rank, int world, WireSlots dst) {
  __shared__ float sh[QT / 32];
  const long long r = blockIdx.x;
  const float* row = gw + r * ld;
  const bool vec = h % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(gw) & 15) == 0;
  const float s = __fdiv_rn(fmaxf(row_absmax(row, h, vec, sh), 1e-12f), 127.0f);
  const long long o = r / slice;
  const long long lr = r - o * slice;
  int8_t* qrow = dst.codes[o] + (static_cast<long long>(slot_rank) * slice + lr) * h;
  if (threadIdx.x == 0) dst.scales[o][static_cast<long long>(slot_rank) * slice + lr] = s;
  if (vec && h % 16 == 0 && (reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {
    for (long long c = threadIdx.x * 16; c < h; c += QT * 16) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 x = *reinterpret_cast<const float4*>(row + c + 4 * k);
        const uint32_t b0 = static_cast<uint8_t>(to_i8(rintf(__fdiv_rn(x.x, s))));
        const uint32_t b1 = static_cast<uint8_t>(to_i8(rintf(__fdiv_rn(x.y, s))));
        const uint32_t b2 = static_cast<uint8_t>(to_i8(rintf(__fdiv_rn(x.z, s))));
        const uint32_t b3 = static_cast<uint8_t>(to_i8(rintf(__fdiv_rn(x.w, s))));
        w[k] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
      }
      *reinterpret_cast<uint4*>(qrow + c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    for (long long c = threadIdx.x; c < h; c += QT) qrow[c] = to_i8(rintf(__fdiv_rn(row[c], s)));
  }
  __threadfence_system();
}

// Owner side of the INT8 wire: row r of this rank's slice is the sum, in rank
// order, of the world dequantised partials q_k * s_k (fp32), kept in shared
// memory and written out, or (quantize) given the INT8 round trip of
// quant_kernel in the same pass.
__global__ void __launch_bounds__(QT) wire_reduce_kernel(WireSlots mine, int world, long long slice, long long h,
                                                         float* out, long long ld, const uint8_t* target_flags,
                                                         int quantize, int stochastic, uint64_t seed, int8_t* q,
                                                         float* scale, long long row_offset) {
  extern __shared__ __align__(16) float xs[];  // h floats
  __shared__ float sh[QT / 32];
  const long long r = blockIdx.x;
  const int8_t* codes = mine.codes[0];
  const float* scales = mine.scales[0];
  for (long long c = threadIdx.x; c < h; c += QT) {
    float acc = 0.0f;
    for (int k = 0; k < world; ++k) {
      const long long pr = static_cast<long long>(k) * slice + r;
      acc += static_cast<float>(codes[pr * h + c]) * scales[pr];
    }
    xs[c] = acc;
  }
  __syncthreads();
  float* orow = out + r * ld;
  if (!quantize) {
    for (long long c = threadIdx.x; c < h; c += QT) orow[c] = xs[c];
    return;
  }
  const float s = __fdiv_rn(fmaxf(row_absmax(xs, h, h % 4 == 0, sh), 1e-12f), 127.0f);
  if (scale && threadIdx.x == 0) scale[r] = s;
  const bool keep = target_flags && target_flags[r];
  int8_t* qrow = q ? q + r * h : nullptr;
  for (long long c = threadIdx.x; c < h; c += QT) {
    const float x = xs[c];
    const float scaled = __fdiv_rn(x, s);
    int8_t qi;
    if (!stochastic) {
      qi = to_i8(rintf(scaled));
    } else {
      const float fl = floorf(scaled);
      const float frac = scaled - fl;
      const float u = splitmix_uniform(seed, static_cast<uint64_t>(r + row_offset) * static_cast<uint64_t>(h) +
                                                 static_cast<uint64_t>(c));
      qi = to_i8(fl + (frac > u ? 1.0f : 0.0f));
    }
    if (qrow) qrow[c] = qi;
    orow[c] = keep ? x : static_cast<float>(qi) * s;
  }
}

}  // namespace

bool launch_slot_reduce_quant(const float* slots, int world, long long slice, long long rows, long long h, float* out,
                              long long ld, const uint8_t* target_flags, int stochastic, uint64_t seed, int8_t* q,
                              float* scale, long long row_offset, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(h) * sizeof(float);
  if (h % 4 != 0 || smem > 48 * 1024) return false;
  if (rows <= 0) return true;
  slot_reduce_quant_kernel<<<static_cast<unsigned>(rows), QT, smem, stream>>>(
      slots, world, slice, h, out, ld, target_flags, stochastic, seed, q, scale, row_offset);
  return true;
}

// Copies rows idx[0..n) of src (ld elements apart) into the dense [n, h]
// dst: the exact target rows of grad_W for the host-Mat entry's compressed
// download. One CTA per row.
__global__ void __launch_bounds__(QT) gather_rows_kernel(const float* __restrict__ src, long long ld,
                                                         const int32_t* __restrict__ idx, long long h,
                                                         float* __restrict__ dst) {
  const long long i = blockIdx.x;
  const float* srow = src + static_cast<long long>(idx[i]) * ld;
  float* drow = dst + i * h;
  if (h % 4 == 0 && ld % 4 == 0) {
    for (long long c = threadIdx.x * 4; c < h; c += QT * 4)
      *reinterpret_cast<float4*>(drow + c) = *reinterpret_cast<const float4*>(srow + c);
  } else {
    for (long long c = threadIdx.x; c < h; c += QT) drow[c] = srow[c];
  }
}

void launch_gather_rows(const float* src, long long ld, const int32_t* idx, long long n, long long h, float* dst,
                        cudaStream_t stream) {
  if (n <= 0) return;
  gather_rows_kernel<<<static_cast<unsigned>(n), QT, 0, stream>>>(src, ld, idx, h, dst);
}

void launch_quant(float* grad_w, long long v, long long h, long long ld, const uint8_t* target_flags,
                  int stochastic, uint64_t seed, int8_t* q, float* scale, cudaStream_t stream,
                  long long row_offset) {
  if (v <= 0 || h <= 0) return;
  quant_kernel<<<static_cast<unsigned>(v), QT, 0, stream>>>(grad_w, h, ld, target_flags, stochastic, seed, q, scale,
                                                            row_offset);
}

void launch_slot_reduce(const float* slots, int world, long long slice, long long rows, long long h, float* out,
                        long long ld, cudaStream_t stream) {
  if (rows <= 0 || h <= 0) return;
  slot_reduce_kernel<<<static_cast<unsigned>(rows), QT, 0, stream>>>(slots, world, slice, h, out, ld);
}

void launch_quant_send(const float* grad_w, long long v, long long h, long long ld, long long slice, int slot_rank,
                       int world, const WireSlots& dst, cudaStream_t stream) {
  if (v <= 0 || h <= 0) return;
  quant_send_kernel<<<static_cast<unsigned>(v), QT, 0, stream>>>(grad_w, h, ld, slice, slot_rank, world, dst);
}

bool launch_wire_reduce(const WireSlots& mine, int world, long long slice, long long rows, long long h, float* out,
                        long long ld, const uint8_t* target_flags, int quantize, int stochastic, uint64_t seed,
                        int8_t* q, float* scale, long long row_offset, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(h) * sizeof(float);
  if (smem > 48 * 1024) return false;
  if (rows <= 0) return true;
  wire_reduce_kernel<<<static_cast<unsigned>(rows), QT, smem, stream>>>(mine, world, slice, h, out, ld, target_flags,
                                                                         quantize, stochastic, seed, q, scale,
                                                                         row_offset);
  return true;
}

}  // namespace orda

// fp32 -> bf16 rounding shared by the device conversion kernel and the host
// conversion of the host-Mat entry, so both give the same bits: round to
// nearest, ties to even, on the bit pattern (correct for normals, subnormals
// and overflow to infinity); a NaN stays a NaN (quiet bit set, sign and the
// top payload bits kept).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define ORDA_HD __host__ __device__ __forceinline__
#else
#define ORDA_HD inline
#endif

namespace orda {

ORDA_HD uint16_t f32_bits_to_bf16(uint32_t b) {
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((b >> 16) | 0x0040u);
  return static_cast<uint16_t>((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}

}  // namespace orda

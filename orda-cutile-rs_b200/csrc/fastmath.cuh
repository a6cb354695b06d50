// fastmath.cuh -- 2^x on the FMA pipe, for the Fast profile.
//
// The SFU (MUFU ex2) delivers 16 results per SM cycle for one issue slot
// each; exp2_fma computes 2^x with about ten FMA-pipe instructions, i.e. ten
// issue slots (128 thread-instructions per SM cycle). Moving exp2 work to it
// pays only where the SFU bounds a loop and issue slots are spare: in the
// logits GEMM epilogue (two exp2 and about eight other instructions per
// element) a quarter of one sum goes to it under the Fast profile; the row
// kernels, already balanced between SFU and issue, measured 23 % slower with
// half their exp2 moved, and keep the SFU.
//
// Method (Cody and Waite's argument reduction, "Software Manual for the
// Elementary Functions", 1980): x = n + f with n = rint(x), f = x - n in
// [-1/2, 1/2] exactly; 2^x = 2^n * 2^f. n is obtained with the 1.5 * 2^23
// rounding constant (two FADDs), 2^f by a degree-6 polynomial in Horner form
// (six FMAs), and 2^n by adding n to the exponent field of the result. The
// coefficients minimise the relative error of the polynomial against 2^f in
// the least-squares sense on 4000 Chebyshev nodes of [-1/2, 1/2] (fitted for
// this library; tests/test_exp2_poly.py refits them and checks these values).
// Approximation error below 2e-9 relative; with fp32 rounding the result is
// within about 1 ulp (tests/test_parity_gpu.py measures it against float64
// on the GPU, next to the SFU's ex2.approx).
//
// Range: arguments are clamped to [-125, 126]; results for x < -125 are
// 2^-125 instead of smaller values (callers only add them to sums of terms
// near 1 or use them where such values are negligible).
#pragma once

namespace orda {

constexpr float kExp2C0 = 1.0f;
constexpr float kExp2C1 = 0.6931471824645996f;
constexpr float kExp2C2 = 0.24022646248340607f;
constexpr float kExp2C3 = 0.05550329014658928f;
constexpr float kExp2C4 = 0.009618519805371761f;
constexpr float kExp2C5 = 0.0013399859890341759f;
constexpr float kExp2C6 = 0.00015337577497120947f;

__device__ __forceinline__ float exp2_fma(float x) {
  x = fminf(fmaxf(x, -125.0f), 126.0f);
  const float t = x + 12582912.0f;  // 1.5 * 2^23: t's low mantissa bits hold rint(x)
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - 12582912.0f);  // exact
  float p = kExp2C6;
  p = fmaf(p, f, kExp2C5);
  p = fmaf(p, f, kExp2C4);
  p = fmaf(p, f, kExp2C3);
  p = fmaf(p, f, kExp2C2);
  p = fmaf(p, f, kExp2C1);
  p = fmaf(p, f, kExp2C0);
  return __int_as_float(__float_as_int(p) + (n << 23));
}

}  // namespace orda

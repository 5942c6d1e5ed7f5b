// 2^x on the FMA pipe, used to take part of the softmax exponentials off the
// transcendental (MUFU/XU) unit, which for head_dim 128 has exactly the throughput
// of the tensor cores and would otherwise bound flash attention.
//
// Method: Cody-Waite style range reduction x = n + f with n = round(x) obtained by
// adding the magic constant 1.5*2^23 (so |f| <= 1/2), a degree-3 minimax (Remez,
// relative error) polynomial for 2^f on [-1/2, 1/2], and scaling by 2^n through an
// integer add into the exponent field.  The coefficients were fitted for this
// library (max relative error 7.5e-5, tested against CUDA's exp2f in
// tests/test_kernels_gpu.py::test_exp2_poly); inputs below -126 return ~2^-126.
#pragma once

namespace tt {

__device__ __forceinline__ float exp2_poly(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.999928074f, c1 = 0.693260985f, c2 = 0.242611122f, c3 = 0.0551716691f;
  x = fmaxf(x, -126.0f);
  const float t = x + kRound;
  const float n = t - kRound;
  const float f = x - n;
  const float p = fmaf(fmaf(fmaf(c3, f, c2), f, c1), f, c0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace tt

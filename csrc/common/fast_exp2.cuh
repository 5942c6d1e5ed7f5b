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

namespace tt {

// ---- packed fp32 pairs (sm_100 f32x2 FMA/ADD: one instruction for two lanes of math)
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// exp2_poly on two values with the packed pipe (same method and coefficients as exp2_poly).
__device__ __forceinline__ void exp2_poly2(float& x0, float& x1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.999928074f, c1 = 0.693260985f, c2 = 0.242611122f, c3 = 0.0551716691f;
  const unsigned long long x = f2_pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const unsigned long long t = f2_add(x, f2_pack(kRound, kRound));
  const unsigned long long n = f2_sub(t, f2_pack(kRound, kRound));
  const unsigned long long f = f2_sub(x, n);
  unsigned long long p = f2_fma(f2_pack(c3, c3), f, f2_pack(c2, c2));
  p = f2_fma(p, f, f2_pack(c1, c1));
  p = f2_fma(p, f, f2_pack(c0, c0));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  x0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  x1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

}  // namespace tt

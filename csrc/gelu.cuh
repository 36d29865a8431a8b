// GELU (erf form) pieces shared by the elementwise kernels and the GEMM
// epilogues that apply the activation or its derivative.
#pragma once

#include "common.cuh"

namespace zq {

// Gaussian CDF and PDF for GELU.  erf uses the rational approximation of
// Abramowitz & Stegun, Handbook of Mathematical Functions (1964), formula
// 7.1.26 (Hastings): for a >= 0,
//   erf(a) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-a^2) + e(a),
//   t = 1 / (1 + p a),  |e(a)| <= 1.5e-7.
// With a = |x| / sqrt(2), exp(-a^2) = exp(-x^2 / 2) is also the unnormalised
// PDF, so one reciprocal and one exponential give both.
struct GeluCP {
  float cdf, pdf;
};

__device__ __forceinline__ GeluCP gelu_cdf_pdf(float x) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f,
                  kA4 = -1.453152027f, kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752f, kInvSqrt2Pi = 0.39894228040143268f;
  const float a = fabsf(x) * kInvSqrt2;
  const float t = __fdividef(1.0f, fmaf(kP, a, 1.0f));
  const float e = __expf(-0.5f * x * x);
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, kA5, kA4), kA3), kA2), kA1);
  const float tail = 0.5f * poly * e;  // = (1 - erf(a)) / 2
  GeluCP r;
  r.cdf = x >= 0.0f ? 1.0f - tail : tail;
  r.pdf = e * kInvSqrt2Pi;
  return r;
}

}  // namespace zq

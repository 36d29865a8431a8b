// SwiGLU (silu(g)·u) pieces shared by the elementwise kernels and the GEMM
// epilogues, so both paths produce the same bits.
//
// sigmoid(g) = 1 / (1 + e^-g) with the fast exponential and reciprocal
// (__expf, __fdividef): relative error of a few ulp in fp32, far below the
// bf16 rounding of every input and output here.  For g < -87 the denominator
// reaches 2^126..inf and __fdividef returns 0, the limit of sigmoid.
#pragma once

#include "common.cuh"

namespace zq {

__device__ __forceinline__ float swiglu_sigmoid(float g) {
  return __fdividef(1.0f, 1.0f + __expf(-g));
}

// silu(g)·u
__device__ __forceinline__ float swiglu_fwd_val(float g, float u) {
  return g * swiglu_sigmoid(g) * u;
}

// gradients of silu(g)·u for an incoming d:
//   du = d·silu(g),  dg = d·u·s·(1 + g·(1 - s)),  s = sigmoid(g)
__device__ __forceinline__ void swiglu_bwd_vals(float d, float g, float u, float& dg, float& du) {
  const float s = swiglu_sigmoid(g);
  du = d * (g * s);
  dg = d * u * s * (1.0f + g * (1.0f - s));
}

}  // namespace zq

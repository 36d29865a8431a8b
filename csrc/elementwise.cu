// Memory-bound kernels of the decoder step: fused residual-add + RMSNorm
// (forward/backward), RoPE, GELU, SwiGLU, fused cross-entropy, AdamW and Lion
// on flat buffers.  All read bf16/fp32 with 16-byte vector accesses where the
// layout allows and compute in fp32.  erf/exp/sin/cos/rsqrt are CUDA's own
// functions.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace zq {

// ----------------------------------------------------------------------------
// RMSNorm (+ residual add).  One CTA of 128 threads per row; each thread owns
// up to 8 chunks of 8 bf16 (D <= 8192, D % 8 == 0).
// ----------------------------------------------------------------------------
constexpr int kNormThreads = 128;
constexpr int kNormMaxChunks = 8;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

__device__ __forceinline__ float block_sum_128(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0] + red[1] + red[2] + red[3];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ d,
    const float* __restrict__ w, __nv_bfloat16* __restrict__ hout, __nv_bfloat16* __restrict__ y,
    float* __restrict__ rstd, int D, float eps) {
  __shared__ float red[4];
  const int64_t row = blockIdx.x;
  const int nch = D >> 3;
  float v[kNormMaxChunks][8];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ch = c * kNormThreads + threadIdx.x;
    if (ch < nch) {
      const int64_t off = row * D + (int64_t)ch * 8;
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(h + off), v[c]);
      if (d != nullptr) {
        float t[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(d + off), t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] += t[i];
        // round the residual stream to bf16, exactly what is stored and reused
        uint4 packed = f32_to_bf16x8(v[c]);
        *reinterpret_cast<uint4*>(hout + off) = packed;
        bf16x8_to_f32(packed, v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  const float tot = block_sum_128(ss, red);
  const float r = rsqrtf(tot / (float)D + eps);
  if (threadIdx.x == 0) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ch = c * kNormThreads + threadIdx.x;
    if (ch < nch) {
      const int64_t off = row * D + (int64_t)ch * 8;
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * w[ch * 8 + i];
      *reinterpret_cast<uint4*>(y + off) = f32_to_bf16x8(o);
    }
  }
}

// dx = r * (g*w - xhat * mean(g*w*xhat)) [+ gh];  dw += sum_rows g * xhat
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ gy, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ w, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ gh, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw_part, int64_t M, int D) {
  __shared__ float red[4];
  const int nch = D >> 3;
  float dwacc[kNormMaxChunks][8];
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) dwacc[c][i] = 0.0f;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const float r = rstd[row];
    float xh[kNormMaxChunks][8], gw[kNormMaxChunks][8];
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
      const int ch = c * kNormThreads + threadIdx.x;
      if (ch < nch) {
        const int64_t off = row * D + (int64_t)ch * 8;
        float g[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + off), xh[c]);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(gy + off), g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] *= r;
          gw[c][i] = g[i] * w[ch * 8 + i];
          dot += gw[c][i] * xh[c][i];
          dwacc[c][i] += g[i] * xh[c][i];
        }
      }
    }
    const float mean = block_sum_128(dot, red) / (float)D;
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
      const int ch = c * kNormThreads + threadIdx.x;
      if (ch < nch) {
        const int64_t off = row * D + (int64_t)ch * 8;
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (gw[c][i] - xh[c][i] * mean);
        if (gh != nullptr) {
          float t[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(gh + off), t);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] += t[i];
        }
        *reinterpret_cast<uint4*>(dx + off) = f32_to_bf16x8(o);
      }
    }
  }
  // this CTA's partial weight gradient: one row of dw_part (summed on the host side)
  float* dst = dw_part + (int64_t)blockIdx.x * D;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const int ch = c * kNormThreads + threadIdx.x;
    if (ch < nch) {
      float4* d4 = reinterpret_cast<float4*>(dst + ch * 8);
      d4[0] = make_float4(dwacc[c][0], dwacc[c][1], dwacc[c][2], dwacc[c][3]);
      d4[1] = make_float4(dwacc[c][4], dwacc[c][5], dwacc[c][6], dwacc[c][7]);
    }
  }
}

// ----------------------------------------------------------------------------
// RoPE, rotate-half convention; x [rows = B*S*H, D], position = (row / H) % S.
// cs: [S, D/2] float2 (cos, sin) table; each thread rotates 8 pairs with
// 16-byte loads/stores from both halves of the row.
// ----------------------------------------------------------------------------
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                            const float2* __restrict__ cs, int64_t rows, int S, int H, int D,
                            float sign) {
  const int half = D >> 1;
  const int groups = half >> 3;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows * groups) return;
  const int64_t row = t / groups;
  const int i0 = (int)(t % groups) * 8;
  const int pos = (int)((row / H) % S);
  float a[8], b[8], oa[8], ob[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + row * D + i0), a);
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + row * D + half + i0), b);
  const float4* c4 = reinterpret_cast<const float4*>(cs + (int64_t)pos * half + i0);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 v = c4[j];  // (cos, sin) of pairs 2j and 2j+1
    const float c0 = v.x, s0 = v.y * sign, c1 = v.z, s1 = v.w * sign;
    oa[2 * j] = a[2 * j] * c0 - b[2 * j] * s0;
    ob[2 * j] = b[2 * j] * c0 + a[2 * j] * s0;
    oa[2 * j + 1] = a[2 * j + 1] * c1 - b[2 * j + 1] * s1;
    ob[2 * j + 1] = b[2 * j + 1] * c1 + a[2 * j + 1] * s1;
  }
  *reinterpret_cast<uint4*>(out + row * D + i0) = f32_to_bf16x8(oa);
  *reinterpret_cast<uint4*>(out + row * D + half + i0) = f32_to_bf16x8(ob);
}

// ----------------------------------------------------------------------------
// GELU (erf form) and SwiGLU
// ----------------------------------------------------------------------------
__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                int64_t n8) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float v[8], o[8];
  bf16x8_to_f32(reinterpret_cast<const uint4*>(x)[t], v);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.5f * v[i] * (1.0f + erff(v[i] * 0.70710678118654752f));
  reinterpret_cast<uint4*>(y)[t] = f32_to_bf16x8(o);
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ dx, int64_t n8) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float v[8], gg[8], o[8];
  bf16x8_to_f32(reinterpret_cast<const uint4*>(x)[t], v);
  bf16x8_to_f32(reinterpret_cast<const uint4*>(g)[t], gg);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float cdf = 0.5f * (1.0f + erff(v[i] * 0.70710678118654752f));
    const float pdf = expf(-0.5f * v[i] * v[i]) * 0.39894228040143268f;
    o[i] = gg[i] * (cdf + v[i] * pdf);
  }
  reinterpret_cast<uint4*>(dx)[t] = f32_to_bf16x8(o);
}

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gate,
                                  const __nv_bfloat16* __restrict__ up, __nv_bfloat16* __restrict__ y,
                                  int64_t n8) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float a[8], b[8], o[8];
  bf16x8_to_f32(reinterpret_cast<const uint4*>(gate)[t], a);
  bf16x8_to_f32(reinterpret_cast<const uint4*>(up)[t], b);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = a[i] / (1.0f + expf(-a[i])) * b[i];
  reinterpret_cast<uint4*>(y)[t] = f32_to_bf16x8(o);
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ g,
                                  const __nv_bfloat16* __restrict__ gate,
                                  const __nv_bfloat16* __restrict__ up,
                                  __nv_bfloat16* __restrict__ dgate, __nv_bfloat16* __restrict__ dup,
                                  int64_t n8) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n8) return;
  float gg[8], a[8], b[8], da[8], db[8];
  bf16x8_to_f32(reinterpret_cast<const uint4*>(g)[t], gg);
  bf16x8_to_f32(reinterpret_cast<const uint4*>(gate)[t], a);
  bf16x8_to_f32(reinterpret_cast<const uint4*>(up)[t], b);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float sg = 1.0f / (1.0f + expf(-a[i]));
    const float silu = a[i] * sg;
    db[i] = gg[i] * silu;
    da[i] = gg[i] * b[i] * sg * (1.0f + a[i] * (1.0f - sg));
  }
  reinterpret_cast<uint4*>(dgate)[t] = f32_to_bf16x8(da);
  reinterpret_cast<uint4*>(dup)[t] = f32_to_bf16x8(db);
}

// ----------------------------------------------------------------------------
// Cross-entropy over [M, Vpad] bf16 logits, first `vocab` columns valid.
// ----------------------------------------------------------------------------
constexpr int kCEThreads = 256;

__global__ void __launch_bounds__(kCEThreads) ce_fwd_kernel(
    const __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets,
    float* __restrict__ loss, float* __restrict__ lse_out, float* __restrict__ count, int64_t Vpad,
    int64_t vocab, int64_t ignore_index) {
  __shared__ float smax[kCEThreads / 32], ssum[kCEThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* lr = logits + row * Vpad;
  float m = -INFINITY, s = 0.0f;
  const int64_t nch = vocab >> 3;  // full 8-wide chunks
  for (int64_t ch = threadIdx.x; ch < nch; ch += kCEThreads) {
    float v[8];
    bf16x8_to_f32(reinterpret_cast<const uint4*>(lr)[ch], v);
    float cm = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) cm = fmaxf(cm, v[i]);
    const float nm = fmaxf(m, cm);
    float acc = s * expf(m - nm);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += expf(v[i] - nm);
    m = nm;
    s = acc;
  }
  for (int64_t c = nch * 8 + threadIdx.x; c < vocab; c += kCEThreads) {
    const float v = __bfloat162float(lr[c]);
    const float nm = fmaxf(m, v);
    s = s * expf(m - nm) + expf(v - nm);
    m = nm;
  }
  // combine (m, s) across the block
  float wm = warp_max(m);
  float ws = s * (m == -INFINITY ? 0.0f : expf(m - wm));
  ws = warp_sum(ws);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { smax[warp] = wm; ssum[warp] = ws; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int i = 0; i < kCEThreads / 32; ++i) M = fmaxf(M, smax[i]);
    float S = 0.0f;
    for (int i = 0; i < kCEThreads / 32; ++i)
      S += smax[i] == -INFINITY ? 0.0f : ssum[i] * expf(smax[i] - M);
    const float lse = M + logf(S);
    lse_out[row] = lse;
    const int64_t t = targets[row];
    if (t == ignore_index || t < 0 || t >= vocab) {
      loss[row] = 0.0f;
    } else {
      loss[row] = lse - __bfloat162float(lr[t]);
      atomicAdd(count, 1.0f);
    }
  }
}

// logits <- (softmax - onehot) * scale, zero for ignored rows and padded columns
__global__ void __launch_bounds__(kCEThreads) ce_bwd_kernel(
    __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets,
    const float* __restrict__ lse, const float* __restrict__ scale_ptr, int64_t Vpad, int64_t vocab,
    int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * Vpad;
  const int64_t t = targets[row];
  const bool ignored = (t == ignore_index || t < 0 || t >= vocab);
  const float L = lse[row];
  const float sc = ignored ? 0.0f : scale_ptr[0];
  const int64_t nch = Vpad >> 3;
  for (int64_t ch = threadIdx.x; ch < nch; ch += kCEThreads) {
    float v[8];
    bf16x8_to_f32(reinterpret_cast<const uint4*>(lr)[ch], v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t c = ch * 8 + i;
      float gval = 0.0f;
      if (c < vocab) gval = (expf(v[i] - L) - (c == t ? 1.0f : 0.0f)) * sc;
      v[i] = gval;
    }
    reinterpret_cast<uint4*>(lr)[ch] = f32_to_bf16x8(v);
  }
}

// ----------------------------------------------------------------------------
// AdamW on flat fp32 buffers (optionally writes a bf16 copy)
// ----------------------------------------------------------------------------
template <typename G>
__global__ void adamw_kernel(float* __restrict__ p, const G* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ pbf, int64_t n,
                             float lr, float b1, float b2, float eps, float wd, float bc1,
                             float bc2, float gscale) {
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = to_f32<G>(g[i]) * gscale;
    float pi = p[i] * (1.0f - lr * wd);
    const float mi = b1 * m[i] + (1.0f - b1) * gi;
    const float vi = b2 * v[i] + (1.0f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    pi -= step_size * mi / (sqrtf(vi) * inv_sqrt_bc2 + eps);
    p[i] = pi;
    if (pbf != nullptr) pbf[i] = __float2bfloat16_rn(pi);
  }
}

// ----------------------------------------------------------------------------
// Lion with stochastic rounding for fp16 masters.  Philox4x32-10 (Salmon et
// al., "Parallel random numbers: as easy as 1, 2, 3", SC'11) keyed by the seed,
// counter = element index.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    const uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += W0;
    key.y += W1;
  }
  return ctr;
}

template <typename P, typename G>
__global__ void lion_kernel(P* __restrict__ master, const G* __restrict__ grad,
                            float* __restrict__ mom, int64_t n, float lr, float b1, float b2,
                            float wd, unsigned long long seed) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float g = to_f32<G>(grad[i]);
    const float mi = mom[i];
    const float c = mi * b1 + g * (1.0f - b1);
    const float upd = (c > 0.0f) ? 1.0f : ((c < 0.0f) ? -1.0f : 0.0f);
    float x = to_f32<P>(master[i]);
    x = x - lr * (upd + wd * x);
    mom[i] = mi * b2 + g * (1.0f - b2);
    if (sizeof(P) == 2) {
      const uint4 r = philox4x32_10(make_uint4((uint32_t)i, (uint32_t)(i >> 32), 0u, 0u),
                                    make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
      const float u = (float)(r.x >> 8) * (1.0f / 16777216.0f) - 0.5f;
      const float eps = fmaxf(fabsf(x) * 9.765625e-4f, 6.103515625e-05f);  // fp16 eps, tiny
      x = x + u * eps;
    }
    master[i] = from_f32<P>(x);
  }
}

}  // namespace zq

using namespace zq;

static inline __nv_bfloat16* bf(at::Tensor& t) {
  return reinterpret_cast<__nv_bfloat16*>(t.data_ptr<at::BFloat16>());
}
static inline const __nv_bfloat16* cbf(const at::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr<at::BFloat16>());
}

static void check_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              ": expected a contiguous CUDA bfloat16 tensor");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, ": 16-byte alignment");
}

void add_rmsnorm_fwd(at::Tensor h, c10::optional<at::Tensor> d, at::Tensor w, at::Tensor hout,
                     at::Tensor y, at::Tensor rstd, double eps) {
  check_bf16(h, "h");
  check_bf16(y, "y");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "norm weight must be fp32");
  const int64_t D = h.size(-1), M = h.numel() / D;
  TORCH_CHECK(w.numel() == D, "norm weight has ", w.numel(), " elements, expected ", D);
  TORCH_CHECK(y.numel() == h.numel() && rstd.numel() >= M && rstd.scalar_type() == at::kFloat,
              "norm output / rstd sizes");
  TORCH_CHECK(D % 8 == 0 && D <= 8 * kNormThreads * kNormMaxChunks, "D must be %8 and <= 8192");
  const at::cuda::CUDAGuard guard(h.device());
  const __nv_bfloat16* dp = nullptr;
  if (d.has_value() && d->defined()) {
    check_bf16(*d, "delta");
    check_bf16(hout, "hout");
    TORCH_CHECK(d->numel() == h.numel() && hout.numel() == h.numel(), "add_rmsnorm: sizes");
    dp = cbf(*d);
  }
  add_rmsnorm_fwd_kernel<<<(unsigned)M, kNormThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(h), dp, w.data_ptr<float>(), dp ? bf(hout) : nullptr, bf(y), rstd.data_ptr<float>(),
      (int)D, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dw_part: [grid, D] fp32 partial sums, grid = dw_part.size(0); caller sums over rows
void rmsnorm_bwd(at::Tensor gy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                 c10::optional<at::Tensor> gh, at::Tensor dx, at::Tensor dw_part) {
  check_bf16(gy, "gy");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  const int64_t D = x.size(-1), M = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8 * kNormThreads * kNormMaxChunks, "D must be %8 and <= 8192");
  TORCH_CHECK(w.numel() == D && w.scalar_type() == at::kFloat, "norm weight must be fp32 [D]");
  TORCH_CHECK(gy.numel() == x.numel() && dx.numel() == x.numel() && rstd.numel() >= M,
              "rmsnorm_bwd: tensor sizes");
  const at::cuda::CUDAGuard guard(x.device());
  const __nv_bfloat16* ghp = nullptr;
  if (gh.has_value() && gh->defined()) {
    check_bf16(*gh, "gh");
    TORCH_CHECK(gh->numel() == x.numel(), "rmsnorm_bwd: gh size");
    ghp = cbf(*gh);
  }
  TORCH_CHECK(dw_part.dim() == 2 && dw_part.size(1) == D && dw_part.is_contiguous() &&
                  dw_part.scalar_type() == at::kFloat, "dw_part must be fp32 [grid, D]");
  const int64_t grid = std::min<int64_t>(M, dw_part.size(0));
  rmsnorm_bwd_kernel<<<(unsigned)grid, kNormThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(gy), cbf(x), w.data_ptr<float>(), rstd.data_ptr<float>(), ghp, bf(dx),
      dw_part.data_ptr<float>(), M, (int)D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope(at::Tensor x, at::Tensor out, at::Tensor cs, double sign) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 4, "rope: x must be [B, S, H, D]");
  TORCH_CHECK(out.numel() == x.numel(), "rope: out size");
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2), D = x.size(3);
  TORCH_CHECK(D % 16 == 0, "rope: head dim must be a multiple of 16");
  TORCH_CHECK(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.numel() >= S * D,
              "rope: cos/sin table must be fp32 [S, D/2, 2]");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t rows = B * S * H;
  const int64_t total = rows * (D / 16);
  const int bs = 256;
  rope_kernel<<<(unsigned)((total + bs - 1) / bs), bs, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(x), bf(out), reinterpret_cast<const float2*>(cs.data_ptr<float>()), rows, (int)S,
      (int)H, (int)D, (float)sign);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static inline unsigned ew_grid(int64_t n8) { return (unsigned)((n8 + 255) / 256); }

void gelu_fwd(at::Tensor x, at::Tensor y) {
  check_bf16(x, "x");
  check_bf16(y, "y");
  TORCH_CHECK(x.numel() % 8 == 0 && y.numel() == x.numel(), "gelu: numel % 8 and equal sizes");
  const int64_t n8 = x.numel() / 8;
  const at::cuda::CUDAGuard guard(x.device());
  gelu_fwd_kernel<<<ew_grid(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(x), bf(y), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_bwd(at::Tensor g, at::Tensor x, at::Tensor dx) {
  check_bf16(g, "g");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  TORCH_CHECK(x.numel() % 8 == 0 && g.numel() == x.numel() && dx.numel() == x.numel(),
              "gelu: numel % 8 and equal sizes");
  const int64_t n8 = x.numel() / 8;
  const at::cuda::CUDAGuard guard(x.device());
  gelu_bwd_kernel<<<ew_grid(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(g), cbf(x), bf(dx), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_fwd(at::Tensor gate, at::Tensor up, at::Tensor y) {
  check_bf16(gate, "gate");
  check_bf16(up, "up");
  check_bf16(y, "y");
  TORCH_CHECK(gate.numel() % 8 == 0 && up.numel() == gate.numel() && y.numel() == gate.numel(),
              "swiglu: numel % 8 and equal sizes");
  const int64_t n8 = gate.numel() / 8;
  const at::cuda::CUDAGuard guard(gate.device());
  swiglu_fwd_kernel<<<ew_grid(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(cbf(gate), cbf(up), bf(y), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_bwd(at::Tensor g, at::Tensor gate, at::Tensor up, at::Tensor dgate, at::Tensor dup) {
  check_bf16(g, "g");
  check_bf16(gate, "gate");
  check_bf16(up, "up");
  check_bf16(dgate, "dgate");
  check_bf16(dup, "dup");
  TORCH_CHECK(gate.numel() % 8 == 0 && g.numel() == gate.numel() && up.numel() == gate.numel() &&
                  dgate.numel() == gate.numel() && dup.numel() == gate.numel(),
              "swiglu_bwd: numel % 8 and equal sizes");
  const int64_t n8 = gate.numel() / 8;
  const at::cuda::CUDAGuard guard(gate.device());
  swiglu_bwd_kernel<<<ew_grid(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(g), cbf(gate), cbf(up), bf(dgate), bf(dup), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_fwd(at::Tensor logits, at::Tensor targets, at::Tensor loss, at::Tensor lse,
            at::Tensor count, int64_t vocab, int64_t ignore_index) {
  check_bf16(logits, "logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "targets int64");
  const int64_t M = logits.size(0), Vpad = logits.size(1);
  TORCH_CHECK(Vpad % 8 == 0 && vocab <= Vpad, "ce: Vpad % 8 and vocab <= Vpad");
  TORCH_CHECK(targets.numel() == M && loss.numel() >= M && lse.numel() >= M, "ce: one target per row");
  const at::cuda::CUDAGuard guard(logits.device());
  ce_fwd_kernel<<<(unsigned)M, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(logits), targets.data_ptr<int64_t>(), loss.data_ptr<float>(), lse.data_ptr<float>(),
      count.data_ptr<float>(), Vpad, vocab, ignore_index);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_bwd(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor scale,
            int64_t vocab, int64_t ignore_index) {
  check_bf16(logits, "logits");
  const int64_t M = logits.size(0), Vpad = logits.size(1);
  TORCH_CHECK(Vpad % 8 == 0 && vocab <= Vpad && targets.numel() == M && lse.numel() >= M &&
                  targets.scalar_type() == at::kLong && scale.numel() >= 1,
              "ce_bwd: sizes");
  const at::cuda::CUDAGuard guard(logits.device());
  ce_bwd_kernel<<<(unsigned)M, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bf(logits), targets.data_ptr<int64_t>(), lse.data_ptr<float>(), scale.data_ptr<float>(),
      Vpad, vocab, ignore_index);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v,
                c10::optional<at::Tensor> pbf16, double lr, double b1, double b2, double eps,
                double wd, double bc1, double bc2, double gscale) {
  TORCH_CHECK(p.is_cuda() && p.scalar_type() == at::kFloat && p.is_contiguous(), "adamw: fp32 param");
  TORCH_CHECK(m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat, "adamw: fp32 moments");
  const int64_t n = p.numel();
  TORCH_CHECK(g.numel() >= n && m.numel() >= n && v.numel() >= n, "adamw: sizes");
  const at::cuda::CUDAGuard guard(p.device());
  __nv_bfloat16* pb = nullptr;
  if (pbf16.has_value() && pbf16->defined()) pb = bf(*pbf16);
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, sms * 16));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (g.scalar_type() == at::kFloat) {
    adamw_kernel<float><<<grid, 256, 0, stream>>>(p.data_ptr<float>(), g.data_ptr<float>(),
        m.data_ptr<float>(), v.data_ptr<float>(), pb, n, (float)lr, (float)b1, (float)b2,
        (float)eps, (float)wd, (float)bc1, (float)bc2, (float)gscale);
  } else {
    TORCH_CHECK(g.scalar_type() == at::kBFloat16, "adamw: grad fp32 or bf16");
    adamw_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p.data_ptr<float>(), cbf(g),
        m.data_ptr<float>(), v.data_ptr<float>(), pb, n, (float)lr, (float)b1, (float)b2,
        (float)eps, (float)wd, (float)bc1, (float)bc2, (float)gscale);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lion_step(at::Tensor master, at::Tensor grad, at::Tensor mom, double lr, double b1, double b2,
               double wd, int64_t seed) {
  TORCH_CHECK(master.is_cuda() && master.is_contiguous() && grad.is_contiguous(), "lion: contiguous CUDA");
  TORCH_CHECK(mom.scalar_type() == at::kFloat, "lion: fp32 momentum");
  const int64_t n = master.numel();
  const at::cuda::CUDAGuard guard(master.device());
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, sms * 16));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto gf = grad.scalar_type() == at::kFloat ? grad : grad.to(at::kFloat);
  if (master.scalar_type() == at::kFloat) {
    lion_kernel<float, float><<<grid, 256, 0, stream>>>(master.data_ptr<float>(), gf.data_ptr<float>(),
        mom.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)wd, (unsigned long long)seed);
  } else {
    TORCH_CHECK(master.scalar_type() == at::kHalf, "lion: fp32 or fp16 master");
    lion_kernel<__half, float><<<grid, 256, 0, stream>>>(
        reinterpret_cast<__half*>(master.data_ptr<at::Half>()), gf.data_ptr<float>(),
        mom.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)wd, (unsigned long long)seed);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

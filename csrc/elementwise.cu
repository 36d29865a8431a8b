// Memory-bound kernels of the decoder step: fused residual-add + RMSNorm
// (forward/backward), RoPE, GELU, SwiGLU, fused cross-entropy, AdamW and Lion
// on flat buffers.  All read bf16/fp32 with 16-byte vector accesses where the
// layout allows and compute in fp32.  erf/exp/sin/cos/rsqrt are CUDA's own
// functions, except the GELU CDF (a named published approximation, below).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gelu.cuh"
#include "swiglu.cuh"

namespace zq {

// ----------------------------------------------------------------------------
// RMSNorm (+ residual add).  A team of TPR lanes (32, 64 or 128) owns one row;
// each lane owns NC chunks of 8 bf16 (D <= 8 * TPR * NC, D % 8 == 0) and
// issues all of its loads before the first use, so a 256-thread CTA keeps
// 256 * NC * 16 B (x2-3 tensors) in flight.  Teams of one warp reduce with
// shuffles only; wider teams add one shared-memory exchange.
// ----------------------------------------------------------------------------
constexpr int kNormThreads = 256;
constexpr int kNormMaxD = 8192;

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

// Sum of v over the TPR lanes of this thread's team.  Every thread of the team
// must call it.  Teams wider than a warp exchange through shared memory under a
// named barrier of their own (id 1 + team, TPR threads), so the teams of a CTA
// never wait for one another and one team's loads overlap another's arithmetic.
template <int TPR>
__device__ __forceinline__ float team_sum(float v, float* red) {
  v = warp_sum(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    constexpr int W = TPR / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bar = 1 + (int)threadIdx.x / TPR;
    if (lane == 0) red[warp] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(TPR) : "memory");
    const int base = (warp / W) * W;
    float r = 0.0f;
#pragma unroll
    for (int i = 0; i < W; ++i) r += red[base + i];
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(TPR) : "memory");
    return r;
  }
}

template <int NC, int TPR>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ d,
    const float* __restrict__ w, __nv_bfloat16* __restrict__ hout, __nv_bfloat16* __restrict__ y,
    float* __restrict__ rstd, int64_t M, int D, float eps) {
  __shared__ float red[kNormThreads / 32];
  constexpr int R = kNormThreads / TPR;
  const int team = threadIdx.x / TPR, tl = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * R + team;
  const bool live = row < M;
  const int nch = D >> 3;
  uint4 hv[NC], dv[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ch = c * TPR + tl;
    if (live && ch < nch) {
      hv[c] = *reinterpret_cast<const uint4*>(h + row * D + (int64_t)ch * 8);
      if (d != nullptr) dv[c] = *reinterpret_cast<const uint4*>(d + row * D + (int64_t)ch * 8);
    }
  }
  float v[NC][8];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ch = c * TPR + tl;
    if (live && ch < nch) {
      bf16x8_to_f32(hv[c], v[c]);
      if (d != nullptr) {
        float t[8];
        bf16x8_to_f32(dv[c], t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] += t[i];
        // round the residual stream to bf16, exactly what is stored and reused
        const uint4 packed = f32_to_bf16x8(v[c]);
        *reinterpret_cast<uint4*>(hout + row * D + (int64_t)ch * 8) = packed;
        bf16x8_to_f32(packed, v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  const float tot = team_sum<TPR>(ss, red);
  if (!live) return;
  const float r = rsqrtf(tot / (float)D + eps);
  if (tl == 0) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ch = c * TPR + tl;
    if (ch < nch) {
      const float4 w0 = reinterpret_cast<const float4*>(w)[ch * 2];
      const float4 w1 = reinterpret_cast<const float4*>(w)[ch * 2 + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * ww[i];
      *reinterpret_cast<uint4*>(y + row * D + (int64_t)ch * 8) = f32_to_bf16x8(o);
    }
  }
}

// dx = r * (g*w - xhat * mean(g*w*xhat)) [+ gh];  dw += sum_rows g * xhat.
// Teams walk rows with a grid stride and keep their dw share in registers; the
// teams of a CTA combine through shared memory into one row of dw_part.  With
// PF the next row group's x, dy and rstd are loaded before this group's
// arithmetic (two groups in flight per team); the residual gradient gh is loaded
// at the top of its own group and first used after the row reduction.
template <int NC, int TPR, bool PF>
__global__ void __launch_bounds__(kNormThreads, (PF && NC <= 3) ? 2 : 1) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ gy, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ w, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ gh, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw_part, int64_t M, int D) {
  __shared__ float red[kNormThreads / 32];
  extern __shared__ float sdw[];  // [D]
  constexpr int R = kNormThreads / TPR;
  const int team = threadIdx.x / TPR, tl = threadIdx.x % TPR;
  const int nch = D >> 3;
  for (int i = threadIdx.x; i < D; i += kNormThreads) sdw[i] = 0.0f;
  float dwacc[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) dwacc[c][i] = 0.0f;
  const float4* w4 = reinterpret_cast<const float4*>(w);  // [D/4], L1-resident
  const int64_t groups = (M + R - 1) / R;
  uint4 xv[NC], gv[NC];
  float r = 0.0f;
  auto load_xg = [&](int64_t row, uint4 (&xo)[NC], uint4 (&go)[NC], float& ro) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int ch = c * TPR + tl;
      if (ch < nch) {
        const int64_t off = row * D + (int64_t)ch * 8;
        xo[c] = *reinterpret_cast<const uint4*>(x + off);
        go[c] = *reinterpret_cast<const uint4*>(gy + off);
      }
    }
    ro = rstd[row];
  };
  if constexpr (PF) {
    const int64_t row0 = (int64_t)blockIdx.x * R + team;
    if (row0 < M) load_xg(row0, xv, gv, r);
  }
  for (int64_t gidx = blockIdx.x; gidx < groups; gidx += gridDim.x) {
    const int64_t row = gidx * R + team;
    const bool live = row < M;
    uint4 hv[NC];
    if (live && gh != nullptr) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int ch = c * TPR + tl;
        if (ch < nch) hv[c] = *reinterpret_cast<const uint4*>(gh + row * D + (int64_t)ch * 8);
      }
    }
    uint4 xn[NC], gn[NC];
    float rn = 0.0f;
    if constexpr (PF) {
      const int64_t nrow = (gidx + gridDim.x) * R + team;  // >= M once past the last group
      if (nrow < M) load_xg(nrow, xn, gn, rn);
    } else {
      if (live) load_xg(row, xv, gv, r);
    }
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int ch = c * TPR + tl;
      if (live && ch < nch) {
        float xf[8], gf[8];
        bf16x8_to_f32(xv[c], xf);
        bf16x8_to_f32(gv[c], gf);
        const float4 w0 = __ldg(w4 + ch * 2), w1 = __ldg(w4 + ch * 2 + 1);
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = xf[i] * r;
          dot += gf[i] * ww[i] * xh;
          dwacc[c][i] += gf[i] * xh;
        }
      }
    }
    const float mean = team_sum<TPR>(dot, red) / (float)D;
    if (live) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int ch = c * TPR + tl;
        if (ch < nch) {
          float xf[8], gf[8], o[8];
          bf16x8_to_f32(xv[c], xf);
          bf16x8_to_f32(gv[c], gf);
          const float4 w0 = __ldg(w4 + ch * 2), w1 = __ldg(w4 + ch * 2 + 1);
          const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = r * (gf[i] * ww[i] - xf[i] * r * mean);
          if (gh != nullptr) {
            float t[8];
            bf16x8_to_f32(hv[c], t);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] += t[i];
          }
          *reinterpret_cast<uint4*>(dx + row * D + (int64_t)ch * 8) = f32_to_bf16x8(o);
        }
      }
    }
    if constexpr (PF) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        xv[c] = xn[c];
        gv[c] = gn[c];
      }
      r = rn;
    }
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int ch = c * TPR + tl;
    if (ch < nch) {
#pragma unroll
      for (int i = 0; i < 8; ++i) atomicAdd(&sdw[ch * 8 + i], dwacc[c][i]);
    }
  }
  __syncthreads();
  float* dst = dw_part + (int64_t)blockIdx.x * D;
  for (int i = threadIdx.x; i < D; i += kNormThreads) dst[i] = sdw[i];
}

// ----------------------------------------------------------------------------
// RoPE, rotate-half convention; x [rows = B*S*H, D], position = (row / H) % S.
// cs: [S, D/2] float2 (cos, sin) table; each thread rotates 8 pairs with
// 16-byte loads/stores from both halves of the row.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void rope_chunk(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                                           const float2* __restrict__ cs, int64_t t, int S, int H, int D,
                                           float sign, int64_t out_ld);

__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                            const float2* __restrict__ cs, int64_t rows, int S, int H, int D,
                            float sign, int64_t out_ld) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows * ((D >> 1) >> 3)) return;
  rope_chunk(x, out, cs, t, S, H, D, sign, out_ld);
}

// Two tensors in one launch (the q and k gradients of a fused projection):
// threads past the first tensor's chunks take the second's.
__global__ void rope2_kernel(const __nv_bfloat16* __restrict__ x1, __nv_bfloat16* __restrict__ out1,
                             int64_t rows1, int H1, int64_t ld1, const __nv_bfloat16* __restrict__ x2,
                             __nv_bfloat16* __restrict__ out2, int64_t rows2, int H2, int64_t ld2,
                             const float2* __restrict__ cs, int S, int D, float sign) {
  const int64_t groups = (D >> 1) >> 3;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n1 = rows1 * groups;
  if (t < n1) {
    rope_chunk(x1, out1, cs, t, S, H1, D, sign, ld1);
  } else if (t - n1 < rows2 * groups) {
    rope_chunk(x2, out2, cs, t - n1, S, H2, D, sign, ld2);
  }
}

// chunk t = (row, 8 rotary pairs) of x [rows = B*S*H, D] rotated into out
__device__ __forceinline__ void rope_chunk(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                                           const float2* __restrict__ cs, int64_t t, int S, int H, int D,
                                           float sign, int64_t out_ld) {
  const int half = D >> 1;
  const int groups = half >> 3;
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
    oa[2 * j] = rope_lo(a[2 * j], b[2 * j], c0, s0);
    ob[2 * j] = rope_hi(a[2 * j], b[2 * j], c0, s0);
    oa[2 * j + 1] = rope_lo(a[2 * j + 1], b[2 * j + 1], c1, s1);
    ob[2 * j + 1] = rope_hi(a[2 * j + 1], b[2 * j + 1], c1, s1);
  }
  // output row of token row / H has pitch out_ld (H * D when contiguous)
  __nv_bfloat16* orow = out + (row / H) * out_ld + (row % H) * D;
  *reinterpret_cast<uint4*>(orow + i0) = f32_to_bf16x8(oa);
  *reinterpret_cast<uint4*>(orow + half + i0) = f32_to_bf16x8(ob);
}

// ----------------------------------------------------------------------------
// GELU (erf form) and SwiGLU
// ----------------------------------------------------------------------------
// Each thread handles kEwIlp chunks of 8 elements, kEwIlp * blockDim apart, and
// issues all loads before computing.
constexpr int kEwIlp = 4;

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                int64_t n8) {
  const int64_t base = (int64_t)blockIdx.x * blockDim.x * kEwIlp + threadIdx.x;
  uint4 in[kEwIlp];
#pragma unroll
  for (int j = 0; j < kEwIlp; ++j) {
    const int64_t t = base + (int64_t)j * blockDim.x;
    if (t < n8) in[j] = reinterpret_cast<const uint4*>(x)[t];
  }
#pragma unroll
  for (int j = 0; j < kEwIlp; ++j) {
    const int64_t t = base + (int64_t)j * blockDim.x;
    if (t < n8) {
      float v[8], o[8];
      bf16x8_to_f32(in[j], v);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[i] * gelu_cdf_pdf(v[i]).cdf;
      reinterpret_cast<uint4*>(y)[t] = f32_to_bf16x8(o);
    }
  }
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ dx, int64_t n8) {
  const int64_t base = (int64_t)blockIdx.x * blockDim.x * kEwIlp + threadIdx.x;
  uint4 xin[kEwIlp], gin[kEwIlp];
#pragma unroll
  for (int j = 0; j < kEwIlp; ++j) {
    const int64_t t = base + (int64_t)j * blockDim.x;
    if (t < n8) {
      xin[j] = reinterpret_cast<const uint4*>(x)[t];
      gin[j] = reinterpret_cast<const uint4*>(g)[t];
    }
  }
#pragma unroll
  for (int j = 0; j < kEwIlp; ++j) {
    const int64_t t = base + (int64_t)j * blockDim.x;
    if (t < n8) {
      float v[8], gg[8], o[8];
      bf16x8_to_f32(xin[j], v);
      bf16x8_to_f32(gin[j], gg);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const GeluCP c = gelu_cdf_pdf(v[i]);
        o[i] = gg[i] * (c.cdf + v[i] * c.pdf);
      }
      reinterpret_cast<uint4*>(dx)[t] = f32_to_bf16x8(o);
    }
  }
}

// fp32 GELU CDF/PDF of the approximation above, for checking its error bound
__global__ void gelu_cdf_pdf_kernel(const float* __restrict__ x, float* __restrict__ cdf,
                                    float* __restrict__ pdf, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const GeluCP c = gelu_cdf_pdf(x[i]);
  cdf[i] = c.cdf;
  pdf[i] = c.pdf;
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
  for (int i = 0; i < 8; ++i) o[i] = swiglu_fwd_val(a[i], b[i]);
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
  for (int i = 0; i < 8; ++i) swiglu_bwd_vals(gg[i], a[i], b[i], da[i], db[i]);
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
    int64_t vocab, int64_t ignore_index, int64_t col0, int64_t vocab_total) {
  // The buffer holds columns [col0, col0 + vocab) of the vocabulary (col0 = 0 and
  // vocab_total = vocab for whole rows): lse is over those columns, and a row
  // whose target lies among them gets loss = lse - logit[target] and is counted.
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
    const bool valid = !(t == ignore_index || t < 0 || t >= vocab_total);
    if (valid && t >= col0 && t < col0 + vocab) {
      loss[row] = lse - __bfloat162float(lr[t - col0]);
      if (count != nullptr) atomicAdd(count, 1.0f);
    } else {
      loss[row] = 0.0f;
    }
  }
}

// logits <- (softmax - onehot) * scale, zero for ignored rows and padded columns
__global__ void __launch_bounds__(kCEThreads) ce_bwd_kernel(
    __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets,
    const float* __restrict__ lse, const float* __restrict__ scale_ptr, int64_t Vpad, int64_t vocab,
    int64_t ignore_index, int64_t col0, int64_t vocab_total) {
  // columns [col0, col0 + vocab) of the vocabulary; lse is the whole row's
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * Vpad;
  const int64_t t = targets[row] - col0;   // chunk-local target column (may be outside)
  const int64_t tg = targets[row];
  const bool ignored = (tg == ignore_index || tg < 0 || tg >= vocab_total);
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
                             float bc2, float gscale, const float* __restrict__ bcp,
                             const float* __restrict__ clip_sq, float max_norm) {
  if (bcp != nullptr) {  // bias corrections from the device-side optimizer clock
    bc1 = bcp[0];
    bc2 = bcp[1];
  }
  // gradient clipping with the squared global norm on the device (no host sync)
  if (clip_sq != nullptr) gscale *= fminf(1.0f, max_norm / (sqrtf(*clip_sq) + 1e-6f));
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

// Team width and chunks per lane for a row of D bf16: the narrowest team whose
// lanes need at most 8 chunks, then the smallest instantiated chunk count.
// Backward team shape: at most 4 chunks per lane up to D = 2048, then 128-lane
// teams (D = 3072: 3 chunks).  Up to 5 chunks per lane the kernel keeps two row
// groups in flight per team (with up to 3 chunks in 128 registers, so two CTAs
// per SM); wider rows load one group at a time.
static void norm_bwd_shape(int64_t D, int* tpr, int* nc) {
  const int64_t chunks = D / 8;
  if (chunks <= 32) { *tpr = 32; *nc = 1; }
  else if (chunks <= 64) { *tpr = 32; *nc = 2; }
  else if (chunks <= 128) { *tpr = 32; *nc = 4; }
  else if (chunks <= 256) { *tpr = 64; *nc = 4; }
  else {
    *tpr = 128;
    const int64_t need = (chunks + 127) / 128;
    *nc = need <= 3 ? 3 : need <= 5 ? (int)need : need <= 6 ? 6 : 8;
  }
}

#define ZQ_NORM_BWD_DISPATCH(TPR, NC, ...)                                        \
  do {                                                                            \
    if (TPR == 32) {                                                              \
      if (NC == 1) rmsnorm_bwd_kernel<1, 32, true>__VA_ARGS__;                    \
      else if (NC == 2) rmsnorm_bwd_kernel<2, 32, true>__VA_ARGS__;               \
      else rmsnorm_bwd_kernel<4, 32, true>__VA_ARGS__;                            \
    } else if (TPR == 64) {                                                       \
      rmsnorm_bwd_kernel<4, 64, true>__VA_ARGS__;                                 \
    } else {                                                                      \
      if (NC == 3) rmsnorm_bwd_kernel<3, 128, true>__VA_ARGS__;                   \
      else if (NC == 4) rmsnorm_bwd_kernel<4, 128, true>__VA_ARGS__;              \
      else if (NC == 5) rmsnorm_bwd_kernel<5, 128, true>__VA_ARGS__;              \
      else if (NC == 6) rmsnorm_bwd_kernel<6, 128, false>__VA_ARGS__;             \
      else rmsnorm_bwd_kernel<8, 128, false>__VA_ARGS__;                          \
    }                                                                             \
  } while (0)

static void norm_shape(int64_t D, int* tpr, int* nc) {
  const int64_t chunks = D / 8;
  *tpr = chunks <= 32 * 8 ? 32 : (chunks <= 64 * 8 ? 64 : 128);
  const int64_t need = (chunks + *tpr - 1) / *tpr;
  *nc = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= 6 ? 6 : 8;
}

#define ZQ_NORM_DISPATCH(TPR, NC, KERNEL, ...)                                     \
  do {                                                                            \
    if (TPR == 32) {                                                              \
      if (NC == 1) KERNEL<1, 32>__VA_ARGS__;                                      \
      else if (NC == 2) KERNEL<2, 32>__VA_ARGS__;                                 \
      else if (NC == 4) KERNEL<4, 32>__VA_ARGS__;                                 \
      else if (NC == 6) KERNEL<6, 32>__VA_ARGS__;                                 \
      else KERNEL<8, 32>__VA_ARGS__;                                              \
    } else if (TPR == 64) {                                                       \
      if (NC == 6) KERNEL<6, 64>__VA_ARGS__;                                      \
      else KERNEL<8, 64>__VA_ARGS__;                                              \
    } else {                                                                      \
      if (NC == 6) KERNEL<6, 128>__VA_ARGS__;                                     \
      else KERNEL<8, 128>__VA_ARGS__;                                             \
    }                                                                             \
  } while (0)

void add_rmsnorm_fwd(at::Tensor h, c10::optional<at::Tensor> d, at::Tensor w, at::Tensor hout,
                     at::Tensor y, at::Tensor rstd, double eps) {
  check_bf16(h, "h");
  check_bf16(y, "y");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "norm weight must be fp32");
  const int64_t D = h.size(-1), M = h.numel() / D;
  TORCH_CHECK(w.numel() == D, "norm weight has ", w.numel(), " elements, expected ", D);
  TORCH_CHECK(y.numel() == h.numel() && rstd.numel() >= M && rstd.scalar_type() == at::kFloat,
              "norm output / rstd sizes");
  TORCH_CHECK(D % 8 == 0 && D <= kNormMaxD, "D must be %8 and <= 8192");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, "norm weight: 16-byte alignment");
  const at::cuda::CUDAGuard guard(h.device());
  const __nv_bfloat16* dp = nullptr;
  if (d.has_value() && d->defined()) {
    check_bf16(*d, "delta");
    check_bf16(hout, "hout");
    TORCH_CHECK(d->numel() == h.numel() && hout.numel() == h.numel(), "add_rmsnorm: sizes");
    dp = cbf(*d);
  }
  if (M == 0) return;
  int tpr, nc;
  norm_shape(D, &tpr, &nc);
  const int rows_per_cta = kNormThreads / tpr;
  const unsigned grid = (unsigned)((M + rows_per_cta - 1) / rows_per_cta);
  auto stream = at::cuda::getCurrentCUDAStream();
  ZQ_NORM_DISPATCH(tpr, nc, add_rmsnorm_fwd_kernel, <<<grid, kNormThreads, 0, stream>>>(
      cbf(h), dp, w.data_ptr<float>(), dp ? bf(hout) : nullptr, bf(y), rstd.data_ptr<float>(), M,
      (int)D, (float)eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace zq {
// Raw-pointer launcher of the backward kernel, shared by the ATen wrapper below
// and the allocation-free entry point (noalloc.cu).  Writes one row of dw_part
// per CTA for at most max_grid CTAs and returns the number of rows written in
// *grid_out.  Allocates nothing.
cudaError_t launch_rmsnorm_bwd(const __nv_bfloat16* gy, const __nv_bfloat16* x, const float* w,
                               const float* rstd, const __nv_bfloat16* gh, __nv_bfloat16* dx,
                               float* dw_part, int64_t M, int D, int64_t max_grid,
                               cudaStream_t stream, int64_t* grid_out) {
  if (M < 1 || D < 8 || D % 8 != 0 || D > kNormMaxD || max_grid < 1) return cudaErrorInvalidValue;
  int tpr, nc;
  norm_bwd_shape(D, &tpr, &nc);
  const int rows_per_cta = kNormThreads / tpr;
  const int64_t groups = (M + rows_per_cta - 1) / rows_per_cta;
  const int64_t grid = std::min<int64_t>(groups, max_grid);
  const size_t smem = (size_t)D * sizeof(float);
  ZQ_NORM_BWD_DISPATCH(tpr, nc, <<<(unsigned)grid, kNormThreads, smem, stream>>>(
      gy, x, w, rstd, gh, dx, dw_part, M, D));
  *grid_out = grid;
  return cudaGetLastError();
}
}  // namespace zq

// dw_part: [G, D] fp32 partial sums; rows past the grid are zeroed, so the
// caller's sum over all G rows is the weight gradient.
void rmsnorm_bwd(at::Tensor gy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                 c10::optional<at::Tensor> gh, at::Tensor dx, at::Tensor dw_part) {
  check_bf16(gy, "gy");
  check_bf16(x, "x");
  check_bf16(dx, "dx");
  const int64_t D = x.size(-1), M = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= kNormMaxD, "D must be %8 and <= 8192");
  TORCH_CHECK(w.numel() == D && w.scalar_type() == at::kFloat && w.is_contiguous(),
              "norm weight must be fp32 [D]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, "norm weight: 16-byte alignment");
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
  if (M == 0) {
    dw_part.zero_();
    return;
  }
  int64_t grid = 0;
  C10_CUDA_CHECK(zq::launch_rmsnorm_bwd(cbf(gy), cbf(x), w.data_ptr<float>(), rstd.data_ptr<float>(),
                                    ghp, bf(dx), dw_part.data_ptr<float>(), M, (int)D,
                                    dw_part.size(0), at::cuda::getCurrentCUDAStream(), &grid));
  if (grid < dw_part.size(0)) dw_part.narrow(0, grid, dw_part.size(0) - grid).zero_();
}

namespace zq {
// out[c] += sum over rows r of part[r, c] (fp32, D % 4 == 0): each block sums
// 16 rows x 256 columns and adds them with one vector reduction per thread, so
// the partial rows of a norm backward fold into the gradient in one pass.
__global__ void __launch_bounds__(64) colsum_accum_kernel(const float4* __restrict__ part, int64_t rows,
                                                          int64_t d4, float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * 64 + threadIdx.x;
  if (c >= d4) return;
  const int64_t r0 = (int64_t)blockIdx.y * 16;
  const int64_t r1 = r0 + 16 < rows ? r0 + 16 : rows;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
  for (int64_t r = r0; r < r1; ++r) {
    const float4 v = __ldg(part + r * d4 + c);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  red_add_v4_f32(out + 4 * c, acc.x, acc.y, acc.z, acc.w);
}
}  // namespace zq

// out [D] fp32 += column sums of part [G, D] fp32 (both contiguous, D % 4 == 0).
void colsum_accum(at::Tensor part, at::Tensor out) {
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == at::kFloat && part.dim() == 2 && part.is_contiguous(),
              "colsum_accum: part must be contiguous fp32 [G, D]");
  const int64_t G = part.size(0), D = part.size(1);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == D &&
                  D % 4 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "colsum_accum: out must be 16-byte aligned contiguous fp32 [D], D % 4 == 0");
  if (G == 0 || D == 0) return;
  const at::cuda::CUDAGuard guard(part.device());
  const dim3 grid((unsigned)((D / 4 + 63) / 64), (unsigned)((G + 15) / 16));
  zq::colsum_accum_kernel<<<grid, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(part.data_ptr<float>()), G, D / 4, out.data_ptr<float>());
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
      (int)H, (int)D, (float)sign, H * D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// RoPE of x [B, S, H, D] written into the first H*D columns of the rows of
// out [B*S, >= H*D] (row pitch out.stride(0)): a slice of a wider buffer.
// rope_into for two (x, out) pairs in one launch (same positions and table)
void rope_into2(at::Tensor x1, at::Tensor out1, at::Tensor x2, at::Tensor out2, at::Tensor cs, double sign) {
  for (auto pr : {std::make_pair(&x1, &out1), std::make_pair(&x2, &out2)}) {
    const at::Tensor& x = *pr.first;
    const at::Tensor& out = *pr.second;
    check_bf16(x, "x");
    TORCH_CHECK(x.dim() == 4, "rope_into2: x must be [B, S, H, D]");
    TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 &&
                    out.size(0) == x.size(0) * x.size(1) && out.size(1) >= x.size(2) * x.size(3) &&
                    out.stride(1) == 1 && out.stride(0) % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
                "rope_into2: out must be bf16 [B*S, >= H*D] with 16-byte aligned rows");
  }
  const int64_t S = x1.size(1), D = x1.size(3);
  TORCH_CHECK(x2.size(1) == S && x2.size(3) == D && x2.size(0) == x1.size(0), "rope_into2: shapes");
  TORCH_CHECK(D % 16 == 0, "rope_into2: head dim must be a multiple of 16");
  TORCH_CHECK(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.numel() >= S * D,
              "rope_into2: cos/sin table must be fp32 [S, D/2, 2]");
  const at::cuda::CUDAGuard guard(x1.device());
  const int64_t rows1 = x1.size(0) * S * x1.size(2), rows2 = x2.size(0) * S * x2.size(2);
  const int64_t total = (rows1 + rows2) * (D / 16);
  rope2_kernel<<<(unsigned)((total + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(x1), reinterpret_cast<__nv_bfloat16*>(out1.data_ptr<at::BFloat16>()), rows1, (int)x1.size(2),
      out1.stride(0), cbf(x2), reinterpret_cast<__nv_bfloat16*>(out2.data_ptr<at::BFloat16>()), rows2,
      (int)x2.size(2), out2.stride(0), reinterpret_cast<const float2*>(cs.data_ptr<float>()), (int)S,
      (int)D, (float)sign);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_into(at::Tensor x, at::Tensor out, at::Tensor cs, double sign) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 4, "rope_into: x must be [B, S, H, D]");
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2), D = x.size(3);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 &&
                  out.size(0) == B * S && out.size(1) >= H * D && out.stride(1) == 1 &&
                  out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "rope_into: out must be bf16 [B*S, >= H*D] with 16-byte aligned rows");
  TORCH_CHECK(D % 16 == 0, "rope_into: head dim must be a multiple of 16");
  TORCH_CHECK(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.numel() >= S * D,
              "rope_into: cos/sin table must be fp32 [S, D/2, 2]");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t rows = B * S * H;
  const int64_t total = rows * (D / 16);
  rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(x), reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
      reinterpret_cast<const float2*>(cs.data_ptr<float>()), rows, (int)S, (int)H, (int)D,
      (float)sign, out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static inline unsigned ew_grid(int64_t n8) { return (unsigned)((n8 + 255) / 256); }

void gelu_fwd(at::Tensor x, at::Tensor y) {
  check_bf16(x, "x");
  check_bf16(y, "y");
  TORCH_CHECK(x.numel() % 8 == 0 && y.numel() == x.numel(), "gelu: numel % 8 and equal sizes");
  const int64_t n8 = x.numel() / 8;
  const at::cuda::CUDAGuard guard(x.device());
  gelu_fwd_kernel<<<ew_grid((n8 + kEwIlp - 1) / kEwIlp), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(x), bf(y), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_cdf_pdf(at::Tensor x, at::Tensor cdf, at::Tensor pdf) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() &&
                  cdf.sizes() == x.sizes() && pdf.sizes() == x.sizes() && cdf.is_contiguous() &&
                  pdf.is_contiguous() && cdf.scalar_type() == at::kFloat &&
                  pdf.scalar_type() == at::kFloat,
              "gelu_cdf_pdf: contiguous fp32 CUDA tensors of one shape");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t n = x.numel();
  if (n == 0) return;
  gelu_cdf_pdf_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), cdf.data_ptr<float>(), pdf.data_ptr<float>(), n);
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
  gelu_bwd_kernel<<<ew_grid((n8 + kEwIlp - 1) / kEwIlp), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(g), cbf(x), bf(dx), n8);
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
            c10::optional<at::Tensor> count, int64_t vocab, int64_t ignore_index, int64_t col0,
            int64_t vocab_total) {
  check_bf16(logits, "logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "targets int64");
  const int64_t M = logits.size(0), Vpad = logits.size(1);
  TORCH_CHECK(Vpad % 8 == 0 && vocab <= Vpad, "ce: Vpad % 8 and vocab <= Vpad");
  TORCH_CHECK(targets.numel() == M && loss.numel() >= M && lse.numel() >= M, "ce: one target per row");
  const at::cuda::CUDAGuard guard(logits.device());
  float* cnt = nullptr;
  if (count.has_value() && count->defined()) cnt = count->data_ptr<float>();
  if (vocab_total < 0) vocab_total = vocab;
  TORCH_CHECK(col0 >= 0 && col0 + vocab <= vocab_total, "ce: chunk outside the vocabulary");
  ce_fwd_kernel<<<(unsigned)M, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbf(logits), targets.data_ptr<int64_t>(), loss.data_ptr<float>(), lse.data_ptr<float>(),
      cnt, Vpad, vocab, ignore_index, col0, vocab_total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_bwd(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor scale,
            int64_t vocab, int64_t ignore_index, int64_t col0, int64_t vocab_total) {
  check_bf16(logits, "logits");
  const int64_t M = logits.size(0), Vpad = logits.size(1);
  TORCH_CHECK(Vpad % 8 == 0 && vocab <= Vpad && targets.numel() == M && lse.numel() >= M &&
                  targets.scalar_type() == at::kLong && scale.numel() >= 1,
              "ce_bwd: sizes");
  const at::cuda::CUDAGuard guard(logits.device());
  if (vocab_total < 0) vocab_total = vocab;
  TORCH_CHECK(col0 >= 0 && col0 + vocab <= vocab_total, "ce_bwd: chunk outside the vocabulary");
  ce_bwd_kernel<<<(unsigned)M, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bf(logits), targets.data_ptr<int64_t>(), lse.data_ptr<float>(), scale.data_ptr<float>(),
      Vpad, vocab, ignore_index, col0, vocab_total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v,
                c10::optional<at::Tensor> pbf16, double lr, double b1, double b2, double eps,
                double wd, double bc1, double bc2, double gscale, c10::optional<at::Tensor> bc,
                c10::optional<at::Tensor> clip_sq, double max_norm) {
  const float* bcp = nullptr;
  const float* sqp = nullptr;
  if (clip_sq.has_value() && clip_sq->defined()) {
    TORCH_CHECK(clip_sq->is_cuda() && clip_sq->scalar_type() == at::kFloat && clip_sq->numel() >= 1 &&
                    max_norm > 0.0, "adamw: clip_sq fp32[1] and a positive max_norm");
    sqp = clip_sq->data_ptr<float>();
  }
  if (bc.has_value() && bc->defined()) {
    TORCH_CHECK(bc->is_cuda() && bc->scalar_type() == at::kFloat && bc->numel() >= 2, "adamw: bc fp32[2]");
    bcp = bc->data_ptr<float>();
  }
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
        (float)eps, (float)wd, (float)bc1, (float)bc2, (float)gscale, bcp, sqp, (float)max_norm);
  } else {
    TORCH_CHECK(g.scalar_type() == at::kBFloat16, "adamw: grad fp32 or bf16");
    adamw_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p.data_ptr<float>(), cbf(g),
        m.data_ptr<float>(), v.data_ptr<float>(), pb, n, (float)lr, (float)b1, (float)b2,
        (float)eps, (float)wd, (float)bc1, (float)bc2, (float)gscale, bcp, sqp, (float)max_norm);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Device-side optimizer clock: clk = int64 [step, epoch], bc = fp32 [1 - b1^step,
// 1 - b2^step].  One thread advances the step (and the cross-rank epoch when
// bump_epoch) and recomputes the bias corrections in double precision, as the
// host does; kernels later on the stream read them, so a CUDA graph that
// captured this launch advances the optimizer on every replay.
__global__ void opt_tick_kernel(int64_t* clk, float* bc, double b1, double b2, int bump_epoch) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int64_t step = ++clk[0];
    if (bump_epoch) ++clk[1];
    bc[0] = (float)(1.0 - pow(b1, (double)step));
    bc[1] = (float)(1.0 - pow(b2, (double)step));
  }
}

void opt_tick(at::Tensor clk, at::Tensor bc, double b1, double b2, bool bump_epoch) {
  TORCH_CHECK(clk.is_cuda() && clk.scalar_type() == at::kLong && clk.numel() >= 2, "opt_tick: clk int64[2]");
  TORCH_CHECK(bc.is_cuda() && bc.scalar_type() == at::kFloat && bc.numel() >= 2, "opt_tick: bc fp32[2]");
  const at::cuda::CUDAGuard guard(clk.device());
  opt_tick_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(clk.data_ptr<int64_t>(), bc.data_ptr<float>(),
                                                                 b1, b2, bump_epoch ? 1 : 0);
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

// Blockwise 4-bit (NF4 / FP4) quantise and dequantise kernels.
//
// Layout (bitsandbytes-compatible): flat input, blocks of `blocksize` values,
// fp32 absmax per block, nearest code of x/absmax (ties to the lower code),
// two codes per byte with the even element in the high nibble.
//
// Quantise: each thread owns 8 consecutive values; the threads of one block
// (blocksize/8 of them) reduce absmax with warp shuffles (blocksize <= 256) or
// through shared memory (512..4096, one CTA per block).  The code index is the
// number of code midpoints strictly below x/absmax (NF4) or the sign bit plus
// the same count over the sorted FP4 magnitudes; midpoints are computed in fp32
// exactly like the PyTorch oracle, so the bytes match it bit for bit.
//
// Dequantise (memory-bound, used by the non-fused gather path and as an
// oracle): each thread expands 8 packed bytes into 16 outputs with the code
// table in shared memory.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace zq {

__constant__ float c_nf4_code[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

__constant__ float c_fp4_code[16] = {0.0f, 0.005208333333f, 0.66666667f, 1.0f, 0.33333333f,
                                     0.5f, 0.16666667f, 0.25f, -0.0f, -0.005208333333f,
                                     -0.66666667f, -1.0f, -0.33333333f, -0.5f, -0.16666667f,
                                     -0.25f};
// FP4 positive magnitudes sorted ascending and their code indices
__constant__ float c_fp4_sorted[8] = {0.0f, 0.005208333333f, 0.16666667f, 0.25f,
                                      0.33333333f, 0.5f, 0.66666667f, 1.0f};
__constant__ int c_fp4_sorted_idx[8] = {0, 1, 6, 7, 4, 5, 2, 3};

__device__ __forceinline__ uint32_t quant_nf4(float x) {
  uint32_t idx = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) {
    const float mid = (c_nf4_code[i] + c_nf4_code[i + 1]) * 0.5f;
    idx += (x > mid) ? 1u : 0u;
  }
  return idx;
}

__device__ __forceinline__ uint32_t quant_fp4(float x) {
  const float a = fabsf(x);
  int pos = 0;
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const float mid = (c_fp4_sorted[i] + c_fp4_sorted[i + 1]) * 0.5f;
    pos += (a > mid) ? 1 : 0;
  }
  uint32_t idx = (uint32_t)c_fp4_sorted_idx[pos];
  if (x < 0.0f) idx |= 8u;
  return idx;
}

template <typename T>
__device__ __forceinline__ void load8(const T* __restrict__ x, int64_t e0, int64_t n, float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = (e0 + j < n) ? to_f32<T>(x[e0 + j]) : 0.0f;
}

template <typename T>
__device__ __forceinline__ void quant_store8(const float (&v)[8], float inv, int qtype,
                                             uint8_t* __restrict__ packed, int64_t e0, int64_t n) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t e = e0 + 2 * j;
    if (e < n) {
      const float a = v[2 * j] * inv, b = v[2 * j + 1] * inv;
      const uint32_t qa = qtype == 0 ? quant_nf4(a) : quant_fp4(a);
      const uint32_t qb = qtype == 0 ? quant_nf4(b) : quant_fp4(b);
      packed[e >> 1] = (uint8_t)((qa << 4) | qb);
    }
  }
}

// blocksize <= 256: blocksize/8 lanes per quantisation block, all in one warp
template <typename T>
__global__ void nf4_quantize_small_kernel(const T* __restrict__ x, uint8_t* __restrict__ packed,
                                          float* __restrict__ absmax, int64_t n, int blocksize,
                                          int qtype) {
  const int tpb = blocksize >> 3;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nblocks = (n + blocksize - 1) / blocksize;
  const int64_t b = t / tpb;
  const int sub = (int)(t % tpb);
  const bool active = b < nblocks;
  const int64_t e0 = b * blocksize + (int64_t)sub * 8;
  float v[8];
  if (active) {
    load8<T>(x, e0, n, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.0f;
  }
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
  for (int o = tpb >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (!active) return;
  const float inv = m > 0.0f ? 1.0f / m : 0.0f;
  quant_store8<T>(v, inv, qtype, packed, e0, n);
  if (sub == 0) absmax[b] = m;
}

// blocksize 512..4096: one CTA (blocksize/8 threads) per quantisation block
template <typename T>
__global__ void nf4_quantize_large_kernel(const T* __restrict__ x, uint8_t* __restrict__ packed,
                                          float* __restrict__ absmax, int64_t n, int blocksize,
                                          int qtype) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  const int64_t e0 = b * blocksize + (int64_t)threadIdx.x * 8;
  float v[8];
  load8<T>(x, e0, n, v);
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
  m = warp_max(m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    float r = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    r = warp_max(r);
    if (lane == 0) red[0] = r;
  }
  __syncthreads();
  m = red[0];
  const float inv = m > 0.0f ? 1.0f / m : 0.0f;
  quant_store8<T>(v, inv, qtype, packed, e0, n);
  if (threadIdx.x == 0) absmax[b] = m;
}

template <typename T>
__global__ void nf4_dequantize_kernel(const uint8_t* __restrict__ packed,
                                      const float* __restrict__ absmax, T* __restrict__ out,
                                      int64_t n, int blocksize, int qtype) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = qtype == 0 ? c_nf4_code[threadIdx.x] : c_fp4_code[threadIdx.x];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t e0 = t * 16;
  if (e0 >= n) return;
  const float s = absmax[e0 / blocksize];
  if (e0 + 16 <= n && (reinterpret_cast<uintptr_t>(packed) & 7) == 0) {
    const uint2 p = *reinterpret_cast<const uint2*>(packed + (e0 >> 1));
    const uint32_t w[2] = {p.x, p.y};
    float v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFF;
      v[2 * i] = lut[byte >> 4] * s;
      v[2 * i + 1] = lut[byte & 0xF] * s;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) out[e0 + i] = from_f32<T>(v[i]);
  } else {
    for (int i = 0; i < 16 && e0 + i < n; ++i) {
      const int64_t e = e0 + i;
      const uint32_t byte = packed[e >> 1];
      const uint32_t q = (e & 1) ? (byte & 0xF) : (byte >> 4);
      out[e] = from_f32<T>(lut[q] * absmax[e / blocksize]);
    }
  }
}

}  // namespace zq

using namespace zq;

void nf4_quantize(at::Tensor x, at::Tensor packed, at::Tensor absmax, int64_t blocksize,
                  int64_t qtype) {
  TORCH_CHECK(x.is_cuda() && packed.is_cuda() && absmax.is_cuda(), "nf4_quantize: CUDA tensors");
  TORCH_CHECK(x.is_contiguous() && packed.is_contiguous() && absmax.is_contiguous(),
              "nf4_quantize: contiguous tensors");
  TORCH_CHECK(packed.scalar_type() == at::kByte && absmax.scalar_type() == at::kFloat,
              "nf4_quantize: packed uint8, absmax float32");
  TORCH_CHECK(blocksize >= 64 && blocksize <= 4096 && (blocksize & (blocksize - 1)) == 0,
              "nf4_quantize: blocksize must be a power of two in [64, 4096]");
  const int64_t n = x.numel();
  const int64_t nb = (n + blocksize - 1) / blocksize;
  TORCH_CHECK(packed.numel() >= (n + 1) / 2 && absmax.numel() >= nb, "nf4_quantize: outputs too small");
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto launch = [&](auto* xp) {
    using T = std::remove_pointer_t<decltype(xp)>;
    if (blocksize <= 256) {
      const int64_t threads = nb * (blocksize / 8);
      const int bs = 256;
      nf4_quantize_small_kernel<T><<<(unsigned)((threads + bs - 1) / bs), bs, 0, stream>>>(
          xp, packed.data_ptr<uint8_t>(), absmax.data_ptr<float>(), n, (int)blocksize, (int)qtype);
    } else {
      nf4_quantize_large_kernel<T><<<(unsigned)nb, (unsigned)(blocksize / 8), 0, stream>>>(
          xp, packed.data_ptr<uint8_t>(), absmax.data_ptr<float>(), n, (int)blocksize, (int)qtype);
    }
  };
  switch (x.scalar_type()) {
    case at::kFloat: launch(x.data_ptr<float>()); break;
    case at::kHalf: launch(reinterpret_cast<__half*>(x.data_ptr<at::Half>())); break;
    case at::kBFloat16: launch(reinterpret_cast<__nv_bfloat16*>(x.data_ptr<at::BFloat16>())); break;
    default: TORCH_CHECK(false, "nf4_quantize: float32/float16/bfloat16 input");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void nf4_dequantize(at::Tensor packed, at::Tensor absmax, at::Tensor out, int64_t n,
                    int64_t blocksize, int64_t qtype) {
  TORCH_CHECK(packed.is_cuda() && absmax.is_cuda() && out.is_cuda(), "nf4_dequantize: CUDA tensors");
  TORCH_CHECK(packed.scalar_type() == at::kByte && absmax.scalar_type() == at::kFloat,
              "nf4_dequantize: packed uint8, absmax float32");
  TORCH_CHECK(out.is_contiguous() && out.numel() >= n, "nf4_dequantize: output too small");
  TORCH_CHECK(packed.numel() >= (n + 1) / 2 && absmax.numel() >= (n + blocksize - 1) / blocksize,
              "nf4_dequantize: inputs too small");
  TORCH_CHECK(blocksize >= 16, "nf4_dequantize: blocksize >= 16");
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t threads = (n + 15) / 16;
  const int bs = 256;
  const unsigned grid = (unsigned)((threads + bs - 1) / bs);
  switch (out.scalar_type()) {
    case at::kFloat:
      nf4_dequantize_kernel<float><<<grid, bs, 0, stream>>>(packed.data_ptr<uint8_t>(),
          absmax.data_ptr<float>(), out.data_ptr<float>(), n, (int)blocksize, (int)qtype);
      break;
    case at::kHalf:
      nf4_dequantize_kernel<__half><<<grid, bs, 0, stream>>>(packed.data_ptr<uint8_t>(),
          absmax.data_ptr<float>(), reinterpret_cast<__half*>(out.data_ptr<at::Half>()), n,
          (int)blocksize, (int)qtype);
      break;
    case at::kBFloat16:
      nf4_dequantize_kernel<__nv_bfloat16><<<grid, bs, 0, stream>>>(packed.data_ptr<uint8_t>(),
          absmax.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
          n, (int)blocksize, (int)qtype);
      break;
    default: TORCH_CHECK(false, "nf4_dequantize: float32/float16/bfloat16 output");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

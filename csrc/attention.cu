// Causal / GQA flash attention, forward and backward, bf16 in, fp32 softmax.
//
// Layout: q [B,S,Hq,D], k/v [B,S,Hk,D], o [B,S,Hq,D] (the projection layout, no
// transposes), lse [B,Hq,S] (natural log).  D in {64, 128}; S % 128 == 0.
//
// Forward: one CTA per (128-query block, head), 8 warps x 16 query rows.  K/V
// tiles of 64 keys are double-buffered in shared memory with cp.async (16-byte
// chunks XOR-swizzled by row so ldmatrix is conflict-free).  Scores and
// P·V use the bf16 m16n8k16 tensor-core MMA with fp32 accumulation; the softmax
// is the online (running max / running sum) form in base 2.
//
// Backward: one CTA per (64-key block, KV head), 4 warps x 16 keys.  For every
// query block at or after the key block (and every query head of the GQA group)
// it recomputes Pᵀ = exp(K Qᵀ - lse), accumulates dV += Pᵀ dO and
// dK += dSᵀ Q in registers (dS = P ∘ (dP - delta), dPᵀ = V dOᵀ), and adds
// dQ += dS K into an fp32 buffer with atomics.  delta = rowsum(dO ∘ O) comes
// from a small pre-pass; a post-pass scales and converts dQ.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace zq {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// byte offset of (row, 8-element chunk) in a swizzled [rows][D] bf16 tile
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

// async copy of `rows` rows of D bf16 (global row pitch `ld` elements) into a swizzled tile
template <int D, int NT>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, int64_t ld, int rows) {
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < rows * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    cp_async16(sbase + swz<D>(r, c), g + (int64_t)r * ld + c * 8);
  }
}

constexpr float kLog2e = 1.4426950408889634f;

// ----------------------------------------------------------------------------
// forward
// ----------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256, 1)
attn_fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                const __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ o,
                float* __restrict__ lse, int S, int Hq, int Hk, float scale, int causal) {
  constexpr int BM = 128, BN = 64, NT = 256;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + BM * D * 2;
  const uint32_t sV = sK + 2 * BN * D * 2;

  const int nqb = S / BM;
  const int qb = nqb - 1 - (int)blockIdx.x;  // heavy (late) blocks first
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hk);
  const int q0 = qb * BM;
  const int64_t ldq = (int64_t)Hq * D, ldk = (int64_t)Hk * D;
  const __nv_bfloat16* qg = q + ((int64_t)b * S + q0) * ldq + (int64_t)h * D;
  const __nv_bfloat16* kg = k + (int64_t)b * S * ldk + (int64_t)hk * D;
  const __nv_bfloat16* vg = v + (int64_t)b * S * ldk + (int64_t)hk * D;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nkb = causal ? (q0 + BM) / BN : S / BN;

  load_tile<D, NT>(sQ, qg, ldq, BM);
  load_tile<D, NT>(sK, kg, ldk, BN);
  load_tile<D, NT>(sV, vg, ldk, BN);
  cp_async_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  uint32_t qf[D / 16][4];
  const float sl2 = scale * kLog2e;
  const int row0 = q0 + warp * 16 + g;  // query index of this thread's first row

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<D, NT>(sK + (buf ^ 1) * BN * D * 2, kg + (int64_t)(j + 1) * BN * ldk, ldk, BN);
      load_tile<D, NT>(sV + (buf ^ 1) * BN * D * 2, vg + (int64_t)(j + 1) * BN * ldk, ldk, BN);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kd = 0; kd < D / 16; ++kd) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kd * 2 + (lane >> 4);
        ldsm_x4(sQ + swz<D>(r, c), qf[kd][0], qf[kd][1], qf[kd][2], qf[kd][3]);
      }
    }
    const uint32_t kb = sK + buf * BN * D * 2, vb = sV + buf * BN * D * 2;
    const int k0 = j * BN;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
    const bool warp_active = !causal || (k0 <= q0 + warp * 16 + 15);
    if (warp_active) {
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
#pragma unroll
        for (int kd = 0; kd < D / 16; ++kd) {
          uint32_t b0, b1, b2, b3;
          const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = kd * 2 + ((lane >> 3) & 1);
          ldsm_x4(kb + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(s[2 * n2], qf[kd], b0, b1);
          mma_bf16_16816(s[2 * n2 + 1], qf[kd], b2, b3);
        }
      }
      // scale, mask, online softmax (rows g and g+8 of this warp)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + n * 8 + 2 * t + (e & 1);
          const int qi = row0 + (e >> 1) * 8;
          float x = s[n][e] * sl2;
          if (causal && key > qi) x = -INFINITY;
          s[n][e] = x;
        }
        mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
        mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
      const float c0 = (m0 == -INFINITY) ? 0.0f : exp2f(m0 - nm0);
      const float c1 = (m1 == -INFINITY) ? 0.0f : exp2f(m1 - nm1);
      m0 = nm0;
      m1 = nm1;
      float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][0] = (nm0 == -INFINITY) ? 0.0f : exp2f(s[n][0] - nm0);
        s[n][1] = (nm0 == -INFINITY) ? 0.0f : exp2f(s[n][1] - nm0);
        s[n][2] = (nm1 == -INFINITY) ? 0.0f : exp2f(s[n][2] - nm1);
        s[n][3] = (nm1 == -INFINITY) ? 0.0f : exp2f(s[n][3] - nm1);
        rs0 += s[n][0] + s[n][1];
        rs1 += s[n][2] + s[n][3];
      }
      l0 = l0 * c0 + rs0;
      l1 = l1 * c1 + rs1;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        acc[i][0] *= c0;
        acc[i][1] *= c0;
        acc[i][2] *= c1;
        acc[i][3] *= c1;
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int d2 = 0; d2 < D / 16; ++d2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = d2 * 2 + (lane >> 4);
          ldsm_x4_t(vb + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * d2], pa, b0, b1);
          mma_bf16_16816(acc[2 * d2 + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  // finalize
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f;
  const float inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  __nv_bfloat16* og = o + ((int64_t)b * S + row0) * ldq + (int64_t)h * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int col = i * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(og + col) = pack_bf16x2(acc[i][0] * inv0, acc[i][1] * inv0);
    *reinterpret_cast<uint32_t*>(og + 8 * ldq + col) = pack_bf16x2(acc[i][2] * inv1, acc[i][3] * inv1);
  }
  if (t == 0) {
    float* lrow = lse + ((int64_t)b * Hq + h) * S;
    lrow[row0] = m0 / kLog2e + logf(l0);
    lrow[row0 + 8] = m1 / kLog2e + logf(l1);
  }
}

// ----------------------------------------------------------------------------
// backward
// ----------------------------------------------------------------------------
// delta[b,h,s] = sum_d dO*O ;  dq_acc = 0
template <int D>
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o,
                                    float* __restrict__ delta, float* __restrict__ dq_acc, int B, int S,
                                    int Hq) {
  // one warp per (b, s, h) row
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * S * Hq) return;
  const int h = (int)(row % Hq);
  const int64_t bs = row / Hq;
  const int s = (int)(bs % S), b = (int)(bs / S);
  float acc = 0.0f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dout + row * D + d));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + row * D + d));
    acc += x.x * y.x + x.y * y.y;
    *reinterpret_cast<float2*>(dq_acc + row * D + d) = make_float2(0.0f, 0.0f);
  }
  acc = warp_sum(acc);
  if (lane == 0) delta[((int64_t)b * Hq + h) * S + s] = acc;
}

template <int D>
__global__ void attn_bwd_post_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq,
                                     int64_t n, float scale) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const float2 v = *reinterpret_cast<const float2*>(dq_acc + i);
  *reinterpret_cast<uint32_t*>(dq + i) = pack_bf16x2(v.x * scale, v.y * scale);
}

template <int D>
__global__ void __launch_bounds__(128, 1)
attn_bwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ dout,
                const float* __restrict__ lse, const float* __restrict__ delta,
                float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                int S, int Hq, int Hk, float scale, int causal) {
  constexpr int BN = 64, BM = 64, NT = 128;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BN * D * 2;
  const uint32_t sQ = sV + BN * D * 2;
  const uint32_t sdO = sQ + BM * D * 2;
  const uint32_t sdS = sdO + BM * D * 2;      // [64 keys][64 queries] bf16, swizzled
  float* sL = reinterpret_cast<float*>(smem + (2 * BN + 2 * BM) * D * 2 + BN * BM * 2);
  float* sDelta = sL + BM;

  const int kb = blockIdx.x;
  const int b = blockIdx.y / Hk, hk = blockIdx.y % Hk;
  const int rep = Hq / Hk;
  const int k0 = kb * BN;
  const int64_t ldq = (int64_t)Hq * D, ldk = (int64_t)Hk * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const float sl2 = scale * kLog2e;

  load_tile<D, NT>(sK, k + ((int64_t)b * S + k0) * ldk + (int64_t)hk * D, ldk, BN);
  load_tile<D, NT>(sV, v + ((int64_t)b * S + k0) * ldk + (int64_t)hk * D, ldk, BN);
  cp_async_commit();

  float dka[D / 8][4], dva[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    dka[i][0] = dka[i][1] = dka[i][2] = dka[i][3] = 0.0f;
    dva[i][0] = dva[i][1] = dva[i][2] = dva[i][3] = 0.0f;
  }
  const int key0 = k0 + warp * 16 + g;  // this thread's first key (rows g, g+8 of the warp tile)
  const int nqb = S / BM;
  const int qb_start = causal ? k0 / BM : 0;

  for (int hh = 0; hh < rep; ++hh) {
    const int h = hk * rep + hh;
    for (int qb = qb_start; qb < nqb; ++qb) {
      const int q0 = qb * BM;
      __syncthreads();  // previous iteration done with sQ/sdO/sdS
      load_tile<D, NT>(sQ, q + ((int64_t)b * S + q0) * ldq + (int64_t)h * D, ldq, BM);
      load_tile<D, NT>(sdO, dout + ((int64_t)b * S + q0) * ldq + (int64_t)h * D, ldq, BM);
      cp_async_commit();
      if (threadIdx.x < BM) {
        sL[threadIdx.x] = lse[((int64_t)b * Hq + h) * S + q0 + threadIdx.x] * kLog2e;
        sDelta[threadIdx.x] = delta[((int64_t)b * Hq + h) * S + q0 + threadIdx.x];
      }
      cp_async_wait<0>();
      __syncthreads();

      // S^T = K_w Q^T  (16 keys x 64 queries)
      float st[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.0f;
#pragma unroll
      for (int kd = 0; kd < D / 16; ++kd) {
        uint32_t a[4];
        {
          const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = kd * 2 + (lane >> 4);
          ldsm_x4(sK + swz<D>(r, c), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t b0, b1, b2, b3;
          const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = kd * 2 + ((lane >> 3) & 1);
          ldsm_x4(sQ + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(st[2 * n2], a, b0, b1);
          mma_bf16_16816(st[2 * n2 + 1], a, b2, b3);
        }
      }
      // P^T = exp2(S^T*scale*log2e - lse2[query]), causal mask key > query
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi_l = n * 8 + 2 * t + (e & 1);
          const int key = key0 + (e >> 1) * 8;
          float p = exp2f(st[n][e] * sl2 - sL[qi_l]);
          if (causal && key > q0 + qi_l) p = 0.0f;
          st[n][e] = p;
        }
      }
      // dV += P^T dO
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
        pa[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
        pa[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
        for (int d2 = 0; d2 < D / 16; ++d2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = d2 * 2 + (lane >> 4);
          ldsm_x4_t(sdO + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(dva[2 * d2], pa, b0, b1);
          mma_bf16_16816(dva[2 * d2 + 1], pa, b2, b3);
        }
      }
      // dP^T = V_w dO^T
      float dpt[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.0f;
#pragma unroll
      for (int kd = 0; kd < D / 16; ++kd) {
        uint32_t a[4];
        {
          const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = kd * 2 + (lane >> 4);
          ldsm_x4(sV + swz<D>(r, c), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t b0, b1, b2, b3;
          const int r = n2 * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = kd * 2 + ((lane >> 3) & 1);
          ldsm_x4(sdO + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(dpt[2 * n2], a, b0, b1);
          mma_bf16_16816(dpt[2 * n2 + 1], a, b2, b3);
        }
      }
      // dS^T = P^T * (dP^T - delta[query]); stash dS^T (bf16) in shared memory
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi_l = n * 8 + 2 * t + (e & 1);
          st[n][e] = st[n][e] * (dpt[n][e] - sDelta[qi_l]);
        }
        const int kr = warp * 16 + g;
        const int qc = n * 8 + 2 * t;
        const uint32_t a0 = sdS + (uint32_t)(kr * 128 + (((qc >> 3) ^ (kr & 7)) << 4) + (qc & 7) * 2);
        const uint32_t a1 = sdS + (uint32_t)((kr + 8) * 128 + (((qc >> 3) ^ ((kr + 8) & 7)) << 4) + (qc & 7) * 2);
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(a0), "r"(pack_bf16x2(st[n][0], st[n][1])));
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(a1), "r"(pack_bf16x2(st[n][2], st[n][3])));
      }
      // dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
        pa[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
        pa[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
        for (int d2 = 0; d2 < D / 16; ++d2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = d2 * 2 + (lane >> 4);
          ldsm_x4_t(sQ + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16_16816(dka[2 * d2], pa, b0, b1);
          mma_bf16_16816(dka[2 * d2 + 1], pa, b2, b3);
        }
      }
      __syncthreads();  // dS^T complete
      // dQ[16 queries of this warp] += dS K  (A = dS from dS^T via ldmatrix.trans)
      {
        float dqa[D / 8][4];
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t a[4];
          {
            const int kr = kk * 16 + (lane & 7) + (lane >> 4) * 8;          // key (stored row)
            const int qc = warp * 16 + ((lane >> 3) & 1) * 8;              // query (stored col)
            ldsm_x4_t(sdS + (uint32_t)(kr * 128 + (((qc >> 3) ^ (kr & 7)) << 4)), a[0], a[1], a[2], a[3]);
          }
#pragma unroll
          for (int d2 = 0; d2 < D / 16; ++d2) {
            uint32_t b0, b1, b2, b3;
            const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int c = d2 * 2 + (lane >> 4);
            ldsm_x4_t(sK + swz<D>(r, c), b0, b1, b2, b3);
            mma_bf16_16816(dqa[2 * d2], a, b0, b1);
            mma_bf16_16816(dqa[2 * d2 + 1], a, b2, b3);
          }
        }
        float* dqg = dq_acc + ((int64_t)b * S + q0 + warp * 16 + g) * ldq + (int64_t)h * D;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
          const int col = i * 8 + 2 * t;
          atomicAdd(dqg + col, dqa[i][0]);
          atomicAdd(dqg + col + 1, dqa[i][1]);
          atomicAdd(dqg + 8 * ldq + col, dqa[i][2]);
          atomicAdd(dqg + 8 * ldq + col + 1, dqa[i][3]);
        }
      }
    }
  }
  // write dK (scaled) and dV for this key block
  __nv_bfloat16* dkg = dk + ((int64_t)b * S + key0) * ldk + (int64_t)hk * D;
  __nv_bfloat16* dvg = dv + ((int64_t)b * S + key0) * ldk + (int64_t)hk * D;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int col = i * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(dkg + col) = pack_bf16x2(dka[i][0] * scale, dka[i][1] * scale);
    *reinterpret_cast<uint32_t*>(dkg + 8 * ldk + col) = pack_bf16x2(dka[i][2] * scale, dka[i][3] * scale);
    *reinterpret_cast<uint32_t*>(dvg + col) = pack_bf16x2(dva[i][0], dva[i][1]);
    *reinterpret_cast<uint32_t*>(dvg + 8 * ldk + col) = pack_bf16x2(dva[i][2], dva[i][3]);
  }
}

}  // namespace zq

using namespace zq;

static void check_qkv(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.dim() == 4,
              name, ": contiguous CUDA bf16 [B,S,H,D]");
}

template <int D>
static void fwd_impl(at::Tensor& q, at::Tensor& k, at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                     bool causal, double scale) {
  const int B = (int)q.size(0), S = (int)q.size(1), Hq = (int)q.size(2), Hk = (int)k.size(2);
  const int smem = (128 + 4 * 64) * D * 2;
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  dim3 grid(S / 128, B * Hq);
  attn_fwd_kernel<D><<<grid, 256, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr<at::BFloat16>()),
      reinterpret_cast<__nv_bfloat16*>(o.data_ptr<at::BFloat16>()), lse.data_ptr<float>(), S, Hq, Hk,
      (float)scale, causal ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, bool causal,
              double scale) {
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_qkv(o, "o");
  const int64_t S = q.size(1), D = q.size(3), Hq = q.size(2), Hk = k.size(2);
  TORCH_CHECK(S % 128 == 0, "attention: S must be a multiple of 128");
  TORCH_CHECK(Hq % Hk == 0, "attention: Hq must be a multiple of Hk");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(1) == S && k.size(3) == D, "attention: k/v shape");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == q.size(0) * Hq * S, "attention: lse");
  const at::cuda::CUDAGuard guard(q.device());
  if (D == 128) fwd_impl<128>(q, k, v, o, lse, causal, scale);
  else if (D == 64) fwd_impl<64>(q, k, v, o, lse, causal, scale);
  else TORCH_CHECK(false, "attention: head dim 64 or 128");
}

template <int D>
static void bwd_impl(at::Tensor& dout, at::Tensor& q, at::Tensor& k, at::Tensor& v, at::Tensor& o,
                     at::Tensor& lse, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, bool causal,
                     double scale) {
  const int B = (int)q.size(0), S = (int)q.size(1), Hq = (int)q.size(2), Hk = (int)k.size(2);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto delta = at::empty({B, Hq, S}, q.options().dtype(at::kFloat));
  auto dq_acc = at::empty(q.sizes(), q.options().dtype(at::kFloat));
  const int64_t rows = (int64_t)B * S * Hq;
  attn_bwd_pre_kernel<D><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(o.data_ptr<at::BFloat16>()), delta.data_ptr<float>(),
      dq_acc.data_ptr<float>(), B, S, Hq);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int smem = 4 * 64 * D * 2 + 64 * 64 * 2 + 2 * 64 * 4;
  static bool configured[64] = {false};
  const int dev = q.get_device();
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  dim3 grid(S / 64, B * Hk);
  attn_bwd_kernel<D><<<grid, 128, smem, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(v.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr<at::BFloat16>()), lse.data_ptr<float>(),
      delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dk.data_ptr<at::BFloat16>()),
      reinterpret_cast<__nv_bfloat16*>(dv.data_ptr<at::BFloat16>()), S, Hq, Hk, (float)scale, causal ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t n = q.numel();
  attn_bwd_post_kernel<D><<<(unsigned)((n / 2 + 255) / 256), 256, 0, stream>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr<at::BFloat16>()), n, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
              at::Tensor dq, at::Tensor dk, at::Tensor dv, bool causal, double scale) {
  check_qkv(dout, "dout");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_qkv(o, "o");
  check_qkv(dq, "dq");
  check_qkv(dk, "dk");
  check_qkv(dv, "dv");
  const int64_t S = q.size(1), D = q.size(3);
  TORCH_CHECK(S % 128 == 0, "attention: S must be a multiple of 128");
  const at::cuda::CUDAGuard guard(q.device());
  if (D == 128) bwd_impl<128>(dout, q, k, v, o, lse, dq, dk, dv, causal, scale);
  else if (D == 64) bwd_impl<64>(dout, q, k, v, o, lse, dq, dk, dv, causal, scale);
  else TORCH_CHECK(false, "attention: head dim 64 or 128");
}

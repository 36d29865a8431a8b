// LoRA adapter products on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// A LoRA adapter on a frozen projection y = x Wᵀ adds s·(x Aᵀ) Bᵀ with A [r, in]
// and B [out, r], r small (16 or 64).  Besides the main GEMMs (which take the
// rank-space products as an extra K slab, csrc/gemm_sm100.cu), training needs
// four skinny products per projection, all memory-bound (they read one
// activation-sized operand once and do r multiply-adds per element):
//
//   U  = x  · (sA)ᵀ      [T, r]   forward        (lora_down)
//   V  = dY · B          [T, r]   backward       (lora_down, W = Bᵀ)
//   dA += s · Vᵀ · x     [r, in]  backward       (lora_wgrad, transposed store)
//   dB += dYᵀ · U        [out, r] backward       (lora_wgrad)
//
// The reference runs these through PEFT's nn.Linear adapters on cuBLAS
// (examples/train_32b_maxwell.py:345-354).  Here:
//
// lora_down: one CTA per 128 rows of P and per K-range; a cluster of CS CTAs
//   splits K, each CTA streams its 128 x 64 P tiles and the matching rows of
//   W through a TMA ring into tcgen05.mma (M = 128, N = nq = the packed rank
//   width, accumulator in TMEM), then the CTAs of the cluster add their partial
//   accumulators through distributed shared memory (ld.shared::cluster) and
//   write the bf16 result twice: row-major [T, upad] zero-padded to the 64-wide
//   slab the main GEMM reads, and transposed [nq, T] (the K-major operand the
//   weight-gradient kernel reads).  P is read exactly once.
// lora_wgrad: the contraction over tokens.  Each CTA owns 128 columns of P and
//   a range of tokens; P tiles are read MN-major (two 64-column TMA boxes per
//   64-token stage, instruction-descriptor A-transpose bit), the rank-space
//   operand K-major from the transposed copy, and the fp32 partial sums are
//   added into the gradient with red.global.add (no separate reduction pass;
//   the summation order over token ranges is not fixed, so results can differ
//   in the last bits from run to run).  Up to four jobs share one launch
//   (column range of P, rows of the rank operand, output groups), which lets
//   the fused q/k/v projection form its three dA in one pass over x and its
//   three dB in one launch.
//
// All mbarrier waits are bounded (common.cuh); a timeout records an error code
// in the device status word read by gemm_status(), the kernel drains its copies
// in flight, frees TMEM and returns.  Every TMA load targets this CTA only.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <vector>

#include "common.cuh"

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn();
zq::DeviceStatus* status_buffer(int device);

namespace zq {

enum LoraErr { kLoraErrProducer = 131, kLoraErrMma = 132, kLoraErrEpi = 133 };

constexpr int kLoraThreads = 128;   // 4 warps: all read TMEM in the epilogue
constexpr int kLoraMaxStages = 8;  // ring depth is a launch argument (<= 8)
constexpr int kLoraTileBytes = 128 * 64 * 2;  // 128 rows x 64 bf16 (or two MN boxes)
constexpr int kLoraMaxJobs = 4;
constexpr int kLoraMaxGroups = 4;

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

// 32 lanes x 16 columns of 32-bit values (thread i: row lane-base + i)
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ uint32_t tmem_cols_for(int nq) {
  uint32_t c = 32;
  while ((int)c < nq) c <<= 1;
  return c;
}

// Wait (bounded, no status) until the last `inflight` TMA loads of the ring
// landed, so no copy targets this CTA's shared memory after it exits.  Loads
// older than those were consumed by the MMA before a newer one was issued.
__device__ __forceinline__ void drain_loads(uint64_t* full_bar, int issued, int stages) {
  const int first = issued > stages ? issued - stages : 0;
  for (int i = first; i < issued; ++i)
    mbar_wait(&full_bar[i % stages], (uint32_t)((i / stages) & 1), nullptr, 0);
}

// global fp32 [gdst, gdst + bytes) += shared fp32 [ssrc, ...): one bulk async
// reduction (both addresses 16-byte aligned, bytes a multiple of 16)
__device__ __forceinline__ void bulk_reduce_add_f32(float* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// Rows [r0, r1) of a 128-row tile: sum the fp32 partials [128][pld] of the CS
// CTAs of this cluster (read through distributed shared memory, all CS loads
// of an item in flight together), round to bf16 and store row-major into
// u [T, upad] (zero past nq) and, if ut != null, transposed into ut [nq, T].
template <int CS>
__device__ __forceinline__ void cluster_reduce_store(uint32_t part_addr, int pld, int nq, int upad, int r0,
                                                     int r1, int t_base, int T, __nv_bfloat16* u,
                                                     int64_t ldu, __nv_bfloat16* ut, int64_t ldt) {
  const int nr = r1 - r0;
  if (nr <= 0) return;
  const int items = nr * (upad / 8);
  for (int it = threadIdx.x; it < items; it += kLoraThreads) {
    const int rr = r0 + it % nr;
    const int col = (it / nr) * 8;
    const int t = t_base + rr;
    if (t >= T) continue;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    if (col < nq) {
      const uint32_t off = part_addr + (uint32_t)((rr * pld + col) * 4);
      float4 lo[CS], hi[CS];
#pragma unroll
      for (int q = 0; q < CS; ++q) {
        const uint32_t a = map_to_cta(off, (uint32_t)q);
        lo[q] = ld_dsmem_f4(a);
        hi[q] = ld_dsmem_f4(a + 16);
      }
#pragma unroll
      for (int q = 0; q < CS; ++q) {
        acc[0] += lo[q].x; acc[1] += lo[q].y; acc[2] += lo[q].z; acc[3] += lo[q].w;
        acc[4] += hi[q].x; acc[5] += hi[q].y; acc[6] += hi[q].z; acc[7] += hi[q].w;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(u + (int64_t)t * ldu + col) = o;
    if (ut != nullptr && col < nq) {
      const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) ut[(int64_t)(col + e) * ldt + t] = ob[e];
    }
  }
}

__device__ __forceinline__ void cluster_reduce_store_any(uint32_t csize, uint32_t part_addr, int pld, int nq,
                                                         int upad, int r0, int r1, int t_base, int T,
                                                         __nv_bfloat16* u, int64_t ldu, __nv_bfloat16* ut,
                                                         int64_t ldt) {
  switch (csize) {
    case 1: cluster_reduce_store<1>(part_addr, pld, nq, upad, r0, r1, t_base, T, u, ldu, ut, ldt); break;
    case 2: cluster_reduce_store<2>(part_addr, pld, nq, upad, r0, r1, t_base, T, u, ldu, ut, ldt); break;
    case 4: cluster_reduce_store<4>(part_addr, pld, nq, upad, r0, r1, t_base, T, u, ldu, ut, ldt); break;
    default: cluster_reduce_store<8>(part_addr, pld, nq, upad, r0, r1, t_base, T, u, ldu, ut, ldt); break;
  }
}

// ----------------------------------------------------------------------------
// lora_down: out[t, j] = sum_k P[t, k] * W[j, k]   (j < nq), bf16 in / bf16 out
// ----------------------------------------------------------------------------
struct LoraDownArgs {
  int T, K, nq;
  __nv_bfloat16* u;   // [T, upad] row-major, row stride ldu
  int64_t ldu;
  int upad;
  __nv_bfloat16* ut;  // [nq, T] row-major, row stride ldt (may be null)
  int64_t ldt;
  int stages;         // ring depth
  int kb;             // 64-wide K boxes per stage
  DeviceStatus* status;
};

__global__ void __launch_bounds__(kLoraThreads, 2)
lora_down_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmW,
                 LoraDownArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nq = args.nq;
  const int S = args.stages, KB = args.kb;
  const int w_bytes = nq * 128;
  // stage: KB boxes of P (128 rows x 64 K each), then KB boxes of W (nq x 64)
  const int stage_bytes = KB * (kLoraTileBytes + w_bytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  float* part = reinterpret_cast<float*>(smem);  // [128][nq + 4] after the MMAs finished
  const int pld = nq + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const int mt = (int)(blockIdx.x / csize);
  const int KT = (args.K + 64 * KB - 1) / (64 * KB);
  const int kt0 = (int)(((int64_t)crank * KT) / csize);
  const int kt1 = (int)(((int64_t)(crank + 1) * KT) / csize);
  const int nk = kt1 - kt0;
  const uint32_t tcols = tmem_cols_for(nq);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmP);
    prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&empty_bar[s], (uint32_t)(((i / S) & 1) ^ 1), args.status, kLoraErrProducer))
        break;
      uint8_t* sa = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full_bar[s], (uint32_t)stage_bytes);
      for (int b = 0; b < KB; ++b) {
        const int kc = ((kt0 + i) * KB + b) * 64;
        tma_load_2d(sa + b * kLoraTileBytes, &tmP, &full_bar[s], kc, mt * 128);
        tma_load_2d(sa + KB * kLoraTileBytes + b * w_bytes, &tmW, &full_bar[s], kc, 0);
      }
      ++issued;
    }
    drain_loads(full_bar, issued, S);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = umma_idesc_bf16(128, nq);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full_bar[s], (uint32_t)((i / S) & 1), args.status, kLoraErrMma)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
      const uint32_t b_addr = a_addr + KB * kLoraTileBytes;
      for (int b = 0; b < KB; ++b) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16_ss(tmem_base, umma_desc_sw128_kmajor(a_addr + b * kLoraTileBytes + kk * 32),
                      umma_desc_sw128_kmajor(b_addr + b * w_bytes + kk * 32), idesc,
                      (i > 0 || b > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&empty_bar[s]);
    }
    umma_commit(done_bar);  // also on an early exit: completes once issued MMAs finished
  }
  __syncwarp();

  // ------------------------------------------------------------ partial -> smem
  // (every TMA load was consumed by an MMA that completed before done_bar, so
  // the ring's shared memory is free for the partial sums)
  const bool have = nk > 0 && mbar_wait(done_bar, 0, args.status, kLoraErrEpi);
  tc_fence_after();
  const int row = warp * 32 + lane;
  float* prow = part + row * pld;
  for (int c = 0; c < nq; c += 16) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
    tmem_ld_wait();
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float4 o = have ? make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(prow + c + 4 * v) = o;
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every CTA's partial is visible cluster-wide

  // ------------------------------------------------------------ cluster reduction
  // This CTA finishes rows [r0, r1) of the tile: sums the cluster's partials,
  // writes bf16 row-major (zero padding up to upad) and transposed.
  {
    const int rows_per = (128 + (int)csize - 1) / (int)csize;
    const int r0 = (int)crank * rows_per;
    cluster_reduce_store_any(csize, smem_u32(part), pld, nq, args.upad, r0, min(128, r0 + rows_per),
                             mt * 128, args.T, args.u, args.ldu, args.ut, args.ldt);
  }
  cluster_sync_all();  // no CTA leaves while another still reads its partial

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

// ----------------------------------------------------------------------------
// lora_wgrad: out_g[...] += alpha * sum_t P[t, i] * Qt[q_row + j, t]
// ----------------------------------------------------------------------------
struct LoraWgradJob {
  int i_begin;   // first column of P (multiple of 64)
  int i_count;   // columns of P in this job
  int q_row;     // first row of Qt
  int tile0;     // first flattened tile index of this job
  float alpha;
  float* out[kLoraMaxGroups];  // one fp32 output per group of gsz rank columns
};

struct LoraWgradArgs {
  int T, nq, gsz, rvalid, njobs, tsplit;
  int stages;  // ring depth
  int kb;      // 64-token blocks per stage
  int64_t ld_out;
  int transposed;  // 1: out[jj * ld_out + i] (dA layout), 0: out[i * ld_out + jj] (dB layout)
  LoraWgradJob jobs[kLoraMaxJobs];
  DeviceStatus* status;
};

__global__ void __launch_bounds__(kLoraThreads, 2)
lora_wgrad_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                  const __grid_constant__ LoraWgradArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nq = args.nq;
  const int S = args.stages, KB = args.kb;
  const int q_bytes = nq * 128;
  // stage: KB blocks of 64 tokens of P (two MN-major 64-column boxes each), then
  // KB boxes of Qt (nq rows x 64 tokens)
  const int stage_bytes = KB * (kLoraTileBytes + q_bytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int jb = 0;
#pragma unroll
  for (int j = 1; j < kLoraMaxJobs; ++j)
    if (j < args.njobs && (int)blockIdx.x >= args.jobs[j].tile0) jb = j;
  const LoraWgradJob& job = args.jobs[jb];
  const int itile = (int)blockIdx.x - job.tile0;
  const int icol = job.i_begin + itile * 128;  // P column of TMEM lane 0
  const int t0 = (int)blockIdx.y * args.tsplit;
  const int t1 = min(args.T, t0 + args.tsplit);
  const int nk = t1 > t0 ? (t1 - t0 + 64 * KB - 1) / (64 * KB) : 0;
  const uint32_t tcols = tmem_cols_for(nq);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmP);
    prefetch_tmap(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    // stage: P tokens [t, t+64) x columns [icol, icol+128) as two MN-major boxes
    // of 64 columns (8 KB apart), then Qt rows [q_row, q_row+nq) x tokens [t, t+64)
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&empty_bar[s], (uint32_t)(((i / S) & 1) ^ 1), args.status, kLoraErrProducer))
        break;
      uint8_t* sa = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full_bar[s], (uint32_t)stage_bytes);
      for (int b = 0; b < KB; ++b) {
        const int t = t0 + (i * KB + b) * 64;
        tma_load_2d(sa + b * kLoraTileBytes, &tmP, &full_bar[s], icol, t);
        tma_load_2d(sa + b * kLoraTileBytes + 8192, &tmP, &full_bar[s], icol + 64, t);
        tma_load_2d(sa + KB * kLoraTileBytes + b * q_bytes, &tmQ, &full_bar[s], t, job.q_row);
      }
      ++issued;
    }
    drain_loads(full_bar, issued, S);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    // D[i, j] += P[t, i] (A, MN-major: transpose bit 15) * Qt[j, t] (B, K-major)
    const uint32_t idesc = umma_idesc_bf16(128, nq) | (1u << 15);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full_bar[s], (uint32_t)((i / S) & 1), args.status, kLoraErrMma)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
      const uint32_t b_addr = a_addr + KB * kLoraTileBytes;
      for (int b = 0; b < KB; ++b) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 16 tokens per MMA: 2048 B within the 64-row atom
          umma_f16_ss(tmem_base, umma_desc_sw128_mnmajor(a_addr + b * kLoraTileBytes + kk * 2048, 8192),
                      umma_desc_sw128_kmajor(b_addr + b * q_bytes + kk * 32), idesc,
                      (i > 0 || b > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&empty_bar[s]);
    }
    umma_commit(done_bar);
  }
  __syncwarp();

  // ------------------------------------------------------------ epilogue
  // (uniform over the CTA, so the barriers below are reached by every thread)
  const bool have = __syncthreads_and(nk > 0 && mbar_wait(done_bar, 0, args.status, kLoraErrEpi));
  tc_fence_after();
  const int row = warp * 32 + lane;
  const int tile_rel = icol - job.i_begin;  // job-relative P column of TMEM lane 0
  const int nvalid = max(0, min(128, job.i_count - tile_rel));
  const int i_rel = tile_rel + row;
  const int64_t ld = args.ld_out;
  const int rv = args.rvalid;
  const int ng = nq / args.gsz;
  // The tile's contribution to each output is contiguous in global memory: one
  // row of 128 columns per rank row (A gradient) or 128 x r values (B gradient
  // with rows of exactly r).  Stage it in shared memory (the ring is free) and
  // add it with bulk asynchronous reductions; other layouts use atomics.
  bool bulk = have && nvalid > 0;
  if (args.transposed)
    bulk = bulk && nvalid % 4 == 0 && ld % 4 == 0 && tile_rel % 4 == 0;
  else
    bulk = bulk && ld == rv && (nvalid * rv) % 4 == 0;
  for (int g = 0; g < ng; ++g) bulk = bulk && aligned16(job.out[g]);
  float* stage = reinterpret_cast<float*>(smem);
  for (int c = 0; c < nq; c += 16) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
    tmem_ld_wait();
    if (!have || i_rel >= job.i_count) continue;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int j = c + e;
      const int g = j / args.gsz, jj = j - g * args.gsz;
      if (jj >= rv) continue;
      const float v = job.alpha * __uint_as_float(r[e]);
      if (bulk) {
        float* sg = stage + g * 128 * rv;
        if (args.transposed)
          sg[jj * 128 + row] = v;
        else
          sg[row * rv + jj] = v;
      } else if (args.transposed) {
        atomicAdd(job.out[g] + (int64_t)jj * ld + i_rel, v);
      } else {
        atomicAdd(job.out[g] + (int64_t)i_rel * ld + jj, v);
      }
    }
  }
  if (bulk) {
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int g = 0; g < ng; ++g) {
        const float* sg = stage + g * 128 * rv;
        if (args.transposed) {
          for (int jj = 0; jj < rv; ++jj)
            bulk_reduce_add_f32(job.out[g] + (int64_t)jj * ld + tile_rel, sg + jj * 128, (uint32_t)nvalid * 4);
        } else {
          bulk_reduce_add_f32(job.out[g] + (int64_t)tile_rel * ld, sg, (uint32_t)(nvalid * rv) * 4);
        }
      }
      bulk_commit_group();
      bulk_wait_group<0>();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}


// ----------------------------------------------------------------------------
// lora_vdb: the backward's two products over dY in ONE pass:
//   V  [T, nqv] = dY · Bt[:nqv]ᵀ        (rank space, as lora_down)
//   dB_s[n, jj] += sum_t dY[t, n] * Ut[q_row_s + jj, t]   (n in segment s)
// A stage holds dY tokens [t0, t0+128) x columns [n, n+64) (K-major A of the V
// MMAs).  Two consecutive stages hold 128 columns, which the dB MMAs read as an
// MN-major A operand (M = 128 columns, LBO = one stage, K = the 128 tokens)
// against the K-major Ut tile of the same tokens; every 128-column pair has its
// own TMEM accumulator, drained by red.global.add at the end.
// ----------------------------------------------------------------------------
struct LoraVdbSeg {
  int n_begin, n_count, q_row;  // columns of dY (multiples of 128), first Ut row
  float* out;                   // dB [n_count, >= rvalid] fp32, row stride ld_out
};

struct LoraVdbArgs {
  int T, N, nqv, nqb, nqu, rvalid, nseg, ppc, vcols;
  LoraVdbSeg seg[kLoraMaxJobs];
  int64_t ld_out;
  __nv_bfloat16* v;   // [T, vpad]
  int64_t ldv;
  int vpad;
  __nv_bfloat16* vt;  // [nqv, >= T]
  int64_t ldvt;
  int stages;         // ring depth (even: a 128-column pair is two adjacent stages)
  DeviceStatus* status;
};

__global__ void __launch_bounds__(kLoraThreads, 2)
lora_vdb_kernel(const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmBt,
                const __grid_constant__ CUtensorMap tmUt, const __grid_constant__ LoraVdbArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nqv = args.nqv, nqb = args.nqb;
  const int S = args.stages;
  const int stage_bytes = kLoraTileBytes + nqv * 128;
  const int ut_atom = args.nqu * 128;  // one 64-token K-major atom of Ut
  uint8_t* ut_smem = smem + S * stage_bytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(ut_smem + 2 * ut_atom);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint64_t* ut_bar = done_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ut_bar + 1);
  float* part = reinterpret_cast<float*>(smem);
  const int pld = nqv + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const int mt = (int)(blockIdx.x / csize);
  const int total_pairs = args.N / 128;
  const int pair0 = min(total_pairs, (int)crank * args.ppc);
  const int npairs = min(total_pairs, pair0 + args.ppc) - pair0;
  const int nk = 2 * npairs;
  uint32_t tcols = 32;
  while ((int)tcols < args.vcols + args.ppc * nqb) tcols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(ut_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmG);
    prefetch_tmap(&tmBt);
    prefetch_tmap(&tmUt);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    bool ut_issued = false;
    if (nk > 0) {
      mbar_arrive_expect_tx(ut_bar, (uint32_t)(2 * ut_atom));
      tma_load_2d(ut_smem, &tmUt, ut_bar, mt * 128, 0);
      tma_load_2d(ut_smem + ut_atom, &tmUt, ut_bar, mt * 128 + 64, 0);
      ut_issued = true;
    }
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&empty_bar[s], (uint32_t)(((i / S) & 1) ^ 1), args.status, kLoraErrProducer))
        break;
      uint8_t* sa = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full_bar[s], (uint32_t)stage_bytes);
      const int n = pair0 * 128 + i * 64;
      tma_load_2d(sa, &tmG, &full_bar[s], n, mt * 128);
      tma_load_2d(sa + kLoraTileBytes, &tmBt, &full_bar[s], n, 0);
      ++issued;
    }
    drain_loads(full_bar, issued, S);
    if (ut_issued) mbar_wait(ut_bar, 0, nullptr, 0);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_v = umma_idesc_bf16(128, nqv);
    const uint32_t idesc_b = umma_idesc_bf16(128, nqb) | (1u << 15);  // A MN-major
    bool ok = nk == 0 || mbar_wait(ut_bar, 0, args.status, kLoraErrMma);
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full_bar[s], (uint32_t)((i / S) & 1), args.status, kLoraErrMma)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
      const uint32_t b_addr = a_addr + kLoraTileBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16_ss(tmem_base, umma_desc_sw128_kmajor(a_addr + kk * 32),
                    umma_desc_sw128_kmajor(b_addr + kk * 32), idesc_v, (i > 0 || kk > 0) ? 1u : 0u);
      if (i & 1) {
        // the pair (stages s-1, s): 128 dY columns x 128 tokens against Ut
        const int p = i >> 1;
        const int n = (pair0 + p) * 128;
        int sg = 0;
#pragma unroll
        for (int q = 1; q < kLoraMaxJobs; ++q)
          if (q < args.nseg && n >= args.seg[q].n_begin) sg = q;
        const uint32_t a0 = smem_u32(smem + (s - 1) * stage_bytes);
        const uint32_t u0 = smem_u32(ut_smem) + (uint32_t)(args.seg[sg].q_row * 128);
        const uint32_t d = tmem_base + (uint32_t)(args.vcols + p * nqb);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 tokens per MMA
          umma_f16_ss(d, umma_desc_sw128_mnmajor(a0 + (kk & 3) * 2048 + (kk >> 2) * 8192, (uint32_t)stage_bytes),
                      umma_desc_sw128_kmajor(u0 + (kk >> 2) * ut_atom + (kk & 3) * 32), idesc_b,
                      kk > 0 ? 1u : 0u);
        umma_commit(&empty_bar[s - 1]);
        umma_commit(&empty_bar[s]);
      }
    }
    umma_commit(done_bar);
  }
  __syncwarp();

  // (uniform over the CTA, so the barriers below are reached by every thread)
  const bool have = __syncthreads_and(nk > 0 && mbar_wait(done_bar, 0, args.status, kLoraErrEpi));
  tc_fence_after();
  const int row = warp * 32 + lane;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  // ------------------------------------------------------------ dB: TMEM -> global
  // A pair's dB tile (128 columns of dY x r) is one contiguous block of the
  // output when its rows hold exactly r values: staged in the (free) ring and
  // added with one bulk asynchronous reduction per pair, as many pairs per
  // round as the ring holds; other layouts use atomics.
  if (have) {
    const int rv = args.rvalid;
    bool bulk = args.ld_out == rv;
    for (int q = 0; q < args.nseg; ++q) bulk = bulk && aligned16(args.seg[q].out);
    float* stage = reinterpret_cast<float*>(smem);
    const int tile_floats = 128 * rv;
    const int slots = max(1, (S * stage_bytes) / (tile_floats * 4));
    for (int p0 = 0; p0 < npairs; p0 += slots) {
      const int pe = min(npairs, p0 + slots);
      for (int p = p0; p < pe; ++p) {
        const int n = (pair0 + p) * 128 + row;
        int sg = 0;
#pragma unroll
        for (int q = 1; q < kLoraMaxJobs; ++q)
          if (q < args.nseg && (pair0 + p) * 128 >= args.seg[q].n_begin) sg = q;
        float* orow = args.seg[sg].out + (int64_t)(n - args.seg[sg].n_begin) * args.ld_out;
        float* srow = stage + (p - p0) * tile_floats + row * rv;
        for (int c = 0; c < nqb; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem_base + lane_base + (uint32_t)(args.vcols + p * nqb + c), r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (c + e >= rv) continue;
            if (bulk)
              srow[c + e] = __uint_as_float(r[e]);
            else
              atomicAdd(orow + c + e, __uint_as_float(r[e]));
          }
        }
      }
      if (bulk) {
        fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
          for (int p = p0; p < pe; ++p) {
            const int n0 = (pair0 + p) * 128;
            int sg = 0;
            for (int q = 1; q < args.nseg; ++q)
              if (n0 >= args.seg[q].n_begin) sg = q;
            bulk_reduce_add_f32(args.seg[sg].out + (int64_t)(n0 - args.seg[sg].n_begin) * args.ld_out,
                                stage + (p - p0) * tile_floats, (uint32_t)tile_floats * 4);
          }
          bulk_commit_group();
          bulk_wait_group<0>();
        }
        __syncthreads();
      }
    }
  }
  // ------------------------------------------------------------ V partial -> smem
  float* prow = part + row * pld;
  for (int c = 0; c < nqv; c += 16) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(tmem_base + lane_base + (uint32_t)c, r);
    tmem_ld_wait();
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float4 o = have ? make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(prow + c + 4 * v) = o;
    }
  }
  tc_fence_before();
  cluster_sync_all();

  // ------------------------------------------------------------ cluster reduction of V
  {
    const int rows_per = (128 + (int)csize - 1) / (int)csize;
    const int r0 = (int)crank * rows_per;
    cluster_reduce_store_any(csize, smem_u32(part), pld, nqv, args.vpad, r0, min(128, r0 + rows_per),
                             mt * 128, args.T, args.v, args.ldv, args.vt, args.ldvt);
  }
  cluster_sync_all();

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

}  // namespace zq

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------
using namespace zq;

namespace {

// 2-D bf16 [rows, cols] (row stride in elements) with a box of 64 columns x
// box_rows rows and the 128-byte swizzle (the tcgen05 operand layouts)
CUtensorMap lora_tmap(const void* base, int64_t rows, int64_t cols, int64_t row_stride, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "lora: TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride * 2) % 16 == 0, "lora: row pitch must be a multiple of 16 bytes");
  TORCH_CHECK(box_rows >= 1 && box_rows <= 256, "lora: TMA box rows out of range");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "lora: cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

size_t lora_smem_bytes(int nq, int stages, int kb) {
  return (size_t)stages * kb * (kLoraTileBytes + nq * 128) + (2 * stages + 1) * 8 + 16 + 1024;
}

void check_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1,
              "lora: ", name, " must be a CUDA bf16 2-D tensor with unit column stride");
  TORCH_CHECK(t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "lora: ", name, " rows must start on 16-byte boundaries");
}

// Dynamic shared memory to request so that the CTAs shared memory lets share an
// SM never need more than the SM's 512 TMEM columns together (a CTA that could
// not allocate would wait for another to exit).
size_t tmem_safe_smem(size_t smem, int tmem_cols) {
  const size_t per_sm = 228 * 1024;  // shared memory per SM on sm_100
  const size_t max_ctas = 512 / (size_t)tmem_cols;
  const size_t floor_bytes = per_sm / (max_ctas + 1) + 1024;
  return std::max(smem, floor_bytes);
}

int host_tmem_cols(int need) {
  int c = 32;
  while (c < need) c <<= 1;
  return c;
}

int sm_count(int dev) {
  static int cache[64] = {0};
  if (cache[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev));
  return cache[dev];
}

}  // namespace

// U [T, upad] (bf16, cols >= nq zero) = P [T, K] · W[:nq]ᵀ, and optionally
// Ut [nq, >= T] = Uᵀ.  nq = w.size(0): a multiple of 16, at most 256.
// cs / stages / kb (0 = automatic): cluster size (K split), ring depth and
// 64-wide K boxes per stage - launch-shape knobs for measurement.
void lora_down(at::Tensor p, at::Tensor w, at::Tensor u, c10::optional<at::Tensor> ut, int64_t cs_req,
               int64_t stages_req, int64_t kb_req) {
  check_operand(p, "P");
  check_operand(w, "W");
  check_operand(u, "U");
  const int64_t T = p.size(0), K = p.size(1), nq = w.size(0);
  TORCH_CHECK(w.size(1) == K, "lora_down: W must be [nq, K]");
  TORCH_CHECK(nq >= 16 && nq <= 256 && nq % 16 == 0, "lora_down: nq must be a multiple of 16 in [16, 256]");
  TORCH_CHECK(u.size(0) == T && u.size(1) >= nq && u.size(1) % 8 == 0, "lora_down: U must be [T, >= nq]");
  TORCH_CHECK(T <= INT32_MAX && K <= INT32_MAX, "lora_down: size");
  __nv_bfloat16* utp = nullptr;
  int64_t ldt = 0;
  if (ut.has_value() && ut->defined()) {
    check_operand(*ut, "Ut");
    TORCH_CHECK(ut->size(0) == nq && ut->size(1) >= T, "lora_down: Ut must be [nq, >= T]");
    utp = reinterpret_cast<__nv_bfloat16*>(ut->data_ptr());
    ldt = ut->stride(0);
  }
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(p.device());
  const int dev = p.get_device();
  const CUtensorMap tp = lora_tmap(p.data_ptr(), T, K, p.stride(0), 128);
  const CUtensorMap tw = lora_tmap(w.data_ptr(), nq, K, w.stride(0), (int)nq);
  LoraDownArgs a;
  a.T = (int)T;
  a.K = (int)K;
  a.nq = (int)nq;
  a.u = reinterpret_cast<__nv_bfloat16*>(u.data_ptr());
  a.ldu = u.stride(0);
  a.upad = (int)u.size(1);
  a.ut = utp;
  a.ldt = ldt;
  a.status = status_buffer(dev);
  const int kb = kb_req > 0 ? (int)kb_req : 1;
  const int stages = stages_req > 0 ? (int)stages_req : 4;
  TORCH_CHECK(kb >= 1 && kb <= 4 && stages >= 2 && stages <= kLoraMaxStages, "lora_down: kb / stages");
  a.stages = stages;
  a.kb = kb;
  // K split over a cluster: enough CTAs for two per SM, at most 8 and at most
  // one K stage each
  const int64_t mtiles = (T + 127) / 128;
  const int64_t kt = (K + 64 * kb - 1) / (64 * kb);
  int cs = 1;
  if (cs_req > 0) {
    TORCH_CHECK(cs_req == 1 || cs_req == 2 || cs_req == 4 || cs_req == 8, "lora_down: cs must be 1, 2, 4 or 8");
    cs = (int)cs_req;
  } else {
    while (cs < 8 && mtiles * cs * 2 <= 2 * (int64_t)sm_count(dev) && cs * 2 <= kt) cs *= 2;
  }
  const size_t smem = tmem_safe_smem(lora_smem_bytes((int)nq, stages, kb), host_tmem_cols((int)nq));
  C10_CUDA_CHECK(cudaFuncSetAttribute(lora_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(mtiles * cs), 1, 1);
  cfg.blockDim = dim3(kLoraThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, lora_down_kernel, tp, tw, a));
}

// For each job b: out_b,g[...] += alpha_b * sum_t P[t, i_begin_b + i] * Qt[q_row_b + j, t]
// for i < i_count_b and j < nq with (j % gsz) < rvalid, g = j / gsz; outs holds
// the njobs x (nq / gsz) fp32 outputs job-major.  transposed: out[jj, i]
// (a LoRA A gradient, [r, in]); else out[i, jj] (a LoRA B gradient, [out, r]).
void lora_wgrad(at::Tensor p, at::Tensor qt, int64_t nq, std::vector<int64_t> i_begin,
                std::vector<int64_t> i_count, std::vector<int64_t> q_row, std::vector<double> alpha,
                std::vector<at::Tensor> outs, int64_t gsz, int64_t rvalid, bool transposed,
                int64_t splits_req, int64_t stages_req, int64_t kb_req) {
  check_operand(p, "P");
  check_operand(qt, "Qt");
  const int64_t T = p.size(0), I = p.size(1);
  const size_t nj = i_begin.size();
  TORCH_CHECK(nj >= 1 && nj <= (size_t)kLoraMaxJobs && i_count.size() == nj && q_row.size() == nj &&
                  alpha.size() == nj, "lora_wgrad: 1 to 4 jobs with matching lists");
  TORCH_CHECK(nq >= 16 && nq <= 256 && nq % 16 == 0, "lora_wgrad: nq must be a multiple of 16 in [16, 256]");
  TORCH_CHECK(gsz >= 1 && nq % gsz == 0 && nq / gsz <= kLoraMaxGroups && rvalid >= 1 && rvalid <= gsz,
              "lora_wgrad: groups");
  const int64_t ng = nq / gsz;
  TORCH_CHECK((int64_t)outs.size() == (int64_t)nj * ng, "lora_wgrad: need njobs x (nq / gsz) outputs");
  TORCH_CHECK(qt.size(1) >= T, "lora_wgrad: Qt must cover every token");
  TORCH_CHECK(T <= INT32_MAX && I <= INT32_MAX, "lora_wgrad: size");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(p.device());
  const int dev = p.get_device();
  LoraWgradArgs a;
  memset(&a, 0, sizeof(a));
  a.T = (int)T;
  a.nq = (int)nq;
  a.gsz = (int)gsz;
  a.rvalid = (int)rvalid;
  a.njobs = (int)nj;
  a.transposed = transposed ? 1 : 0;
  a.ld_out = -1;
  int64_t tiles = 0;
  for (size_t b = 0; b < nj; ++b) {
    TORCH_CHECK(i_begin[b] >= 0 && i_begin[b] % 64 == 0 && i_count[b] >= 1 && i_begin[b] + i_count[b] <= I,
                "lora_wgrad: job column range");
    TORCH_CHECK(q_row[b] >= 0 && q_row[b] + nq <= qt.size(0), "lora_wgrad: job rows of Qt");
    LoraWgradJob& j = a.jobs[b];
    j.i_begin = (int)i_begin[b];
    j.i_count = (int)i_count[b];
    j.q_row = (int)q_row[b];
    j.tile0 = (int)tiles;
    j.alpha = (float)alpha[b];
    tiles += (i_count[b] + 127) / 128;
    for (int64_t g = 0; g < ng; ++g) {
      at::Tensor& o = outs[b * ng + g];
      TORCH_CHECK(o.is_cuda() && o.scalar_type() == at::kFloat && o.dim() == 2 && o.stride(1) == 1 &&
                      o.get_device() == dev, "lora_wgrad: outputs must be fp32 2-D CUDA tensors");
      if (transposed) {
        TORCH_CHECK(o.size(0) >= rvalid && o.size(1) >= i_count[b], "lora_wgrad: output [r, in] too small");
      } else {
        TORCH_CHECK(o.size(0) >= i_count[b] && o.size(1) >= rvalid, "lora_wgrad: output [out, r] too small");
      }
      TORCH_CHECK(a.ld_out < 0 || a.ld_out == o.stride(0), "lora_wgrad: outputs must share one row stride");
      a.ld_out = o.stride(0);
      j.out[g] = o.data_ptr<float>();
    }
  }
  a.status = status_buffer(dev);
  const int kb = kb_req > 0 ? (int)kb_req : 1;
  const int stages = stages_req > 0 ? (int)stages_req : 4;
  TORCH_CHECK(kb >= 1 && kb <= 4 && stages >= 2 && stages <= kLoraMaxStages, "lora_wgrad: kb / stages");
  a.stages = stages;
  a.kb = kb;
  // token ranges: whole stages of 64 * kb tokens, enough CTAs for two per SM
  const int64_t tstage = 64 * kb;
  const int64_t ttiles = (T + tstage - 1) / tstage;
  int64_t splits = splits_req > 0 ? splits_req : (2 * (int64_t)sm_count(dev) + tiles - 1) / tiles;
  splits = std::max<int64_t>(1, std::min(splits, ttiles));
  const int64_t tsplit = ((ttiles + splits - 1) / splits) * tstage;
  splits = (T + tsplit - 1) / tsplit;
  a.tsplit = (int)tsplit;
  const CUtensorMap tp = lora_tmap(p.data_ptr(), T, I, p.stride(0), 64);
  const CUtensorMap tq = lora_tmap(qt.data_ptr(), qt.size(0), T, qt.stride(0), (int)nq);
  const size_t smem = tmem_safe_smem(lora_smem_bytes((int)nq, stages, kb), host_tmem_cols((int)nq));
  C10_CUDA_CHECK(cudaFuncSetAttribute(lora_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  lora_wgrad_kernel<<<dim3((unsigned)tiles, (unsigned)splits, 1), kLoraThreads, smem,
                      at::cuda::getCurrentCUDAStream()>>>(tp, tq, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// The backward's V = dY·Bt[:nqv]ᵀ (into V [T, vpad] and Vt [nqv, >= T]) and the
// B gradients dB_s += dY[:, seg_s]ᵀ · Ut[q_row_s : q_row_s + nqb]ᵀ in one pass
// over dY.  Returns false (nothing launched) when the shape does not fit this
// kernel (columns of dY or segment bounds not multiples of 128, or more TMEM
// than two CTAs per SM can hold); the caller then runs lora_down + lora_wgrad.
bool lora_vdb(at::Tensor g, at::Tensor bt, at::Tensor ut, at::Tensor v, at::Tensor vt, int64_t nqb,
              std::vector<int64_t> n_begin, std::vector<int64_t> n_count, std::vector<int64_t> q_row,
              std::vector<at::Tensor> outs, int64_t rvalid, int64_t cs_req, int64_t stages_req) {
  check_operand(g, "dY");
  check_operand(bt, "Bt");
  check_operand(ut, "Ut");
  check_operand(v, "V");
  check_operand(vt, "Vt");
  const int64_t T = g.size(0), N = g.size(1), nqv = bt.size(0), nqu = ut.size(0);
  const size_t ns = n_begin.size();
  TORCH_CHECK(bt.size(1) == N, "lora_vdb: Bt must be [nqv, N]");
  TORCH_CHECK(nqv >= 16 && nqv <= 256 && nqv % 16 == 0, "lora_vdb: nqv must be a multiple of 16 in [16, 256]");
  TORCH_CHECK(nqb >= 16 && nqb <= 256 && nqb % 16 == 0 && rvalid >= 1 && rvalid <= nqb, "lora_vdb: nqb / rvalid");
  TORCH_CHECK(nqu % 8 == 0 && nqu <= 256 && ut.size(1) >= T, "lora_vdb: Ut must be [nqu (multiple of 8), >= T]");
  TORCH_CHECK(v.size(0) == T && v.size(1) >= nqv && v.size(1) % 8 == 0, "lora_vdb: V must be [T, >= nqv]");
  TORCH_CHECK(vt.size(0) == nqv && vt.size(1) >= T, "lora_vdb: Vt must be [nqv, >= T]");
  TORCH_CHECK(ns >= 1 && ns <= (size_t)kLoraMaxJobs && n_count.size() == ns && q_row.size() == ns &&
                  outs.size() == ns, "lora_vdb: 1 to 4 segments with matching lists");
  TORCH_CHECK(T <= INT32_MAX && N <= INT32_MAX, "lora_vdb: size");
  if (N % 128 != 0) return false;
  const at::cuda::CUDAGuard guard(g.device());
  const int dev = g.get_device();
  LoraVdbArgs a;
  memset(&a, 0, sizeof(a));
  a.ld_out = -1;
  int64_t covered = 0;
  for (size_t i = 0; i < ns; ++i) {
    if (n_begin[i] % 128 != 0 || n_count[i] % 128 != 0) return false;
    TORCH_CHECK(n_begin[i] == covered, "lora_vdb: segments must tile the columns of dY in order");
    covered += n_count[i];
    TORCH_CHECK(q_row[i] >= 0 && q_row[i] % 8 == 0 && q_row[i] + nqb <= nqu, "lora_vdb: segment rows of Ut");
    const at::Tensor& o = outs[i];
    TORCH_CHECK(o.is_cuda() && o.scalar_type() == at::kFloat && o.dim() == 2 && o.stride(1) == 1 &&
                    o.size(0) >= n_count[i] && o.size(1) >= rvalid && o.get_device() == dev,
                "lora_vdb: dB outputs must be fp32 [>= n_count, >= r] CUDA tensors");
    TORCH_CHECK(a.ld_out < 0 || a.ld_out == o.stride(0), "lora_vdb: outputs must share one row stride");
    a.ld_out = o.stride(0);
    a.seg[i].n_begin = (int)n_begin[i];
    a.seg[i].n_count = (int)n_count[i];
    a.seg[i].q_row = (int)q_row[i];
    a.seg[i].out = o.data_ptr<float>();
  }
  TORCH_CHECK(covered == N, "lora_vdb: segments must cover every column of dY");
  if (T == 0) return true;
  a.T = (int)T;
  a.N = (int)N;
  a.nqv = (int)nqv;
  a.nqb = (int)nqb;
  a.nqu = (int)nqu;
  a.rvalid = (int)rvalid;
  a.nseg = (int)ns;
  a.vcols = (int)((nqv + 15) / 16 * 16);
  a.v = reinterpret_cast<__nv_bfloat16*>(v.data_ptr());
  a.ldv = v.stride(0);
  a.vpad = (int)v.size(1);
  a.vt = reinterpret_cast<__nv_bfloat16*>(vt.data_ptr());
  a.ldvt = vt.stride(0);
  a.status = status_buffer(dev);
  const int stages = stages_req > 0 ? (int)stages_req : 4;
  TORCH_CHECK(stages >= 2 && stages <= kLoraMaxStages && stages % 2 == 0, "lora_vdb: stages must be even");
  a.stages = stages;
  // cluster size: enough CTAs for two per SM, and few enough 128-column pairs
  // per CTA that V plus the dB accumulators fit in 256 TMEM columns
  const int64_t mtiles = (T + 127) / 128;
  const int64_t pairs = N / 128;
  auto tmem_need = [&](int c) { return a.vcols + (int)((pairs + c - 1) / c) * (int)nqb; };
  int cs = 1;
  if (cs_req > 0) {
    TORCH_CHECK(cs_req == 1 || cs_req == 2 || cs_req == 4 || cs_req == 8, "lora_vdb: cs must be 1, 2, 4 or 8");
    cs = (int)cs_req;
  } else {
    // measured on B200 (8192 rows, r = 16): one pass wins at cluster sizes up to 4
    // (27.6 vs 37.3 us for 3072 columns); where TMEM would force 8 CTAs per
    // cluster (9216 / 12288 columns) the two separate kernels are as fast or faster
    while (cs < 4 && cs * 2 <= pairs &&
           (mtiles * cs * 2 <= 2 * (int64_t)sm_count(dev) || tmem_need(cs) > 256))
      cs *= 2;
  }
  if (tmem_need(cs) > 256) return false;
  a.ppc = (int)((pairs + cs - 1) / cs);
  const size_t smem = tmem_safe_smem((size_t)stages * (kLoraTileBytes + nqv * 128) + 2 * nqu * 128 +
                                         (2 * stages + 2) * 8 + 16 + 1024,
                                     host_tmem_cols(tmem_need(cs)));
  const CUtensorMap tg = lora_tmap(g.data_ptr(), T, N, g.stride(0), 128);
  const CUtensorMap tb = lora_tmap(bt.data_ptr(), nqv, N, bt.stride(0), (int)nqv);
  const CUtensorMap tu = lora_tmap(ut.data_ptr(), nqu, T, ut.stride(0), (int)nqu);
  C10_CUDA_CHECK(cudaFuncSetAttribute(lora_vdb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(mtiles * cs), 1, 1);
  cfg.blockDim = dim3(kLoraThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, lora_vdb_kernel, tg, tb, tu, a));
  return true;
}

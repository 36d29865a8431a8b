// tcgen05 GEMM for sm_100a:  C[M,N] (bf16) = A[M,K] · B[N,K]^T  (+ A2[M,64] · B2[N,64]^T)
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer - one elected thread streams 128x64 A tiles and
//                 BNx64 B tiles (128-byte swizzle) into a STAGES-deep ring.
//   warp 1      : MMA issuer - allocates TMEM, one thread issues
//                 tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) and
//                 commits to the ring's "empty" barriers and to the
//                 accumulator's "full" barrier.
//   warps 2..5  : epilogue - tcgen05.ld 32x32b.x32 from TMEM, fp32 -> bf16,
//                 16-byte stores; then release the accumulator buffer.
// Two accumulator buffers in TMEM (2 x BN fp32 columns) let the epilogue of
// tile i overlap the MMAs of tile i+1.  Tiles are visited in groups of
// kGroupM row-blocks so that concurrently running CTAs share A and B tiles in
// L2.
//
// The optional second operand pair (A2, B2) is one extra K=64 slab appended to
// the K loop; the NF4 linear layer uses it for the LoRA up-projection
// (A2 = s·X·Aᵀ zero-padded to 64 columns, B2 = lora_B zero-padded).
//
// Every mbarrier wait is bounded (see common.cuh); on timeout the kernel
// records an error in a device status word, stops its loops, and still frees
// its TMEM before exiting.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "peer_gather.cuh"
#include "gelu.cuh"
#include "swiglu.cuh"

namespace zq {

constexpr int kBM = 128;
constexpr int kBK = 64;          // one 128-byte swizzle atom of bf16
constexpr int kGroupM = 8;
constexpr int kGemmThreads = 192;

enum GemmErr { kErrProducer = 101, kErrMma = 102, kErrMmaAcc = 103, kErrEpi = 104, kErrAgWait = 105 };

struct GemmArgs {
  int M, N, K;           // main problem; K % 64 == 0
  int extra_k16;         // K=16 MMA steps in the extra slab (0 = none); the pair kernel
                         // takes 4, 8, 12 or 16 (one pipeline stage per 64 columns)
  int tiles_m, tiles_n;
  __nv_bfloat16* C;
  int64_t ldc;
  DeviceStatus* status;
  // NF4/FP4 B operand decoded in the kernel (Q4 variants only): the weight
  // W [q_rows, q_cols] in the bitsandbytes layout (flat blocks of q_block along
  // the row-major order, element 2i in the high nibble, fp32 absmax per block)
  const uint8_t* q_packed;
  const float* q_absmax;
  int q_rows, q_cols, q_block, q_type;  // q_type: 0 = nf4, 1 = fp4
  // stream-K tail (pair kernel): tiles [sk_first, sk_first + sk_tiles) are split
  // along K into sk_splits parts on different clusters (sk_splits <= 1: off).
  // Each part adds its fp32 result into the tile's block of sk_ws (zero between
  // GEMMs); the last part to arrive at the tile's counter in sk_cnt reads the
  // sum, stores the tile, zeroes the block and resets the counter.
  int sk_first, sk_tiles, sk_splits;
  float* sk_ws;
  int* sk_cnt;
  // gather mode (AG variants only): B = W [N, K] is assembled inside the kernel
  // from its owners' 4-bit shards (ag) into the local bf16 buffer ag_w, which the
  // B tensor map reads.  Gather warps claim items of 8 rows x 1024 columns in
  // tile order from ag_sync[kAgClaim] and count finished items per N tile in
  // ag_sync[tn]; the producer loads a tile's B once its counter is full.  N
  // tiles are visited starting at ag_rot (this rank's own rows first).  The
  // last CTA to leave resets every counter (ag_sync[kAgExit] counts exits).
  AgSource ag;
  __nv_bfloat16* ag_w;
  int* ag_sync;
  int ag_rot, ag_kchunks, ag_cols;  // ag_cols: columns per gather item
  // epilogue input (kEpiGeluBwd): the pre-activation h [M, N], row pitch epi_ld;
  // (kEpiSwigluFwd / kEpiSwigluBwd): the gate pre-activation g [M, N]
  const __nv_bfloat16* epi_src;
  int64_t epi_ld;
  // second epilogue input (kEpiSwigluBwd): the up-projection output u [M, N]
  const __nv_bfloat16* epi_src2;
  int64_t epi_ld2;
  // epilogue input (kEpiRope): (cos, sin) table [epi_S, 64] of float2
  const float2* epi_cs;
  int epi_S;
  int epi_ncols;   // kEpiRope: only heads in columns [0, epi_ncols) are rotated
};

// Pair-kernel epilogues.  kEpiGeluFwd stores C = bf16(acc) through tmC and
// gelu(C) through tmC2 (the up-projection writes the pre-activation for the
// backward and the activation for the next GEMM); kEpiGeluBwd stores
// bf16(bf16(acc) * gelu'(h)) (the input gradient of the down-projection turned
// into the gradient of the pre-activation).  Both round the accumulator to bf16
// first, so they equal a separate GELU kernel applied to the stored GEMM output.
//
// kEpiRope applies rotary position embedding (rotate-half pairs (i, i + 64) of
// every 128-wide head) to the bf16-rounded output: row m is position m % S and
// epi_cs holds (cos, sin) of each position and pair (fp32, [S, 64, 2]) - the
// arithmetic of the standalone RoPE kernel, so q/k projections need no RoPE pass.
//
// SwiGLU MLP halves (gate g and up u are separate projections of the same x):
// kEpiSwigluFwd is the up-projection: it stores u = bf16(acc) through tmC and
// silu(g)·u through tmC2, reading g [M, N] (epi_src) - the activation kernel's
// three passes over [M, N] become one extra read.  kEpiSwigluBwd is the input
// gradient of the down-projection, dact = bf16(acc): it reads g (epi_src) and
// u (epi_src2) and stores dg = dact·u·silu'(g) through tmC and du = dact·silu(g)
// through tmC2, so dact is never stored.  Both use the arithmetic of the
// standalone SwiGLU kernels on the bf16-rounded values (swiglu.cuh).
enum PairEpi { kEpiPlain = 0, kEpiGeluFwd = 1, kEpiGeluBwd = 2, kEpiRope = 3, kEpiSwigluFwd = 4,
               kEpiSwigluBwd = 5 };

constexpr int kAgMaxTilesN = 4096;
constexpr int kAgClaim = kAgMaxTilesN, kAgExit = kAgMaxTilesN + 1, kAgSyncWords = kAgMaxTilesN + 2;

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// generic-proxy global writes <-> async-proxy (TMA) global reads
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Work item w of a pair cluster: data-parallel tiles first (whole K), then at
// most one stream-K part of a tail tile.
struct PairWork {
  int tile, k0, k1;   // K range in pipeline stages
  bool extra;         // this part also runs the extra 64-wide slab
  int sk, split;      // stream-K tile index and part (sk < 0: whole tile)
};

__device__ __forceinline__ bool pair_work(const GemmArgs& a, int cluster_id, int num_clusters, int w,
                                          int main_k, PairWork& out) {
  const int dp = a.sk_splits > 1 ? a.sk_first : a.tiles_m * a.tiles_n;
  const int n_dp = dp > cluster_id ? (dp - cluster_id + num_clusters - 1) / num_clusters : 0;
  if (w < n_dp) {
    out.tile = cluster_id + w * num_clusters;
    out.k0 = 0;
    out.k1 = main_k;
    out.extra = true;
    out.sk = -1;
    out.split = 0;
    return true;
  }
  if (a.sk_splits > 1 && w == n_dp && cluster_id < a.sk_tiles * a.sk_splits) {
    const int sk = cluster_id / a.sk_splits, sp = cluster_id % a.sk_splits;
    out.tile = a.sk_first + sk;
    out.k0 = sp * main_k / a.sk_splits;
    out.k1 = (sp + 1) * main_k / a.sk_splits;
    out.extra = sp == a.sk_splits - 1;
    out.sk = sk;
    out.split = sp;
    return true;
  }
  return false;
}

__constant__ float c_code_nf4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};
__constant__ float c_code_fp4[16] = {0.0f, 0.005208333333f, 0.66666667f, 1.0f, 0.33333333f,
                                     0.5f, 0.16666667f, 0.25f, -0.0f, -0.005208333333f,
                                     -0.66666667f, -1.0f, -0.33333333f, -0.5f, -0.16666667f,
                                     -0.25f};



template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int group_size = kGroupM * tiles_n;
  const int g = tile / group_size;
  const int first_m = g * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int r = tile % group_size;
  tm = first_m + r % gm;
  tn = r / gm;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
               GemmArgs args) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int k_tiles = args.K / kBK + (args.extra_k16 > 0 ? 1 : 0);
  const int main_k_tiles = args.K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4 * 32);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (args.extra_k16 > 0) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, args.tiles_m, args.tiles_n, tm, tn);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.status, kErrProducer)) { ok = false; break; }
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], L::kStageBytes);
          if (kt < main_k_tiles) {
            tma_load_2d(sa, &tmA, &full_bar[stage], kt * kBK, tm * kBM);
            tma_load_2d(sb, &tmB, &full_bar[stage], kt * kBK, tn * BN);
          } else {
            tma_load_2d(sa, &tmA2, &full_bar[stage], 0, tm * kBM);
            tma_load_2d(sb, &tmB2, &full_bar[stage], 0, tn * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: wait (bounded) until every load issued has landed, so no TMA
      // write targets this CTA's shared memory after it exits.
      for (int i = 0; i < STAGES; ++i) {
        mbar_wait(&empty_bar[stage], phase ^ 1, nullptr, 0);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty_bar[buf], acc_phase ^ 1, args.status, kErrMmaAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * 256);
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full_bar[stage], phase, args.status, kErrMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
          const int nk = kt < main_k_tiles ? kBK / 16 : args.extra_k16;
          for (int kk = 0; kk < nk; ++kk) {
            const uint64_t adesc = umma_desc_sw128_kmajor(a_addr + kk * 32);
            const uint64_t bdesc = umma_desc_sw128_kmajor(b_addr + kk * 32);
            umma_f16_ss(d_tmem, adesc, bdesc, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&tfull_bar[buf]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
      int tm, tn;
      tile_coords(tile, args.tiles_m, args.tiles_n, tm, tn);
      const int buf = it & 1;
      if (!mbar_wait(&tfull_bar[buf], (it >> 1) & 1, args.status, kErrEpi)) { ok = false; break; }
      tc_fence_after();
      const int m = tm * kBM + row_in_tile;
      const int n0 = tn * BN;
      __nv_bfloat16* crow = args.C + (int64_t)m * args.ldc;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256 + c * 32), r);
        tmem_ld_wait();
        const int ncol = n0 + c * 32;
        if (m < args.M) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int nc = ncol + v * 8;
            if (nc + 8 <= args.N) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
              o.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
              o.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
              o.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
              *reinterpret_cast<uint4*>(crow + nc) = o;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ----------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): one MMA of M=256 x BN
// per k-step, issued by the leader CTA.  Each CTA stages its own 128 rows of A
// and its own BN/2 rows of B (so every SM reads half of B from its shared
// memory), and holds its 128 rows x BN accumulator columns in its own TMEM.
//   full[s]   (leader): one arrive.expect_tx by the leader's producer for both
//             CTAs' bytes; both CTAs' TMA loads complete_tx on it.
//   empty[s]  (each CTA): the leader's commits (one per CTA address) free the
//             stage in both CTAs.
//   tfull[b]  (each CTA): the leader's commits after a tile's last k-step.
//   tempty[b] (leader): 2 x 128 epilogue threads of both CTAs arrive.
// ----------------------------------------------------------------------------
template <int BN, int STAGES, int KB>
struct PairSmem {
  // KB 128-byte-wide K atoms per stage (BK = 64 * KB): 8 MMAs per commit at
  // KB = 2, which measured markedly lower pipeline overhead than KB = 1
  static constexpr int kAAtom = kBM * kBK * 2;             // 128 rows x 64 K of A
  static constexpr int kBAtom = (BN / 2) * kBK * 2;        // BN/2 rows x 64 K of B
  static constexpr int kABytes = kAAtom * KB;              // this CTA's 128 rows of A
  static constexpr int kBBytes = kBAtom * KB;              // this CTA's half of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;         // 2 x [128 rows][32 cols] bf16
  static constexpr int kEpiBytes = 128 * 32 * 2;
  static constexpr int kBarOffset = kEpiOffset + 2 * kEpiBytes;
  static constexpr int kLutOffset = kBarOffset + 128;      // 16 fp32 decode values (Q4)
  static constexpr int kBytes = kBarOffset + 256 + 1024;
};

constexpr int kQ4DecodeWarps = 4;
constexpr int kGemmQ4Threads = kGemmThreads + 32 * kQ4DecodeWarps;

// 32 consecutive 4-bit codes (16 bytes, element 2i in the high nibble) times
// their block's absmax -> four 16-byte chunks of bf16, stored at
// dst + ((chunk0 + i) ^ swz) * 16 for i = 0..3 (the 128-byte swizzle of the
// tcgen05 operand layout).  The decode is fp32 table lookup x fp32 absmax then
// one round to bf16 - the same arithmetic as the standalone dequantize kernels.
__device__ __forceinline__ void q4_decode_store32(const uint4& raw, float am, const float* lut,
                                                  uint8_t* dst, int chunk0, int swz) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t byte = (w[i] >> (8 * q)) & 0xFFu;
      o[q] = pack_bf16x2(lut[byte >> 4] * am, lut[byte & 15u] * am);
    }
    *reinterpret_cast<uint4*>(dst + (((chunk0 + i) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Output tile (tm, tn) of work tile `tile`: grouped rasterisation, and in
// gather mode the N tiles rotated to start at this rank's own rows.
__device__ __forceinline__ void pair_tile_coords(const GemmArgs& a, int tile, bool ag, int& tm, int& tn) {
  tile_coords(tile, a.tiles_m, a.tiles_n, tm, tn);
  if (ag) {
    tn += a.ag_rot;
    if (tn >= a.tiles_n) tn -= a.tiles_n;
  }
}

template <int BN, int STAGES, int KB, bool BMN, bool Q4 = false, bool AG = false, int EPI = kEpiPlain>
__global__ void __launch_bounds__((Q4 || AG) ? kGemmQ4Threads : kGemmThreads, 1)
gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                    GemmArgs args) {
  using L = PairSmem<BN, STAGES, KB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cr = cluster_ctarank();        // 0 = leader
  const uint32_t peer = cr ^ 1u;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_tiles = args.tiles_m * args.tiles_n;  // tiles of 256 x BN
  const int main_k_tiles = args.K / (kBK * KB);
  const int k_tiles = main_k_tiles + args.extra_k16 / 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // Q4: the leader's producer arrival plus one per decode warp of both CTAs
      mbar_init(&full_bar[s], Q4 ? 1 + 2 * kQ4DecodeWarps : 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * 4 * 32);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    if (!Q4) prefetch_tmap(&tmB);
    if (args.extra_k16 > 0) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if ((Q4 || AG) && threadIdx.x < 16) {
    reinterpret_cast<float*>(smem + L::kLutOffset)[threadIdx.x] =
        args.q_type == 1 ? c_code_fp4[threadIdx.x] : c_code_nf4[threadIdx.x];
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      PairWork pw;
      for (int w = 0; ok && pair_work(args, cluster_id, num_clusters, w, main_k_tiles, pw); ++w) {
        int tm, tn;
        pair_tile_coords(args, pw.tile, AG, tm, tn);
        if (AG) {
          // this N tile's rows of W must be assembled before its B is loaded
          const int need = (BN / kAgRows) * args.ag_kchunks;
          const int* rp = args.ag_sync + tn;
          if (ld_acquire_gpu_s32(rp) < need) {
            const unsigned long long t0 = globaltimer();
            while (ld_acquire_gpu_s32(rp) < need) {
              if (globaltimer() - t0 > kWaitTimeoutNs) {
                record_error(args.status, kErrAgWait, tn);
                ok = false;
                break;
              }
              __nanosleep(64);
            }
            if (!ok) break;
          }
          fence_proxy_async_global();
        }
        const int arow = tm * (2 * kBM) + (int)cr * kBM;
        const int brow = tn * BN + (int)cr * (BN / 2);
        const int kt_end = pw.k1 + (pw.extra ? args.extra_k16 / 4 : 0);
        for (int kt = pw.k0; kt < kt_end; ++kt) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.status, kErrProducer)) { ok = false; break; }
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          const uint32_t leader_full = map_to_cta(smem_u32(&full_bar[stage]), 0);
          if (kt < main_k_tiles) {
            if (cr == 0)
              mbar_arrive_expect_tx(&full_bar[stage], 2 * (Q4 ? L::kABytes : L::kStageBytes));
            for (int kb = 0; kb < KB; ++kb) {
              const int kc = (kt * KB + kb) * kBK;
              tma_load_2d_pair(sa + kb * L::kAAtom, &tmA, leader_full, kc, arow);
              if (Q4) {
                // B is decoded into shared memory by the decode warps
              } else if (BMN) {
                // B is [K, N] row-major: boxes of 64 N-columns x 64 K-rows
                for (int ch = 0; ch < BN / 128; ++ch)
                  tma_load_2d_pair(sb + kb * L::kBAtom + ch * 8192, &tmB, leader_full,
                                   brow + ch * 64, kc);
              } else {
                tma_load_2d_pair(sb + kb * L::kBAtom, &tmB, leader_full, kc, brow);
              }
            }
          } else {  // extra slab: one 64-wide atom per stage, first atom of the stage only
            const int ec = (kt - main_k_tiles) * kBK;
            if (cr == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * (L::kAAtom + L::kBAtom));
            tma_load_2d_pair(sa, &tmA2, leader_full, ec, arow);
            if (BMN) {
              for (int ch = 0; ch < BN / 128; ++ch)
                tma_load_2d_pair(sb + ch * 8192, &tmB2, leader_full, brow + ch * 64, ec);
            } else {
              tma_load_2d_pair(sb, &tmB2, leader_full, ec, brow);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      for (int i = 0; i < STAGES; ++i) {  // drain: every issued load has landed
        mbar_wait(&empty_bar[stage], phase ^ 1, nullptr, 0);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && cr == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      constexpr uint32_t idesc = BMN ? umma_idesc_bf16_bmn(2 * kBM, BN) : umma_idesc_bf16(2 * kBM, BN);
      PairWork pw;
      for (int w = 0; ok && pair_work(args, cluster_id, num_clusters, w, main_k_tiles, pw); ++w, ++it) {
        const int buf = it & 1;
        if (!mbar_wait(&tempty_bar[buf], ((it >> 1) & 1) ^ 1, args.status, kErrMmaAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * 256);
        const int kt_end = pw.k1 + (pw.extra ? args.extra_k16 / 4 : 0);
        for (int kt = pw.k0; kt < kt_end; ++kt) {
          if (!mbar_wait(&full_bar[stage], phase, args.status, kErrMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
          const int nk = kt < main_k_tiles ? KB * (kBK / 16) : 4;
          for (int kk = 0; kk < nk; ++kk) {
            const uint32_t ao = (uint32_t)((kk >> 2) * L::kAAtom + (kk & 3) * 32);
            uint64_t bdesc;
            if (BMN) {  // 16 K-rows per MMA = 2048 B within a 64-row K atom
              const uint32_t bo = (uint32_t)((kk >> 2) * L::kBAtom + (kk & 3) * 2048);
              bdesc = umma_desc_sw128_mnmajor(b_addr + bo, 8192);
            } else {
              const uint32_t bo = (uint32_t)((kk >> 2) * L::kBAtom + (kk & 3) * 32);
              bdesc = umma_desc_sw128_kmajor(b_addr + bo);
            }
            umma_f16_ss_pair(d_tmem, umma_desc_sw128_kmajor(a_addr + ao), bdesc, idesc,
                             (kt > pw.k0 || kk > 0) ? 1u : 0u);
          }
          const uint32_t e = smem_u32(&empty_bar[stage]);
          umma_commit_pair(map_to_cta(e, 0));
          umma_commit_pair(map_to_cta(e, 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        const uint32_t f = smem_u32(&tfull_bar[buf]);
        umma_commit_pair(map_to_cta(f, 0));
        umma_commit_pair(map_to_cta(f, 1));
      }
    }
  } else if (AG && warp >= 6) {
    // ---------------------------------------------------------------- W gather (both CTAs)
    // Claim items in tile order (the next claim is issued before the current
    // item is worked on), decode each into ag_w, publish it to the producers.
    const float* lut = reinterpret_cast<const float*>(smem + L::kLutOffset);
    const int ipt = (BN / kAgRows) * args.ag_kchunks;
    const int total = args.tiles_n * ipt;
    int* claim = args.ag_sync + kAgClaim;
    int item = 0;
    if (lane == 0) item = atomicAdd(claim, 1);
    item = __shfl_sync(0xffffffffu, item, 0);
    while (item < total) {
      int next = 0;
      if (lane == 0) next = atomicAdd(claim, 1);
      const int p = item / ipt, j = item - p * ipt;
      int tn = p + args.ag_rot;
      if (tn >= args.tiles_n) tn -= args.tiles_n;
      const int rg = j / args.ag_kchunks, kc = j - rg * args.ag_kchunks;
      if (args.ag.kind == kAgF32)
        ag_item_f32(args.ag, args.N, args.K, tn * BN + rg * kAgRows, kc * args.ag_cols, args.ag_w, lane);
      else
        ag_item(args.ag, lut, args.N, args.K, args.q_block, tn * BN + rg * kAgRows, kc * args.ag_cols,
                args.ag_w, lane);
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (lane == 0) red_release_gpu_add(args.ag_sync + tn, 1);
      item = __shfl_sync(0xffffffffu, next, 0);
    }
  } else if (Q4 && warp >= 6) {
    // ---------------------------------------------------------------- B decode (both CTAs)
    // This CTA's B half per stage: 128 rows x 128 K (K-major, BMN = false) or
    // 128 K-rows x 128 N (MN-major, BMN = true) decoded from 4-bit codes.
    // Thread mapping per pass p (4 passes): row r = p*32 + dw*8 + lane/4 and a
    // 32-element chunk kc = lane%4 along the weight's row (16 packed bytes, one
    // absmax).  Loads for the next stage are issued before waiting for the
    // current stage's buffer, so global latency overlaps the pipeline wait.
    static_assert(!Q4 || (BN == 256 && KB == 2), "Q4 decode covers 128 x 128 per CTA and stage");
    const int dw = warp - 6;
    const int sub = dw * 8 + (lane >> 2);
    const int kc = lane & 3;
    const float* lut = reinterpret_cast<const float*>(smem + L::kLutOffset);
    const int64_t pitch = (int64_t)args.q_cols >> 1;
    bool ok = true;
    int stage = 0;
    uint32_t phase = 0;
    // work item w = (tile iteration) * k_tiles + kt for this cluster
    const int my_tiles = num_tiles > cluster_id ? (num_tiles - cluster_id + num_clusters - 1) / num_clusters : 0;
    const int total = my_tiles * k_tiles;
    uint4 raw[4];
    float am[4];
    auto load = [&](int w, uint4 (&rr)[4], float (&aa)[4]) {
      const int ti = w / k_tiles, kt = w - ti * k_tiles;
      int tm, tn;
      tile_coords(cluster_id + ti * num_clusters, args.tiles_m, args.tiles_n, tm, tn);
      const int nb = tn * BN + (int)cr * (BN / 2);   // first output column of this CTA's half
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int r = p * 32 + sub;
        int wrow, wcol;
        if (BMN) { wrow = kt * 128 + r; wcol = nb + kc * 32; }
        else     { wrow = nb + r;       wcol = kt * 128 + kc * 32; }
        if (kt < main_k_tiles && wrow < args.q_rows && wcol < args.q_cols) {
          rr[p] = __ldg(reinterpret_cast<const uint4*>(args.q_packed + (int64_t)wrow * pitch + (wcol >> 1)));
          aa[p] = __ldg(args.q_absmax + ((int64_t)wrow * args.q_cols + wcol) / args.q_block);
        } else {
          rr[p] = make_uint4(0u, 0u, 0u, 0u);
          aa[p] = 0.0f;
        }
      }
    };
    if (total > 0) load(0, raw, am);
    for (int w = 0; w < total && ok; ++w) {
      uint4 cur[4];
      float cam[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) { cur[p] = raw[p]; cam[p] = am[p]; }
      if (w + 1 < total) load(w + 1, raw, am);
      const int kt = w % k_tiles;
      const bool got = mbar_wait(&empty_bar[stage], phase ^ 1, args.status, kErrProducer);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
      if (kt < main_k_tiles) {
        uint8_t* sb = smem + stage * L::kStageBytes + L::kABytes;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int r = p * 32 + sub;
          uint8_t* dst;
          int swz;
          if (BMN) {  // atom = 64 K-rows; box of 64 N per 8 KB; row kk at kk*128
            const int kk = r & 63;
            dst = sb + (r >> 6) * L::kBAtom + (kc >> 1) * 8192 + kk * 128;
            swz = kk & 7;
          } else {    // atom = 64 K per row of 128 B; row r at r*128
            dst = sb + (kc >> 1) * L::kBAtom + r * 128;
            swz = r & 7;
          }
          q4_decode_store32(cur[p], cam[p], lut, dst, (kc & 1) * 4, swz);
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&full_bar[stage]), 0));
      if (++stage == STAGES) { stage = 0; phase ^= 1; }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    // TMEM -> registers -> bf16 -> 64-byte-swizzled staging tile in shared
    // memory -> one TMA tensor store per 128 x 32 chunk (double-buffered).
    const int q = warp & 3;
    const int row = q * 32 + lane;                 // row within this CTA's 128 rows
    const bool leader_thread = (warp == 2 && lane == 0);
    uint8_t* epi = smem + L::kEpiOffset;
    int it = 0, chunk_no = 0;
    bool ok = true;
    __shared__ int sk_last;   // stream-K: this CTA arrived last at its tile's counter
    // 32 packed bf16 pairs' worth of one row (16 words) -> 64-byte-swizzled
    // staging tile -> one TMA store of the 128 x 32 chunk through `map`
    auto stage_store = [&](const uint32_t (&o)[16], const CUtensorMap* map, int n_col, int m0) {
      uint8_t* st = epi + (chunk_no & 1) * L::kEpiBytes;
      // the store that last used this staging buffer (two chunks ago) must have read it
      if (leader_thread) bulk_wait_group_read<1>();
      named_barrier(1, 128);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pj = j ^ ((row >> 1) & 3);   // 64-byte swizzle
        *reinterpret_cast<uint4*>(st + row * 64 + pj * 16) =
            make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      }
      fence_proxy_async_smem();
      named_barrier(1, 128);
      if (leader_thread) {
        tma_store_2d(map, st, n_col, m0);
        bulk_commit_group();
      }
      ++chunk_no;
    };
    // epilogue inputs of this thread's row for columns n_col .. n_col+31
    constexpr bool kSide = EPI == kEpiGeluBwd || EPI == kEpiSwigluFwd || EPI == kEpiSwigluBwd;
    constexpr bool kSide2 = EPI == kEpiSwigluBwd;
    auto load_side = [&](const __nv_bfloat16* src, int64_t ld, int n_col, int m0, uint4 (&hv)[4]) {
      const int64_t grow = m0 + row;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = n_col + 8 * j;
        hv[j] = (grow < args.M && c < args.N)
                    ? *reinterpret_cast<const uint4*>(src + grow * ld + c)
                    : make_uint4(0u, 0u, 0u, 0u);
      }
    };
    auto load_h = [&](int n_col, int m0, uint4 (&hv)[4], uint4 (&hv2)[4]) {
      if constexpr (kSide) load_side(args.epi_src, args.epi_ld, n_col, m0, hv);
      if constexpr (kSide2) load_side(args.epi_src2, args.epi_ld2, n_col, m0, hv2);
    };
    // fp32 chunk of 32 columns -> epilogue -> staging -> TMA store(s)
    auto store_chunk = [&](const float (&v)[32], int n_col, int m0, const uint4 (&hv)[4],
                           const uint4 (&hv2)[4]) {
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      if constexpr (EPI == kEpiSwigluFwd || EPI == kEpiSwigluBwd) {
        const uint32_t gw[16] = {hv[0].x, hv[0].y, hv[0].z, hv[0].w, hv[1].x, hv[1].y, hv[1].z, hv[1].w,
                                 hv[2].x, hv[2].y, hv[2].z, hv[2].w, hv[3].x, hv[3].y, hv[3].z, hv[3].w};
        if constexpr (EPI == kEpiSwigluFwd) {
          stage_store(o, &tmC, n_col, m0);   // u
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 g = bf16x2_to_f2(gw[i]);
            const float2 u = bf16x2_to_f2(o[i]);
            o[i] = pack_bf16x2(swiglu_fwd_val(g.x, u.x), swiglu_fwd_val(g.y, u.y));
          }
          stage_store(o, &tmC2, n_col, m0);  // silu(g)·u
        } else {
          const uint32_t uw[16] = {hv2[0].x, hv2[0].y, hv2[0].z, hv2[0].w, hv2[1].x, hv2[1].y,
                                   hv2[1].z, hv2[1].w, hv2[2].x, hv2[2].y, hv2[2].z, hv2[2].w,
                                   hv2[3].x, hv2[3].y, hv2[3].z, hv2[3].w};
          uint32_t du[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 d = bf16x2_to_f2(o[i]);
            const float2 g = bf16x2_to_f2(gw[i]);
            const float2 u = bf16x2_to_f2(uw[i]);
            float dg0, du0, dg1, du1;
            swiglu_bwd_vals(d.x, g.x, u.x, dg0, du0);
            swiglu_bwd_vals(d.y, g.y, u.y, dg1, du1);
            du[i] = pack_bf16x2(du0, du1);
            o[i] = pack_bf16x2(dg0, dg1);
          }
          stage_store(o, &tmC, n_col, m0);    // dg
          stage_store(du, &tmC2, n_col, m0);  // du
        }
        return;
      }
      if constexpr (EPI == kEpiGeluBwd) {
        const uint32_t hw[16] = {hv[0].x, hv[0].y, hv[0].z, hv[0].w, hv[1].x, hv[1].y, hv[1].z, hv[1].w,
                                 hv[2].x, hv[2].y, hv[2].z, hv[2].w, hv[3].x, hv[3].y, hv[3].z, hv[3].w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 g = bf16x2_to_f2(o[i]);
          const float2 x = bf16x2_to_f2(hw[i]);
          const GeluCP c0 = gelu_cdf_pdf(x.x), c1 = gelu_cdf_pdf(x.y);
          o[i] = pack_bf16x2(g.x * (c0.cdf + x.x * c0.pdf), g.y * (c1.cdf + x.y * c1.pdf));
        }
      }
      stage_store(o, &tmC, n_col, m0);
      if constexpr (EPI == kEpiGeluFwd) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = bf16x2_to_f2(o[i]);
          o[i] = pack_bf16x2(x.x * gelu_cdf_pdf(x.x).cdf, x.y * gelu_cdf_pdf(x.y).cdf);
        }
        stage_store(o, &tmC2, n_col, m0);
      }
    };
    PairWork pw;
    for (int w = 0; ok && pair_work(args, cluster_id, num_clusters, w, main_k_tiles, pw); ++w, ++it) {
      int tm, tn;
      pair_tile_coords(args, pw.tile, AG, tm, tn);
      const int buf = it & 1;
      const bool got = mbar_wait(&tfull_bar[buf], (it >> 1) & 1, args.status, kErrEpi);
      if (!named_barrier_and(1, 128, got)) { ok = false; break; }  // same decision in all 128
      tc_fence_after();
      const int m0 = tm * (2 * kBM) + (int)cr * kBM;
      const int n0 = tn * BN;
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
      if (EPI == kEpiRope && pw.sk < 0) {
        // pairs of chunks (c, c + 2) of each 128-wide head: x1 = cols i, x2 = i + 64
        const float2* cs = args.epi_cs + (int64_t)((m0 + row) % args.epi_S) * 64;
        const uint4 none[4] = {};
#pragma unroll 1
        for (int hp = 0; hp < BN / 64; ++hp) {
          const int c0 = (hp >> 1) * 4 + (hp & 1), c1 = c0 + 2;
          float4 t[16];   // (cos, sin) of pairs (hp & 1) * 32 + 0..31
          const float4* cs4 = reinterpret_cast<const float4*>(cs + (hp & 1) * 32);
#pragma unroll
          for (int i = 0; i < 16; ++i) t[i] = __ldg(cs4 + i);
          uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(trow + (uint32_t)(c0 * 32), ra);
          tmem_ld_32x32b_x32(trow + (uint32_t)(c1 * 32), rb);
          tmem_ld_wait();
          float oa[32], ob[32];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 a = bf16x2_to_f2(pack_bf16x2(__uint_as_float(ra[i]), __uint_as_float(ra[i + 1])));
            const float2 b = bf16x2_to_f2(pack_bf16x2(__uint_as_float(rb[i]), __uint_as_float(rb[i + 1])));
            const float4 v = t[i >> 1];  // (cos, sin) of pairs i and i + 1
            oa[i] = rope_lo(a.x, b.x, v.x, v.y);
            ob[i] = rope_hi(a.x, b.x, v.x, v.y);
            oa[i + 1] = rope_lo(a.y, b.y, v.z, v.w);
            ob[i + 1] = rope_hi(a.y, b.y, v.z, v.w);
          }
          if (n0 + c0 * 32 < args.epi_ncols) {
            store_chunk(oa, n0 + c0 * 32, m0, none, none);
            store_chunk(ob, n0 + c1 * 32, m0, none, none);
          } else {  // a head past the rotated columns (v of a fused q/k/v GEMM): as is
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              oa[i] = __uint_as_float(ra[i]);
              ob[i] = __uint_as_float(rb[i]);
            }
            store_chunk(oa, n0 + c0 * 32, m0, none, none);
            store_chunk(ob, n0 + c1 * 32, m0, none, none);
          }
        }
      } else if (pw.sk < 0) {
        uint4 hnext[4] = {}, hnext2[4] = {};
        load_h(n0, m0, hnext, hnext2);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint4 hv[4], hv2[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            hv[j] = hnext[j];
            hv2[j] = hnext2[j];
          }
          // the next chunk's epilogue-input loads overlap this chunk's work
          if (c + 1 < BN / 32) load_h(n0 + (c + 1) * 32, m0, hnext, hnext2);
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + (uint32_t)(c * 32), r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          store_chunk(v, n0 + c * 32, m0, hv, hv2);
        }
      } else {
        // stream-K part: add this part's fp32 block into the tile's accumulation
        // buffer (vector reductions, no return), then arrive at the tile's counter
        const int S = args.sk_splits;
        float* acc = args.sk_ws + ((size_t)pw.sk * 2 + cr) * ((size_t)128 * BN) + (size_t)row * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + (uint32_t)(c * 32), r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            red_add_v4_f32(acc + c * 32 + 4 * i, __uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                           __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        }
        __threadfence();                 // this part's additions done before the arrival below
        named_barrier(1, 128);
        if (leader_thread) {
          int* cnt = args.sk_cnt + pw.sk * 2 + cr;
          const int old = atomicAdd(cnt, 1);
          sk_last = old == S - 1;
          if (old == S - 1) *cnt = 0;    // every part has arrived: reset for the next GEMM
        }
        named_barrier(1, 128);
        if (sk_last) {
          __threadfence();               // acquire the other parts' additions
#pragma unroll 1
          for (int c = 0; c < BN / 32; c += 2) {   // two chunks per round trip
            float4 x[16];
            const float4* src = reinterpret_cast<const float4*>(acc + c * 32);
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = __ldcg(src + i);
            float4* z = reinterpret_cast<float4*>(acc + c * 32);
#pragma unroll
            for (int i = 0; i < 16; ++i) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);  // clean for the next GEMM
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint4 hv[4] = {}, hv2[4] = {};
              load_h(n0 + (c + h2) * 32, m0, hv, hv2);
              float v[32];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                v[4 * i] = x[8 * h2 + i].x;
                v[4 * i + 1] = x[8 * h2 + i].y;
                v[4 * i + 2] = x[8 * h2 + i].z;
                v[4 * i + 3] = x[8 * h2 + i].w;
              }
              store_chunk(v, n0 + (c + h2) * 32, m0, hv, hv2);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(map_to_cta(smem_u32(&tempty_bar[buf]), 0));
    }
    if (leader_thread) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its pair may still touch its smem/TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
  if (AG && threadIdx.x == 0) {
    // every warp of this CTA is done with the counters; the last CTA out resets them
    __threadfence();
    if (atomicAdd(args.ag_sync + kAgExit, 1) == (int)gridDim.x - 1) {
      __threadfence();
      for (int t = 0; t < args.tiles_n; ++t) args.ag_sync[t] = 0;
      args.ag_sync[kAgClaim] = 0;
      args.ag_sync[kAgExit] = 0;
    }
  }
}

// ----------------------------------------------------------------------------
// NF4 -> bf16 operand producers (memory-bound).  `transpose=false` writes
// W [N,K] as is; `transpose=true` writes Wᵀ [K,N] (for the input-gradient GEMM)
// through a 64x64 shared-memory tile so both the packed reads and the bf16
// writes stay coalesced.
// ----------------------------------------------------------------------------
// 64x64 tile per CTA of 256 threads; each thread expands 16 values (8 bytes).
__global__ void __launch_bounds__(256) nf4_to_bf16_tile_kernel(
    const uint8_t* __restrict__ packed, const float* __restrict__ absmax,
    __nv_bfloat16* __restrict__ out, int rows, int cols, int blocksize, int qtype, int transpose) {
  __shared__ float lut[16];
  __shared__ __align__(16) __nv_bfloat16 tile[64][64 + 8];
  if (threadIdx.x < 16) lut[threadIdx.x] = qtype == 0 ? c_code_nf4[threadIdx.x] : c_code_fp4[threadIdx.x];
  __syncthreads();
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const int tr = threadIdx.x >> 2;         // 0..63 row in tile
  const int tc = (threadIdx.x & 3) * 16;   // 0,16,32,48
  const int r = r0 + tr, c = c0 + tc;
  float v[16];
  if (r < rows && c + 16 <= cols) {
    const int64_t e0 = (int64_t)r * cols + c;
    const uint2 p = *reinterpret_cast<const uint2*>(packed + (e0 >> 1));
    const float s = absmax[e0 / blocksize];
    const uint32_t w[2] = {p.x, p.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFF;
      v[2 * i] = lut[byte >> 4] * s;
      v[2 * i + 1] = lut[byte & 0xF] * s;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = 0.0f;
      const int cc = c + i;
      if (r < rows && cc < cols) {
        const int64_t e = (int64_t)r * cols + cc;
        const uint32_t byte = packed[e >> 1];
        const uint32_t qv = (e & 1) ? (byte & 0xF) : (byte >> 4);
        v[i] = lut[qv] * absmax[e / blocksize];
      }
    }
  }
  if (!transpose) {
    if (r < rows) {
      if (c + 16 <= cols) {
        uint4 o0, o1;
        o0.x = pack_bf16x2(v[0], v[1]);   o0.y = pack_bf16x2(v[2], v[3]);
        o0.z = pack_bf16x2(v[4], v[5]);   o0.w = pack_bf16x2(v[6], v[7]);
        o1.x = pack_bf16x2(v[8], v[9]);   o1.y = pack_bf16x2(v[10], v[11]);
        o1.z = pack_bf16x2(v[12], v[13]); o1.w = pack_bf16x2(v[14], v[15]);
        uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)r * cols + c);
        dst[0] = o0;
        dst[1] = o1;
      } else {
        for (int i = 0; i < 16 && c + i < cols; ++i) out[(int64_t)r * cols + c + i] = __float2bfloat16_rn(v[i]);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) tile[tc + i][tr] = __float2bfloat16_rn(v[i]);
  __syncthreads();
  // write Wᵀ: out row = source column, 64 contiguous source rows per out row
  const int oc = c0 + tr;           // out row (source column)
  const int orow0 = r0 + tc;        // out column start (source row)
  if (oc < cols) {
    __nv_bfloat16* dst = out + (int64_t)oc * rows + orow0;
    if (orow0 + 16 <= rows) {
      uint4 o0, o1;
      const uint32_t* s = reinterpret_cast<const uint32_t*>(&tile[tr][tc]);
      o0 = make_uint4(s[0], s[1], s[2], s[3]);
      o1 = make_uint4(s[4], s[5], s[6], s[7]);
      reinterpret_cast<uint4*>(dst)[0] = o0;
      reinterpret_cast<uint4*>(dst)[1] = o1;
    } else {
      for (int i = 0; i < 16 && orow0 + i < rows; ++i) dst[i] = tile[tr][tc + i];
    }
  }
}

}  // namespace zq

using namespace zq;

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

// 2-D bf16 row-major [rows, cols] tensor map with a box of [box_rows, 64] and 128-B swizzle
static CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems,
                                  int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

// [rows, cols] bf16 output tensor map for the epilogue's TMA store: box of 128
// rows x 32 columns, 64-byte swizzle (matches the staging tile layout)
static CUtensorMap make_tmap_store_bf16(const void* base, int64_t rows, int64_t cols,
                                        int64_t row_stride_elems) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA store base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA store row pitch must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * 2)};
  cuuint32_t box[2] = {32u, 128u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store) failed with code ", (int)r);
  return map;
}

// Stream-K state, one zeroed set per (device, stream): arrival counters and the
// fp32 accumulation blocks (kSkMaxTiles tiles x 2 CTAs x 128 x 256).  GEMMs on
// one stream run in order, so no two running GEMMs share them; the last part of
// a tile resets its counter and zeroes its blocks.
constexpr int kSkMaxTiles = 64;
static int* sk_counters(int device, cudaStream_t stream, float** acc) {
  struct State { int* cnt; float* acc; };
  static std::map<std::pair<int, cudaStream_t>, State> bufs;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  State& st = bufs[{device, stream}];
  if (st.cnt == nullptr) {
    const size_t acc_bytes = (size_t)kSkMaxTiles * 2 * 128 * 256 * sizeof(float);
    C10_CUDA_CHECK(cudaMalloc(&st.cnt, 2 * kSkMaxTiles * sizeof(int)));
    C10_CUDA_CHECK(cudaMalloc(&st.acc, acc_bytes));
    C10_CUDA_CHECK(cudaMemsetAsync(st.cnt, 0, 2 * kSkMaxTiles * sizeof(int), stream));
    C10_CUDA_CHECK(cudaMemsetAsync(st.acc, 0, acc_bytes, stream));
  }
  *acc = st.acc;
  return st.cnt;
}

DeviceStatus* status_buffer(int device) {
  static DeviceStatus* bufs[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (bufs[device] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&bufs[device], sizeof(DeviceStatus)));
    C10_CUDA_CHECK(cudaMemset(bufs[device], 0, sizeof(DeviceStatus)));
  }
  return bufs[device];
}

// Returns and clears the device error status (code, detail) of the GEMM kernels.
std::vector<int64_t> gemm_status(int64_t device) {
  DeviceStatus h{0, 0};
  DeviceStatus* d = status_buffer((int)device);
  C10_CUDA_CHECK(cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost));
  C10_CUDA_CHECK(cudaMemset(d, 0, sizeof(DeviceStatus)));
  return {h.code, h.detail};
}

template <int BN, int STAGES>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                        const CUtensorMap& tb2, GemmArgs args, cudaStream_t stream, int sms) {
  using L = GemmSmem<BN, STAGES>;
  static bool configured[64] = {false};
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_tn_kernel<BN, STAGES>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[dev] = true;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  const int grid = std::min(tiles, sms);
  gemm_tn_kernel<BN, STAGES><<<grid, kGemmThreads, L::kBytes, stream>>>(ta, tb, ta2, tb2, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, int STAGES, int KB, bool BMN, bool Q4 = false, bool AG = false, int EPI = kEpiPlain>
static void launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                             const CUtensorMap& tb2, const CUtensorMap& tc, GemmArgs args,
                             cudaStream_t stream, int sms, const CUtensorMap* tc2 = nullptr) {
  using L = PairSmem<BN, STAGES, KB>;
  static bool configured[64] = {false};
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_tn_pair_kernel<BN, STAGES, KB, BMN, Q4, AG, EPI>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    configured[dev] = true;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  const int clusters = std::max(1, std::min(tiles, sms / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3((Q4 || AG) ? kGemmQ4Threads : kGemmThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tn_pair_kernel<BN, STAGES, KB, BMN, Q4, AG, EPI>, ta, tb, ta2,
                                    tb2, tc, tc2 != nullptr ? *tc2 : tc, args));
}

// Pick the N tile that minimises wave quantisation over the SMs.
static int choose_bn(int M, int N, int sms) {
  const int tm = (M + kBM - 1) / kBM;
  double best = 1e30;
  int best_bn = 256;
  for (int bn : {256, 192, 128}) {
    const int tn = (N + bn - 1) / bn;
    const int tiles = tm * tn;
    const int waves = (tiles + sms - 1) / sms;
    // cost ~ waves * per-tile time (proportional to bn); small penalty for narrow tiles
    const double cost = (double)waves * bn * (bn == 128 ? 1.15 : 1.0);
    if (cost < best - 1e-9) { best = cost; best_bn = bn; }
  }
  return best_bn;
}

// Stream-K tail: when the last wave of tiles would leave more than half the
// clusters idle, split its tiles along K over the clusters (ZEROQ_STREAMK=0: off).
static void setup_streamk(GemmArgs& args, int main_k, int sms, int dev, cudaStream_t stream) {
  static const bool sk_on = [] {
    const char* e = std::getenv("ZEROQ_STREAMK");
    return e == nullptr || std::atoi(e) != 0;
  }();
  const int tiles = args.tiles_m * args.tiles_n;
  const int C = std::max(1, std::min(tiles, sms / 2));
  const int full = tiles / C, r = tiles % C;
  // the split costs ~25 us (fp32 reductions, fence, fix-up): measured on B200 it
  // pays off from ~48 pipeline stages per tile (8192 x 3072 x 12288: -7%)
  // and loses below (8192 x 3072 x 3072: +9%)
  if (sk_on && r > 0 && full >= 1 && 2 * r <= C && r <= kSkMaxTiles && main_k >= 48) {
    const int S = std::min(C / r, main_k / 2);
    if (S >= 2) {
      args.sk_first = full * C;
      args.sk_tiles = r;
      args.sk_splits = S;
      args.sk_cnt = sk_counters(dev, stream, &args.sk_ws);
    }
  }
}

static int g_pair_mode = 1;  // 1: use the CTA-pair kernel when M >= 256 (set_gemm_pair_mode)

// CTA-pair tiles are 256 x BN; BN in {256, 192, 128} (BN/2 rows of B per CTA)
static int choose_bn_pair(int M, int N, int sms) {
  const int tm = (M + 2 * kBM - 1) / (2 * kBM);
  const int pairs = std::max(1, sms / 2);
  double best = 1e30;
  int best_bn = 256;
  // measured on B200: 256x192 pair tiles run slower per tile than 256x256, so
  // only 256 and 128 are considered
  for (int bn : {256, 128}) {
    const int tn = (N + bn - 1) / bn;
    const int waves = (tm * tn + pairs - 1) / pairs;
    const double cost = (double)waves * bn * (bn == 128 ? 1.1 : 1.0);
    if (cost < best - 1e-9) { best = cost; best_bn = bn; }
  }
  return best_bn;
}

void set_gemm_pair_mode(int64_t mode) { g_pair_mode = (int)mode; }

// b_mn = false: B is [N, K] row-major (C = A·Bᵀ); true: B is [K, N] row-major (C = A·B)
static void gemm_impl(const at::Tensor& a, const at::Tensor& b, at::Tensor& c,
                      const c10::optional<at::Tensor>& a2, const c10::optional<at::Tensor>& b2,
                      bool b_mn = false, int epi = kEpiPlain, const at::Tensor* aux = nullptr,
                      int64_t rope_ncols = -1, const at::Tensor* aux2 = nullptr,
                      const at::Tensor* c2 = nullptr) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 &&
                  c.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm: 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm: row-major operands");
  const int64_t M = a.size(0), K = a.size(1), N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: K mismatch");
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "gemm: C shape");
  TORCH_CHECK(K % 64 == 0 && K > 0, "gemm: K must be a positive multiple of 64");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) == 0 && (c.stride(0) % 8) == 0,
              "gemm: C must be 16-byte aligned with a row pitch multiple of 8");
  TORCH_CHECK(M < (1LL << 31) && N < (1LL << 31), "gemm: dims too large");
  const at::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const bool pair = (g_pair_mode != 0 || b_mn) && M >= 2 * kBM;
  TORCH_CHECK(!b_mn || pair, "gemm: B as [K, N] needs M >= 256");
  TORCH_CHECK(!b_mn || N % 64 == 0, "gemm: B as [K, N] needs N % 64 == 0");
  const int bn = pair ? choose_bn_pair((int)M, (int)N, sms) : choose_bn((int)M, (int)N, sms);

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.extra_k16 = 0;
  args.tiles_m = pair ? (int)((M + 2 * kBM - 1) / (2 * kBM)) : (int)((M + kBM - 1) / kBM);
  args.tiles_n = (int)((N + bn - 1) / bn);
  args.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr<at::BFloat16>());
  args.ldc = c.stride(0);
  args.status = status_buffer(dev);

  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), kBM);
  const int b_box = pair ? bn / 2 : bn;
  // [K, N] operands are read as boxes of 64 N-columns x 64 K-rows
  CUtensorMap tb = b_mn ? make_tmap_bf16(b.data_ptr(), K, N, b.stride(0), 64)
                        : make_tmap_bf16(b.data_ptr(), N, K, b.stride(0), b_box);
  CUtensorMap ta2 = ta, tb2 = tb;
  if (a2.has_value() && a2->defined()) {
    TORCH_CHECK(b2.has_value() && b2->defined(), "gemm: extra slab needs both operands");
    const at::Tensor& x2 = *a2;
    const at::Tensor& y2 = *b2;
    TORCH_CHECK(x2.scalar_type() == at::kBFloat16 && y2.scalar_type() == at::kBFloat16, "extra slab bf16");
    // width 64 everywhere; 128, 192 or 256 (one stage per 64 columns) on the pair kernel
    const int64_t E = x2.size(1);
    TORCH_CHECK(E == 64 || (E % 64 == 0 && E <= 256 && pair),
                "extra slab width must be 64 (or 128/192/256 on the CTA-pair kernel, M >= 256)");
    if (b_mn) {
      TORCH_CHECK(x2.size(0) == M && y2.size(0) == E && y2.size(1) == N &&
                      x2.stride(1) == 1 && y2.stride(1) == 1,
                  "extra slab operands must be [M,E] and [E,N] row-major");
    } else {
      TORCH_CHECK(x2.size(0) == M && y2.size(0) == N && y2.size(1) == E &&
                      x2.stride(1) == 1 && y2.stride(1) == 1,
                  "extra slab operands must be [M,E] and [N,E] row-major");
    }
    ta2 = make_tmap_bf16(x2.data_ptr(), M, E, x2.stride(0), kBM);
    tb2 = b_mn ? make_tmap_bf16(y2.data_ptr(), E, N, y2.stride(0), 64)
               : make_tmap_bf16(y2.data_ptr(), N, E, y2.stride(0), b_box);
    args.extra_k16 = (int)(E / 16);
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(epi == kEpiPlain || (pair && K % 128 == 0 && aux != nullptr),
              "gemm: fused epilogues need M >= 256, K % 128 == 0 and the auxiliary tensor");
  if (pair) {
    const CUtensorMap tc = make_tmap_store_bf16(c.data_ptr(), M, N, c.stride(0));
    const bool k128 = (K % 128) == 0;
    // (the SwiGLU epilogues take their shapes' many waves without a stream-K tail)
    if (epi != kEpiRope && epi != kEpiSwigluFwd && epi != kEpiSwigluBwd)
      setup_streamk(args, (int)(K / (k128 ? 128 : 64)), sms, dev, stream);
    if (epi == kEpiRope) {
      const at::Tensor& t = *aux;
      TORCH_CHECK(!b_mn && N % 128 == 0, "gemm: the RoPE epilogue needs [N, K] weights and 128-wide heads");
      TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && t.dim() == 3 && t.size(1) == 64 &&
                      t.size(2) == 2 && M % t.size(0) == 0,
                  "gemm: RoPE table must be fp32 [S, 64, 2] with M a multiple of S");
      args.epi_cs = reinterpret_cast<const float2*>(t.data_ptr<float>());
      args.epi_S = (int)t.size(0);
      args.epi_ncols = rope_ncols < 0 ? (int)N : (int)rope_ncols;
      TORCH_CHECK(args.epi_ncols % 128 == 0, "gemm: rotated columns must be whole 128-wide heads");
      if (bn == 256) launch_gemm_pair<256, 3, 2, false, false, false, kEpiRope>(ta, tb, ta2, tb2, tc, args, stream, sms);
      else launch_gemm_pair<128, 4, 2, false, false, false, kEpiRope>(ta, tb, ta2, tb2, tc, args, stream, sms);
      return;
    }
    auto check_mn = [&](const at::Tensor& x) {
      TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(0) == M &&
                      x.size(1) == N && x.stride(1) == 1 && (x.stride(0) % 8) == 0 &&
                      (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0,
                  "gemm: epilogue tensors must be bf16 [M, N], 16-byte aligned rows");
    };
    if (epi == kEpiSwigluFwd || epi == kEpiSwigluBwd) {
      TORCH_CHECK(c2 != nullptr, "gemm: the SwiGLU epilogues need a second output");
      check_mn(*aux);
      check_mn(*c2);
      args.epi_src = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr<at::BFloat16>());
      args.epi_ld = aux->stride(0);
      const CUtensorMap tc2 = make_tmap_store_bf16(c2->data_ptr(), M, N, c2->stride(0));
      if (epi == kEpiSwigluFwd) {
        TORCH_CHECK(!b_mn, "gemm: the SwiGLU-output epilogue is for the [N, K] weight layout");
        if (bn == 256) launch_gemm_pair<256, 3, 2, false, false, false, kEpiSwigluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
        else launch_gemm_pair<128, 4, 2, false, false, false, kEpiSwigluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
      } else {
        TORCH_CHECK(b_mn && aux2 != nullptr, "gemm: the SwiGLU-gradient epilogue is for the [K, N] "
                    "weight layout and needs g and u");
        check_mn(*aux2);
        args.epi_src2 = reinterpret_cast<const __nv_bfloat16*>(aux2->data_ptr<at::BFloat16>());
        args.epi_ld2 = aux2->stride(0);
        if (bn == 256) launch_gemm_pair<256, 3, 2, true, false, false, kEpiSwigluBwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
        else launch_gemm_pair<128, 4, 2, true, false, false, kEpiSwigluBwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
      }
      return;
    }
    if (epi != kEpiPlain) {
      const at::Tensor& x = *aux;
      check_mn(x);
      if (epi == kEpiGeluFwd) {
        TORCH_CHECK(!b_mn, "gemm: the GELU-output epilogue is for the [N, K] weight layout");
        const CUtensorMap tc2 = make_tmap_store_bf16(x.data_ptr(), M, N, x.stride(0));
        if (bn == 256) launch_gemm_pair<256, 3, 2, false, false, false, kEpiGeluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
        else launch_gemm_pair<128, 4, 2, false, false, false, kEpiGeluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
      } else {
        TORCH_CHECK(b_mn, "gemm: the GELU-gradient epilogue is for the [K, N] weight layout");
        args.epi_src = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
        args.epi_ld = x.stride(0);
        if (bn == 256) launch_gemm_pair<256, 3, 2, true, false, false, kEpiGeluBwd>(ta, tb, ta2, tb2, tc, args, stream, sms);
        else launch_gemm_pair<128, 4, 2, true, false, false, kEpiGeluBwd>(ta, tb, ta2, tb2, tc, args, stream, sms);
      }
      return;
    }
    if (b_mn) {
      if (bn == 256) {
        if (k128) launch_gemm_pair<256, 3, 2, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
        else launch_gemm_pair<256, 6, 1, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
      } else {
        if (k128) launch_gemm_pair<128, 4, 2, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
        else launch_gemm_pair<128, 8, 1, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
      }
      return;
    }
    if (bn == 256) {
      if (k128) launch_gemm_pair<256, 3, 2, false>(ta, tb, ta2, tb2, tc, args, stream, sms);
      else launch_gemm_pair<256, 6, 1, false>(ta, tb, ta2, tb2, tc, args, stream, sms);
    } else {
      if (k128) launch_gemm_pair<128, 4, 2, false>(ta, tb, ta2, tb2, tc, args, stream, sms);
      else launch_gemm_pair<128, 8, 1, false>(ta, tb, ta2, tb2, tc, args, stream, sms);
    }
    return;
  }
  if (bn == 256) launch_gemm<256, 4>(ta, tb, ta2, tb2, args, stream, sms);
  else if (bn == 192) launch_gemm<192, 5>(ta, tb, ta2, tb2, args, stream, sms);
  else launch_gemm<128, 6>(ta, tb, ta2, tb2, args, stream, sms);
}

void gemm_bf16_tn(at::Tensor a, at::Tensor b, at::Tensor c) {
  gemm_impl(a, b, c, c10::nullopt, c10::nullopt);
}

void gemm_bf16_tn_extra(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor a2, at::Tensor b2) {
  gemm_impl(a, b, c, a2, b2);
}

// C[M,N] = A[M,K] · B[K,N] (+ A2[M,64] · B2[64,N]); B read MN-major by the tensor core
void gemm_bf16_nn(at::Tensor a, at::Tensor b, at::Tensor c, c10::optional<at::Tensor> a2,
                  c10::optional<at::Tensor> b2) {
  gemm_impl(a, b, c, a2, b2, true);
}

// GEMM with the GELU epilogues (needs M >= 256 and K % 128 == 0):
//   b_mn = false: H = A·Bᵀ (+ A2·B2ᵀ) stored in c and GELU(H) in aux;
//   b_mn = true:  c = (A·B (+ A2·B2)) * GELU'(aux), aux = the pre-activation.
void gemm_gelu(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor aux, bool b_mn,
               c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2) {
  gemm_impl(a, b, c, a2, b2, b_mn, b_mn ? kEpiGeluBwd : kEpiGeluFwd, &aux);
}

// GEMM with the SwiGLU epilogues (needs M >= 256 and K % 128 == 0):
//   b_mn = false: c = U = A·Bᵀ (+ A2·B2ᵀ) and c2 = silu(g)·U   (u unused);
//   b_mn = true:  D = A·B (+ A2·B2); c = D·u·silu'(g) (dg), c2 = D·silu(g) (du).
void gemm_swiglu(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor c2, at::Tensor g,
                 c10::optional<at::Tensor> u, bool b_mn, c10::optional<at::Tensor> a2,
                 c10::optional<at::Tensor> b2) {
  const at::Tensor* up = (u.has_value() && u->defined()) ? &*u : nullptr;
  gemm_impl(a, b, c, a2, b2, b_mn, b_mn ? kEpiSwigluBwd : kEpiSwigluFwd, &g, -1, up, &c2);
}

// C = rope(A·Bᵀ (+ A2·B2ᵀ)) for 128-wide heads; cs: fp32 [S, 64, 2] (cos, sin) per
// position and pair, row m of C at position m % S; only columns [0, ncols) are
// rotated (ncols < 0: all).  Needs M >= 256, K % 128 == 0.
void gemm_rope(at::Tensor a, at::Tensor b, at::Tensor c, at::Tensor cs,
               c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2, int64_t ncols) {
  gemm_impl(a, b, c, a2, b2, false, kEpiRope, &cs, ncols);
}

// GEMM whose B operand is a 4-bit weight W [rows, cols] decoded inside the
// kernel (no bf16 copy of W exists at any time):
//   w_is_kn = false:  C[M, rows] = A[M, cols] · Wᵀ   (forward,        K-major B)
//   w_is_kn = true:   C[M, cols] = A[M, rows] · W    (input gradient, MN-major B)
// plus the optional extra 64-wide K slab A2 · B2 (same shapes as gemm_bf16_tn_extra /
// gemm_bf16_nn).  Needs M >= 256, K % 128 == 0, N % 64 == 0, cols % 32 == 0 and a
// block size that is a multiple of 32.
void gemm_nf4(at::Tensor a, at::Tensor packed, at::Tensor absmax, int64_t rows, int64_t cols,
              int64_t blocksize, int64_t quant_type, bool w_is_kn, at::Tensor c,
              c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2) {
  TORCH_CHECK(a.is_cuda() && c.is_cuda() && packed.is_cuda() && absmax.is_cuda(), "gemm_nf4: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16, "gemm_nf4: bf16 A and C");
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.is_contiguous() && packed.numel() * 2 == rows * cols,
              "gemm_nf4: packed must be contiguous uint8 with rows*cols/2 bytes");
  TORCH_CHECK(absmax.scalar_type() == at::kFloat && absmax.is_contiguous() && blocksize > 0 &&
                  blocksize % 32 == 0 && absmax.numel() * blocksize >= rows * cols,
              "gemm_nf4: fp32 absmax per block (block size a multiple of 32)");
  TORCH_CHECK(quant_type == 0 || quant_type == 1, "gemm_nf4: quant_type 0 (nf4) or 1 (fp4)");
  TORCH_CHECK(cols % 32 == 0 && (reinterpret_cast<uintptr_t>(packed.data_ptr()) & 15) == 0,
              "gemm_nf4: cols % 32 == 0 and 16-byte aligned packed data");
  TORCH_CHECK(a.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && c.stride(1) == 1, "gemm_nf4: row-major A, C");
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = w_is_kn ? cols : rows;
  TORCH_CHECK(K == (w_is_kn ? rows : cols), "gemm_nf4: K mismatch");
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "gemm_nf4: C shape");
  TORCH_CHECK(M >= 2 * kBM && M < (1LL << 31), "gemm_nf4: needs M >= 256");
  TORCH_CHECK(K % 128 == 0 && N % 64 == 0, "gemm_nf4: needs K % 128 == 0 and N % 64 == 0");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) == 0 && (c.stride(0) % 8) == 0,
              "gemm_nf4: C must be 16-byte aligned with a row pitch multiple of 8");
  TORCH_CHECK(rows < (1LL << 31) && cols < (1LL << 31), "gemm_nf4: weight too large");
  const at::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  constexpr int bn = 256;

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + 2 * kBM - 1) / (2 * kBM));
  args.tiles_n = (int)((N + bn - 1) / bn);
  args.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr<at::BFloat16>());
  args.ldc = c.stride(0);
  args.status = status_buffer(dev);
  args.q_packed = packed.data_ptr<uint8_t>();
  args.q_absmax = absmax.data_ptr<float>();
  args.q_rows = (int)rows;
  args.q_cols = (int)cols;
  args.q_block = (int)blocksize;
  args.q_type = (int)quant_type;

  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), kBM);
  CUtensorMap ta2 = ta, tb2 = ta;
  if (a2.has_value() && a2->defined()) {
    TORCH_CHECK(b2.has_value() && b2->defined(), "gemm_nf4: extra slab needs both operands");
    const at::Tensor& x2 = *a2;
    const at::Tensor& y2 = *b2;
    TORCH_CHECK(x2.scalar_type() == at::kBFloat16 && y2.scalar_type() == at::kBFloat16, "extra slab bf16");
    if (w_is_kn) {
      TORCH_CHECK(x2.size(0) == M && x2.size(1) == 64 && y2.size(0) == 64 && y2.size(1) == N &&
                      x2.stride(1) == 1 && y2.stride(1) == 1,
                  "extra slab operands must be [M,64] and [64,N] row-major");
      tb2 = make_tmap_bf16(y2.data_ptr(), 64, N, y2.stride(0), 64);
    } else {
      TORCH_CHECK(x2.size(0) == M && y2.size(0) == N && x2.size(1) == 64 && y2.size(1) == 64 &&
                      x2.stride(1) == 1 && y2.stride(1) == 1,
                  "extra slab operands must be [M,64] and [N,64] row-major");
      tb2 = make_tmap_bf16(y2.data_ptr(), N, 64, y2.stride(0), bn / 2);
    }
    ta2 = make_tmap_bf16(x2.data_ptr(), M, 64, x2.stride(0), kBM);
    args.extra_k16 = 4;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  const CUtensorMap tc = make_tmap_store_bf16(c.data_ptr(), M, N, c.stride(0));
  if (w_is_kn) launch_gemm_pair<256, 3, 2, true, true>(ta, ta, ta2, tb2, tc, args, stream, sms);
  else launch_gemm_pair<256, 3, 2, false, true>(ta, ta, ta2, tb2, tc, args, stream, sms);
}

// Gather-mode counters, one zeroed set per (device, stream); the kernel's last
// CTA resets them, so consecutive launches on a stream reuse them.
static int* ag_sync_buffer(int device, cudaStream_t stream) {
  static std::map<std::pair<int, cudaStream_t>, int*> bufs;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  int*& p = bufs[{device, stream}];
  if (p == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&p, kAgSyncWords * sizeof(int)));
    C10_CUDA_CHECK(cudaMemsetAsync(p, 0, kAgSyncWords * sizeof(int), stream));
  }
  return p;
}

// C[M, N] = A[M, K] · Wᵀ (+ A2[M, 64] · B2[N, 64]) where W [N, K] is a 4-bit
// weight split over the ranks of the node: rank q holds packed bytes
// [pstarts[q], pstarts[q+1]) at device address psrc[q] and absmax entries
// [astarts[q], astarts[q+1]) at asrc[q] (addresses valid in this process: this
// rank's own memory or CUDA IPC mappings of the peers').  One kernel gathers
// and dequantises W into wbuf (bf16 [N, K], left assembled for the caller) and
// multiplies it with tcgen05, each N tile starting as soon as its rows are in.
static void ag_gemm_impl(int kind, at::Tensor a, std::vector<int64_t> psrc, std::vector<int64_t> pstarts,
                         std::vector<int64_t> asrc, std::vector<int64_t> astarts, int64_t packed_total,
                         int64_t absmax_total, int64_t rank, int64_t N, int64_t K, int64_t blocksize,
                         int64_t quant_type, at::Tensor wbuf, at::Tensor c, c10::optional<at::Tensor> a2,
                         c10::optional<at::Tensor> b2, const at::Tensor* swiglu_g = nullptr,
                         const at::Tensor* swiglu_out = nullptr) {
  const int world = (int)psrc.size();
  TORCH_CHECK(world >= 1 && world <= kAgMaxRanks && (int)pstarts.size() == world &&
                  (int)asrc.size() == world && (int)astarts.size() == world,
              "ag_gemm_nf4: one pointer and start per rank (at most 8 ranks)");
  TORCH_CHECK(rank >= 0 && rank < world, "ag_gemm_nf4: rank out of range");
  TORCH_CHECK(a.is_cuda() && c.is_cuda() && wbuf.is_cuda(), "ag_gemm_nf4: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16 &&
                  wbuf.scalar_type() == at::kBFloat16, "ag_gemm_nf4: bf16 A, C and W buffer");
  TORCH_CHECK(a.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && c.stride(1) == 1,
              "ag_gemm_nf4: row-major A and C");
  const int64_t M = a.size(0);
  TORCH_CHECK(a.size(1) == K && c.size(0) == M && c.size(1) == N, "ag_gemm_nf4: shapes");
  TORCH_CHECK(M >= 2 * kBM && M < (1LL << 31) && N < (1LL << 31), "ag_gemm_nf4: needs M >= 256");
  TORCH_CHECK(K % 128 == 0 && N % 8 == 0, "ag_gemm_nf4: needs K % 128 == 0 and N % 8 == 0");
  if (kind == kAgNf4) {
    TORCH_CHECK(blocksize > 0 && blocksize % 32 == 0, "ag_gemm_nf4: block size a multiple of 32");
    TORCH_CHECK(quant_type == 0 || quant_type == 1, "ag_gemm_nf4: quant_type 0 (nf4) or 1 (fp4)");
    TORCH_CHECK(packed_total * 2 == N * K && absmax_total * blocksize >= N * K,
                "ag_gemm_nf4: packed/absmax totals do not cover W");
  } else {
    TORCH_CHECK(packed_total >= N * K, "ag_gemm_f32: the pieces do not cover W");
  }
  TORCH_CHECK(wbuf.is_contiguous() && wbuf.numel() == N * K &&
                  (reinterpret_cast<uintptr_t>(wbuf.data_ptr()) & 15) == 0,
              "ag_gemm_nf4: W buffer must be contiguous, N*K elements, 16-byte aligned");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) == 0 && (c.stride(0) % 8) == 0,
              "ag_gemm_nf4: C must be 16-byte aligned with a row pitch multiple of 8");
  for (int q = 0; q < world; ++q) {
    const int64_t pend = q + 1 < world ? pstarts[q + 1] : packed_total;
    const int64_t aend = q + 1 < world ? astarts[q + 1] : absmax_total;
    TORCH_CHECK(pstarts[q] >= 0 && pstarts[q] <= pend && astarts[q] >= 0 && astarts[q] <= aend,
                "ag_gemm_nf4: starts must be non-decreasing");
    TORCH_CHECK(pend == pstarts[q] || psrc[q] != 0, "ag_gemm_nf4: null shard pointer");
    TORCH_CHECK(kind == kAgF32 || aend == astarts[q] || (asrc[q] != 0 && (asrc[q] & 3) == 0),
                "ag_gemm_nf4: absmax pointers must be 4-byte aligned");
    TORCH_CHECK(kind == kAgNf4 || pend == pstarts[q] || (psrc[q] & 3) == 0,
                "ag_gemm_f32: fp32 pieces must be 4-byte aligned");
  }
  const at::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int bn = choose_bn_pair((int)M, (int)N, sms);

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + 2 * kBM - 1) / (2 * kBM));
  args.tiles_n = (int)((N + bn - 1) / bn);
  TORCH_CHECK(args.tiles_n <= kAgMaxTilesN, "ag_gemm_nf4: N too large");
  args.C = reinterpret_cast<__nv_bfloat16*>(c.data_ptr<at::BFloat16>());
  args.ldc = c.stride(0);
  args.status = status_buffer(dev);
  args.q_block = (int)blocksize;
  args.q_type = (int)quant_type;
  args.ag.world = world;
  args.ag.kind = kind;
  for (int q = 0; q < kAgMaxRanks; ++q) {
    const bool in = q < world;
    args.ag.packed[q] = in ? reinterpret_cast<const uint8_t*>(psrc[q]) : nullptr;
    args.ag.absmax[q] = in ? reinterpret_cast<const float*>(asrc[q]) : nullptr;
    args.ag.pstart[q] = in ? pstarts[q] : packed_total;
    args.ag.astart[q] = in ? astarts[q] : absmax_total;
  }
  args.ag.pstart[kAgMaxRanks] = packed_total;
  args.ag.astart[kAgMaxRanks] = absmax_total;
  args.ag_w = reinterpret_cast<__nv_bfloat16*>(wbuf.data_ptr<at::BFloat16>());
  args.ag_cols = kind == kAgF32 ? kAgColsF32 : kAgCols;
  args.ag_kchunks = (int)((K + args.ag_cols - 1) / args.ag_cols);
  {  // start at the N tile holding this rank's first own row
    const int64_t pend = rank + 1 < world ? pstarts[rank + 1] : packed_total;
    const int64_t first_elem = kind == kAgF32 ? pstarts[rank] : 2 * pstarts[rank];
    const int64_t first_row = pend > pstarts[rank] ? std::min<int64_t>(first_elem / K, N - 1) : 0;
    args.ag_rot = (int)std::min<int64_t>(first_row / bn, args.tiles_n - 1);
  }

  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), kBM);
  CUtensorMap tb = make_tmap_bf16(wbuf.data_ptr(), N, K, K, bn / 2);
  CUtensorMap ta2 = ta, tb2 = tb;
  if (a2.has_value() && a2->defined()) {
    TORCH_CHECK(b2.has_value() && b2->defined(), "ag_gemm_nf4: extra slab needs both operands");
    const at::Tensor& x2 = *a2;
    const at::Tensor& y2 = *b2;
    TORCH_CHECK(x2.scalar_type() == at::kBFloat16 && y2.scalar_type() == at::kBFloat16 &&
                    x2.size(0) == M && y2.size(0) == N && x2.size(1) == 64 && y2.size(1) == 64 &&
                    x2.stride(1) == 1 && y2.stride(1) == 1,
                "ag_gemm_nf4: extra slab operands must be bf16 [M,64] and [N,64] row-major");
    ta2 = make_tmap_bf16(x2.data_ptr(), M, 64, x2.stride(0), kBM);
    tb2 = make_tmap_bf16(y2.data_ptr(), N, 64, y2.stride(0), bn / 2);
    args.extra_k16 = 4;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  args.ag_sync = ag_sync_buffer(dev, stream);
  const CUtensorMap tc = make_tmap_store_bf16(c.data_ptr(), M, N, c.stride(0));
  if (swiglu_g != nullptr) {  // c = u, swiglu_out = silu(g)·u
    for (const at::Tensor* x : {swiglu_g, swiglu_out})
      TORCH_CHECK(x->scalar_type() == at::kBFloat16 && x->dim() == 2 && x->size(0) == M &&
                      x->size(1) == N && x->stride(1) == 1 && (x->stride(0) % 8) == 0 &&
                      (reinterpret_cast<uintptr_t>(x->data_ptr()) & 15) == 0,
                  "ag_gemm_nf4: SwiGLU tensors must be bf16 [M, N], 16-byte aligned rows");
    args.epi_src = reinterpret_cast<const __nv_bfloat16*>(swiglu_g->data_ptr<at::BFloat16>());
    args.epi_ld = swiglu_g->stride(0);
    const CUtensorMap tc2 = make_tmap_store_bf16(swiglu_out->data_ptr(), M, N, swiglu_out->stride(0));
    if (bn == 256) launch_gemm_pair<256, 3, 2, false, false, true, kEpiSwigluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
    else launch_gemm_pair<128, 4, 2, false, false, true, kEpiSwigluFwd>(ta, tb, ta2, tb2, tc, args, stream, sms, &tc2);
    return;
  }
  setup_streamk(args, (int)(K / 128), sms, dev, stream);
  if (bn == 256) launch_gemm_pair<256, 3, 2, false, false, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
  else launch_gemm_pair<128, 4, 2, false, false, true>(ta, tb, ta2, tb2, tc, args, stream, sms);
}

void ag_gemm_nf4(at::Tensor a, std::vector<int64_t> psrc, std::vector<int64_t> pstarts,
                 std::vector<int64_t> asrc, std::vector<int64_t> astarts, int64_t packed_total,
                 int64_t absmax_total, int64_t rank, int64_t N, int64_t K, int64_t blocksize,
                 int64_t quant_type, at::Tensor wbuf, at::Tensor c, c10::optional<at::Tensor> a2,
                 c10::optional<at::Tensor> b2, c10::optional<at::Tensor> swiglu_g,
                 c10::optional<at::Tensor> swiglu_out) {
  const bool sw = swiglu_g.has_value() && swiglu_g->defined();
  TORCH_CHECK(!sw || (swiglu_out.has_value() && swiglu_out->defined()),
              "ag_gemm_nf4: the SwiGLU epilogue needs g and an output");
  ag_gemm_impl(kAgNf4, a, psrc, pstarts, asrc, astarts, packed_total, absmax_total, rank, N, K,
               blocksize, quant_type, wbuf, c, a2, b2, sw ? &*swiglu_g : nullptr,
               sw ? &*swiglu_out : nullptr);
}

// The same with W [N, K] held as fp32 pieces (flat elements [starts[q],
// starts[q+1]) at src[q]; total >= N*K, a zero-padded tail allowed): gather,
// cast to bf16 into wbuf and multiply in one kernel.
void ag_gemm_f32(at::Tensor a, std::vector<int64_t> src, std::vector<int64_t> starts, int64_t total,
                 int64_t rank, int64_t N, int64_t K, at::Tensor wbuf, at::Tensor c,
                 c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2) {
  std::vector<int64_t> none(src.size(), 0);
  ag_gemm_impl(kAgF32, a, src, starts, none, none, total, 0, rank, N, K, 64, 0, wbuf, c, a2, b2);
}

// NF4 weight [rows, cols] -> bf16 [rows, cols] (transpose=false) or [cols, rows].
// Non-transposed expansion is a flat map over the row-major order.  A work unit
// is 4 packed bytes (8 codes) -> one 16-byte bf16 store; consecutive lanes take
// consecutive units so every warp load (128 B) and store (512 B) is contiguous.
// Each thread handles kFlatIlp units 256 apart and issues their loads first.
constexpr int kFlatIlp = 4;

__global__ void __launch_bounds__(256) nf4_to_bf16_flat_kernel(
    const uint32_t* __restrict__ packed, const float* __restrict__ absmax, uint4* __restrict__ out,
    int64_t n8, int blocksize, int qtype) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = qtype == 0 ? c_code_nf4[threadIdx.x] : c_code_fp4[threadIdx.x];
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * blockDim.x * kFlatIlp + threadIdx.x;
  uint32_t raw[kFlatIlp];
  float am[kFlatIlp];
#pragma unroll
  for (int j = 0; j < kFlatIlp; ++j) {
    const int64_t i = base + (int64_t)j * blockDim.x;
    if (i < n8) {
      raw[j] = __ldg(packed + i);
      am[j] = __ldg(absmax + (i * 8) / blocksize);
    }
  }
#pragma unroll
  for (int j = 0; j < kFlatIlp; ++j) {
    const int64_t i = base + (int64_t)j * blockDim.x;
    if (i < n8) {
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t byte = (raw[j] >> (8 * q)) & 0xFFu;
        o[q] = pack_bf16x2(lut[byte >> 4] * am[j], lut[byte & 15u] * am[j]);
      }
      out[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Several 4-bit weights decoded into consecutive ranges of one bf16 buffer in one
// launch (the operand of a fused projection, e.g. q/k/v): segment s covers flat
// 8-code units [start[s], start[s+1]) of the output, reading its own packed
// bytes and absmax.  Same per-unit arithmetic as nf4_to_bf16_flat_kernel.
constexpr int kMaxDecodeSegs = 4;
struct DecodeSegs {
  const uint32_t* packed[kMaxDecodeSegs];
  const float* absmax[kMaxDecodeSegs];
  int64_t start[kMaxDecodeSegs + 1];   // in 8-code units
  int nseg;
};

__global__ void __launch_bounds__(256) nf4_to_bf16_segments_kernel(const __grid_constant__ DecodeSegs sg,
                                                                   uint4* __restrict__ out, int blocksize,
                                                                   int qtype) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = qtype == 0 ? c_code_nf4[threadIdx.x] : c_code_fp4[threadIdx.x];
  __syncthreads();
  const int64_t n8 = sg.start[sg.nseg];
  const int64_t base = (int64_t)blockIdx.x * blockDim.x * kFlatIlp + threadIdx.x;
  uint32_t raw[kFlatIlp];
  float am[kFlatIlp];
#pragma unroll
  for (int j = 0; j < kFlatIlp; ++j) {
    const int64_t i = base + (int64_t)j * blockDim.x;
    if (i < n8) {
      int s = 0;
      while (s + 1 < sg.nseg && i >= sg.start[s + 1]) ++s;
      const int64_t li = i - sg.start[s];
      raw[j] = __ldg(sg.packed[s] + li);
      am[j] = __ldg(sg.absmax[s] + (li * 8) / blocksize);
    }
  }
#pragma unroll
  for (int j = 0; j < kFlatIlp; ++j) {
    const int64_t i = base + (int64_t)j * blockDim.x;
    if (i < n8) {
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t byte = (raw[j] >> (8 * q)) & 0xFFu;
        o[q] = pack_bf16x2(lut[byte >> 4] * am[j], lut[byte & 15u] * am[j]);
      }
      out[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// out (bf16, contiguous) = the weights of `packed[s]` / `absmax[s]` (numel[s]
// elements each, row-major) one after the other; every numel a multiple of the
// block size and of 8, at most 4 segments.
void nf4_to_bf16_segments(std::vector<at::Tensor> packed, std::vector<at::Tensor> absmax,
                          std::vector<int64_t> numel, at::Tensor out, int64_t blocksize, int64_t qtype) {
  const int ns = (int)packed.size();
  TORCH_CHECK(ns >= 1 && ns <= kMaxDecodeSegs && (int)absmax.size() == ns && (int)numel.size() == ns,
              "nf4_to_bf16_segments: 1-4 segments with packed, absmax and numel each");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                  (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "nf4_to_bf16_segments: out must be contiguous, 16-byte aligned bf16");
  TORCH_CHECK(blocksize > 0 && blocksize % 8 == 0 && (qtype == 0 || qtype == 1),
              "nf4_to_bf16_segments: block size a multiple of 8, qtype 0 or 1");
  DecodeSegs sg{};
  sg.nseg = ns;
  int64_t total = 0;
  for (int s = 0; s < ns; ++s) {
    TORCH_CHECK(numel[s] % 8 == 0 && numel[s] % blocksize == 0, "nf4_to_bf16_segments: numel % 8 and % blocksize");
    TORCH_CHECK(packed[s].is_cuda() && packed[s].scalar_type() == at::kByte && packed[s].numel() * 2 >= numel[s] &&
                    (reinterpret_cast<uintptr_t>(packed[s].data_ptr()) & 3) == 0,
                "nf4_to_bf16_segments: packed must be 4-byte aligned uint8 covering numel");
    TORCH_CHECK(absmax[s].scalar_type() == at::kFloat && absmax[s].numel() * blocksize >= numel[s],
                "nf4_to_bf16_segments: absmax must be fp32 covering numel");
    sg.packed[s] = reinterpret_cast<const uint32_t*>(packed[s].data_ptr<uint8_t>());
    sg.absmax[s] = absmax[s].data_ptr<float>();
    sg.start[s] = total / 8;
    total += numel[s];
  }
  sg.start[ns] = total / 8;
  TORCH_CHECK(out.numel() >= total, "nf4_to_bf16_segments: out too small");
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t n8 = total / 8;
  const int64_t blocks = (n8 + 256 * kFlatIlp - 1) / (256 * kFlatIlp);
  if (blocks == 0) return;
  nf4_to_bf16_segments_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      sg, reinterpret_cast<uint4*>(out.data_ptr<at::BFloat16>()), (int)blocksize, (int)qtype);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void nf4_to_bf16(at::Tensor packed, at::Tensor absmax, at::Tensor out, int64_t rows, int64_t cols,
                 int64_t blocksize, int64_t qtype, bool transpose) {
  TORCH_CHECK(packed.is_cuda() && packed.scalar_type() == at::kByte, "nf4_to_bf16: uint8 packed");
  TORCH_CHECK(absmax.scalar_type() == at::kFloat, "nf4_to_bf16: fp32 absmax");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == rows * cols,
              "nf4_to_bf16: out bf16 [rows*cols]");
  TORCH_CHECK(cols % 16 == 0 && (!transpose || rows % 16 == 0), "nf4_to_bf16: 16-aligned dims");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(packed.data_ptr()) & 7) == 0, "nf4_to_bf16: packed 8-byte aligned");
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t total = rows * cols;
  if (!transpose && total % 8 == 0 && blocksize % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(packed.data_ptr()) & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0) {
    const int64_t n8 = total / 8;
    const int64_t blocks = (n8 + 256 * kFlatIlp - 1) / (256 * kFlatIlp);
    if (blocks == 0) return;
    nf4_to_bf16_flat_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const uint32_t*>(packed.data_ptr<uint8_t>()), absmax.data_ptr<float>(),
        reinterpret_cast<uint4*>(out.data_ptr<at::BFloat16>()), n8, (int)blocksize, (int)qtype);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  nf4_to_bf16_tile_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      packed.data_ptr<uint8_t>(), absmax.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), (int)rows, (int)cols,
      (int)blocksize, (int)qtype, transpose ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

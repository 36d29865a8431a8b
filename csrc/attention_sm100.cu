// Flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// q, k, v, o: [B, S, H, D] bf16 (projection layout, no transposes), D = 128,
// S % 128 == 0, GQA (Hq a multiple of Hk); lse [B, Hq, S] fp32, natural log of
// the softmax denominator of the scaled scores (what the backward expects).
//
// One CTA per (128-query tile, head, batch); 352 threads:
//   warps 0-7  softmax + epilogue: warps w and w+4 share TMEM lane quadrant w
//              (query rows 32w..32w+31); warp w handles key columns 0-63 of
//              S (and O columns 0-63), warp w+4 columns 64-127.  The two halves
//              of a row exchange their partial row maxima (and, at the end,
//              row sums) through shared memory under a 64-thread named barrier.
//   warp 8     MMA issuer (one thread) and TMEM owner (512 columns:
//              S double buffer at columns 0 / 128, O at 256, Q at 384).
//   warps 9-10 TMA loaders (one thread each, in different warps so neither
//              waits behind the other's spin): warp 9 loads Q once and K tiles
//              of 128 keys into a three-stage ring, warp 10 V tiles into a
//              two-stage ring (4-D tensor maps over [B, S, H, D], 128-byte
//              swizzle).  A K stage is released when S_j has consumed it, a V
//              stage when PV_j has, so the next K tiles are in flight while
//              softmax and PV of the current one run.
// Q is copied once from shared into tensor memory (bf16 pairs, one row per
// lane) by the softmax threads, so both MMAs read their A operand from tensor
// memory and only K and V stream through shared memory: an M=N=128 MMA with
// both operands in shared memory would need the whole shared-memory bandwidth.
// Per key tile j:
//   S_j = Q K_jᵀ            tcgen05.mma, A = Q (tensor memory), B = K_j (smem, K-major)
//   softmax_j (registers)   row max; P_j = exp2(S_j·scale·log2e - m) as bf16, written
//                           back over S_j's own tensor-memory columns (tcgen05.st);
//                           row sums in fp32
//   O += P_j V_j            tcgen05.mma with A = P_j read from tensor memory and
//                           B = V_j (smem) read MN-major
// The MMA thread issues S_{j+1} before PV_j so softmax_{j+1} overlaps PV_j.  The
// running max m only moves when a row's new max exceeds it by more than 8 (log2
// units): exponentials stay <= 2^8 and O (in TMEM) is rescaled only then, which
// after the first tiles is rare.  The final O / l and lse use the same m, so the
// result is exact softmax attention.
//
// Causal: query tile qt visits key tiles 0..qt; only the diagonal tile is masked.
// CTAs are numbered head-major (K/V reuse in L2), longest query tile first.
//
// Every mbarrier wait is bounded (common.cuh); a timeout records an error code
// in the device status word, and each role drains what it issued before the
// CTA frees its TMEM and exits.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "common.cuh"

// defined in gemm_sm100.cu
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn();
zq::DeviceStatus* status_buffer(int device);

namespace zq {

constexpr int kAttRows = 128;      // queries per CTA = TMEM lanes
constexpr int kAttKeys = 128;      // keys per tile
constexpr int kAttD = 128;         // head dim
constexpr int kAttThreads = 352;
constexpr int kSoftmaxWarps = 8;
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kTraceSlots = 32;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum AttErr { kErrAttLoad = 301, kErrAttMma = 302, kErrAttSoftmax = 303 };

struct AttSmem {
  // a 128 x 128 bf16 tile = two 128-byte-swizzled atoms of 128 rows x 64 columns
  static constexpr int kTile = kAttRows * kAttD * 2;   // 32 KB
  static constexpr int kAtom = kTile / 2;              // 16 KB
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;                 // kKStages stages
  static constexpr int kV = kK + kKStages * kTile;      // kVStages stages
  static constexpr int kXMax = kV + kVStages * kTile;   // [2 parity][2 halves][128 rows] fp32
  static constexpr int kXSum = kXMax + 2 * 2 * 128 * 4; // [2 halves][128 rows] fp32
  static constexpr int kBar = kXSum + 2 * 128 * 4;
  static constexpr int kBytes = kBar + 256 + 1024;      // barriers + alignment slack
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kAttThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                   float* __restrict__ lse, int B, int S, int Hq, int Hk, float scale_log2,
                   int causal, DeviceStatus* status, unsigned long long* __restrict__ trace) {
  // trace (optional, [grid][kTraceSlots] ns from %globaltimer): 0 CTA start,
  // 1 first S tile ready; for key tiles j = 1..2, slots 2 + 12(j-1) + i:
  //   softmax warp 0 lane 0: i = 0 S_j ready, 1 row max exchanged,
  //     2 exponentials done, 3 P stored, 4 p_full arrived;
  //   MMA thread: 5 K_{j+1} seen, 6 S_{j+1} issued, 7 p_full(j) seen,
  //     8 V_j seen, 9 PV_j issued;
  //   loaders: 10 K_{j+1} load issued, 11 V_j load issued;
  // kTraceSlots-2 epilogue end, kTraceSlots-1 number of key tiles
  unsigned long long* tr = trace ? trace + (size_t)blockIdx.x * kTraceSlots : nullptr;
  using L = AttSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;     // [kKStages]
  uint64_t* k_empty = bars + 4;    // [kKStages]
  uint64_t* v_full = bars + 7;     // [kVStages]
  uint64_t* v_empty = bars + 9;    // [kVStages]
  uint64_t* s_full = bars + 11;    // [2]
  uint64_t* p_full = bars + 13;    // [2]
  uint64_t* pv_done = bars + 15;   // [2]
  uint64_t* drain = bars + 17;
  uint64_t* q_tmem = bars + 18;    // Q copied into tensor memory (one arrival per softmax warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nqt = S / kAttRows;
  // head-major order: the query tiles of one (batch, head) run side by side and
  // share its K/V tiles in L2; within a head the longest (last) tile starts first
  const int bh = (int)(blockIdx.x / (unsigned)nqt);
  const int qt = nqt - 1 - (int)(blockIdx.x % (unsigned)nqt);
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hk);
  const int n_kv = causal ? qt + 1 : nqt;

  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftmaxWarps);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(q_tmem, kSoftmaxWarps);
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint8_t* sQ = smem + L::kQ;

  if (warp >= 9) {
    // ------------------------------------------------------------ TMA loaders
    if (lane == 0) {
      const bool is_k = warp == 9;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, L::kTile);
        tma_load_4d(sQ, &tmQ, q_full, 0, h, qt * kAttRows, b);
        tma_load_4d(sQ + L::kAtom, &tmQ, q_full, 64, h, qt * kAttRows, b);
      }
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint64_t* full = is_k ? k_full : v_full;
      uint8_t* ring = smem + (is_k ? L::kK : L::kV);
      const int nst = is_k ? kKStages : kVStages;
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % nst;
        if (!mbar_wait(&empty[st], ((j / nst) & 1) ^ 1, status, kErrAttLoad)) { ok = false; break; }
        uint8_t* dst = ring + st * L::kTile;
        if (tr && is_k && j >= 2 && j <= 3) tr[2 + 12 * (j - 2) + 10] = globaltimer();
        if (tr && !is_k && j >= 1 && j <= 2) tr[2 + 12 * (j - 1) + 11] = globaltimer();
        mbar_arrive_expect_tx(&full[st], L::kTile);
        tma_load_4d(dst, map, &full[st], 0, hk, j * kAttKeys, b);
        tma_load_4d(dst + L::kAtom, map, &full[st], 64, hk, j * kAttKeys, b);
        issued = j + 1;
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        if (is_k) mbar_wait(q_full, 0, nullptr, 0);
        for (int j = (issued > nst ? issued - nst : 0); j < issued; ++j)
          mbar_wait(&full[j % nst], (j / nst) & 1, nullptr, 0);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kAttRows, kAttKeys);
      constexpr uint32_t idesc_pv = umma_idesc_bf16_bmn(kAttRows, kAttD);
      bool ok = mbar_wait(q_tmem, 0, status, kErrAttMma);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;                       // S buffer in tensor memory
        const int ks = j % kKStages;                // K stage
        if (!mbar_wait(&k_full[ks], (j / kKStages) & 1, status, kErrAttMma)) return false;
        if (tr && j >= 2 && j <= 3) tr[2 + 12 * (j - 2) + 5] = globaltimer();
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kK + ks * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {
          // Q: 16 head dims = 8 tensor-memory columns; K: +32 B inside a swizzle atom
          const uint32_t off = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          umma_f16_ts(tmem + (uint32_t)(st * kAttKeys), tmem + 384u + (uint32_t)(kk * 8),
                      umma_desc_sw128_kmajor(k_addr + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[ks]);   // K_j consumed
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        unsigned long long* tj = (tr && j >= 1 && j <= 2) ? tr + 2 + 12 * (j - 1) : nullptr;
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        if (tj) tj[6] = globaltimer();
        const int st = j & 1;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1, status, kErrAttMma)) { ok = false; break; }
        if (tj) tj[7] = globaltimer();
        const int vs = j % kVStages;
        if (!mbar_wait(&v_full[vs], (j / kVStages) & 1, status, kErrAttMma)) { ok = false; break; }
        if (tj) tj[8] = globaltimer();
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + L::kV + vs * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttKeys / 16; ++kk) {
          // P_j (bf16) sits in S_j's columns: 16 keys = 8 columns per MMA.
          // V tile: two 64-column (D) atoms of 128 key rows; 16 keys = 2048 B
          umma_f16_ts(tmem + 256u, tmem + (uint32_t)(st * kAttKeys + kk * 8),
                      umma_desc_sw128_mnmajor(v_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[vs]);   // V_j consumed
        umma_commit(&pv_done[st]);
        if (tj) tj[9] = globaltimer();
      }
      // every MMA issued by this thread has completed before TMEM can be freed
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;                      // TMEM lane quadrant
    const int half = warp >> 2;                     // 0: key/O columns 0-63, 1: 64-127
    const int row = quad * 32 + lane;               // query row in the tile = TMEM lane
    const int col0 = half * 64;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float* xmax = reinterpret_cast<float*>(smem + L::kXMax);
    float* xsum = reinterpret_cast<float*>(smem + L::kXSum);
    const int pair_bar = 1 + quad;                  // warps quad and quad+4
    float m_used = -INFINITY;
    float l = 0.0f;                                 // this half's share of the row sum
    bool ok = true;
    {
      // Q row `row`, head dims [64*half, 64*half + 64): one swizzle atom row of
      // 128 B in shared memory -> 32 tensor-memory columns at 384 + 32*half
      const bool qin = mbar_wait(q_full, 0, status, kErrAttSoftmax);
      ok = named_barrier_and(pair_bar, 64, qin);
      if (ok) {
        const uint8_t* qrow = sQ + half * L::kAtom + row * 128;
        uint32_t qv[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 u = *reinterpret_cast<const uint4*>(qrow + ((c ^ (row & 7)) << 4));
          qv[4 * c + 0] = u.x;
          qv[4 * c + 1] = u.y;
          qv[4 * c + 2] = u.z;
          qv[4 * c + 3] = u.w;
        }
        tmem_st_32x32b_x32(tmem + lane_base + 384u + (uint32_t)(half * 32), qv);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_tmem);
      }
    }
    // Every exit from this loop is decided by a vote over both warps of the
    // pair, so neither can leave the other waiting at a named barrier.
    for (int j = 0; j < n_kv && ok; ++j) {
      const int st = j & 1;
      const bool got = mbar_wait(&s_full[st], (j >> 1) & 1, status, kErrAttSoftmax);
      if (!named_barrier_and(pair_bar, 64, got)) { ok = false; break; }
      const bool trj = tr && threadIdx.x == 0 && j >= 1 && j <= 2;
      unsigned long long* tj = trj ? tr + 2 + 12 * (j - 1) : nullptr;
      if (tr && j == 0 && threadIdx.x == 0) tr[1] = globaltimer();
      if (trj) tj[0] = globaltimer();
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(st * kAttKeys + col0),
                         *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(st * kAttKeys + col0 + 32),
                         *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      const bool diag = causal && j == qt;
      if (diag) {  // causal mask on the diagonal tile: keys after the query -> -inf
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (col0 + c > row) r[c] = __float_as_uint(-INFINITY);
      }
      // 8 independent partial maxima, then a tree (no 64-long dependency chain)
      float pm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int c = 8; c < 64; c += 8)
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = fmaxf(pm[i], __uint_as_float(r[c + i]));
      float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                       fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      // full-row max from both halves (buffered by tile parity so a fast half
      // cannot overwrite a value its partner has not read yet)
      float* xm = xmax + (st * 2) * 128;
      xm[half * 128 + row] = mx;
      // both halves have read their S columns before either writes P over them
      tc_fence_before();
      named_barrier(pair_bar, 64);
      tc_fence_after();
      mx = fmaxf(xm[row], xm[128 + row]) * scale_log2;
      if (trj) tj[1] = globaltimer();
      const bool need = mx > m_used + kRescaleThreshold;
      // the pair covers the same rows with the same maxima: both take this branch
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_used;
        const float factor = (m_used == -INFINITY) ? 0.0f : fast_exp2(m_used - m_new);
        if (j > 0) {
          // O holds PV_0..PV_{j-1}: wait for PV_{j-1}, then scale this half of the rows
          const bool pv = mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, status, kErrAttSoftmax);
          if (!named_barrier_and(pair_bar, 64, pv)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            const uint32_t addr = tmem + lane_base + 256u + (uint32_t)(col0 + c * 32);
            tmem_ld_32x32b_x32(addr, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st_32x32b_x32(addr, o);
          }
          tmem_st_wait();
        }
        l *= factor;
        m_used = m_new;
      }
      // P_j (bf16 pairs) over S_j's columns: half h owns columns [32h, 32h + 32)
      float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {  // masked keys hold -inf: exp2 gives exactly 0
        const float p0 = fast_exp2(fmaf(__uint_as_float(r[2 * i]), scale_log2, -m_used));
        const float p1 = fast_exp2(fmaf(__uint_as_float(r[2 * i + 1]), scale_log2, -m_used));
        ps[i & 3] += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      if (trj) tj[2] = globaltimer();
      tmem_st_32x32b_x32(tmem + lane_base + (uint32_t)(st * kAttKeys + half * 32), pk);
      tmem_st_wait();
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      if (trj) tj[3] = globaltimer();
      tc_fence_before();          // TMEM loads/stores of this step ordered before the arrive
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
      if (trj) tj[4] = globaltimer();
    }
    if (named_barrier_and(pair_bar, 64, ok)) {
      const int jl = n_kv - 1;
      const bool done = mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, status, kErrAttSoftmax);
      xsum[half * 128 + row] = l;
      if (named_barrier_and(pair_bar, 64, done)) {
        tc_fence_after();
        const float lt = xsum[row] + xsum[128 + row];
        const float inv = 1.0f / lt;
        const int q = qt * kAttRows + row;
        __nv_bfloat16* orow = O + (((int64_t)b * S + q) * Hq + h) * kAttD + col0;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256u + (uint32_t)(col0 + c * 32), o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + i * 8) = v;
          }
        }
        if (half == 0) lse[((int64_t)b * Hq + h) * S + q] = (m_used + __log2f(lt)) * 0.69314718055994531f;
        if (tr && threadIdx.x == 0) {
          tr[kTraceSlots - 2] = globaltimer();
          tr[kTraceSlots - 1] = (unsigned long long)n_kv;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// Forward over two query tiles per CTA (256 queries of one head).
//
// Tensor memory holds S and O of both tiles: S_A 0-127, S_B 128-255, O_A
// 256-383, O_B 384-511; P (bf16 pairs) is written over the first 64 columns of
// its tile's S.  Q_A and Q_B stay in shared memory (the score MMAs read both
// operands there), K and V stream through two-stage TMA rings shared by both
// tiles, so every K/V tile is loaded once for 256 queries.
//
// 320 threads: warps 0-3 are the softmax/epilogue warpgroup of tile A, warps
// 4-7 that of tile B (thread = one query row = one TMEM lane, the whole
// 128-key row in registers), warp 8 issues the MMAs, warp 9 loads.  The MMA
// order per key tile j is
//     PV_A(j), S_A(j+1) | PV_B(j), S_B(j+1) | PV_A(j+1), S_A(j+2) | ...
// so tile A's exponentials of key tile j+1 run while the tensor core does tile
// B's PV and next scores, and the other way round.
//
// Ten warps put three on some SMSP, whose 16K registers then cap a thread at
// 168 registers: the row (128 fp32 scores) fits, with the O rescale moved
// after the P store so the two are never live together.
//
// Softmax arithmetic uses Blackwell's packed fp32 pairs (fma/add .f32x2) and
// 3-input maxima.  Exponentials: 2^x by ex2.approx on the special-function
// unit, and for every POLY_EVERY-th pair of columns by a polynomial on the FMA
// pipes (Cody-Waite range reduction x = j + f, f in [-1/2, 1/2], 2^f by a
// degree-3 polynomial, 2^j added to the exponent field).  The coefficients are
// a relative-error least-squares fit on 4000 Chebyshev nodes of [-1/2, 1/2]
// (max relative error 7.8e-5 in fp32, against 2^-9 for the bf16 P).
//
// Causal: the CTA takes query tiles 2p and 2p+1 (key tiles 0..2p and 0..2p+1);
// CTAs are ordered longest first over all heads.  Other rules (lazy rescale by
// more than 2^8, bounded waits, draining before TMEM is freed) as above.
// ============================================================================
constexpr int kF2Threads = 320;
constexpr int kF2KStages = 2;
constexpr int kF2VStages = 2;

struct Fwd2Smem {
  static constexpr int kTile = AttSmem::kTile, kAtom = AttSmem::kAtom;
  static constexpr int kQ = 0;                               // Q_A, Q_B
  static constexpr int kK = 2 * kTile;                       // kF2KStages stages
  static constexpr int kV = kK + kF2KStages * kTile;         // kF2VStages stages
  static constexpr int kBar = kV + kF2VStages * kTile;
  static constexpr int kBytes = kBar + 256 + 1024;
};

// Packed fp32 pairs (Blackwell f32x2 arithmetic: one instruction for two values).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair, x <= 64, by range reduction and a degree-3 polynomial (see
// above); x below -120 is clamped there (2^-120 ~ 7.5e-37 instead of 0).
__device__ __forceinline__ void exp2_poly3_x2(float a0, float a1, float& p0, float& p1) {
  const uint64_t x = f2_pack(fmaxf(a0, -120.0f), fmaxf(a1, -120.0f));
  const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);   // 1.5 * 2^23
  const uint64_t t = f2_add(x, magic);        // round(x) in the low mantissa bits
  const uint64_t f = f2_sub(x, f2_sub(t, magic));   // [-1/2, 1/2]
  uint64_t p = f2_fma(f2_pack(0.05508868396282196f, 0.05508868396282196f), f,
                      f2_pack(0.24260404706001282f, 0.24260404706001282f));
  p = f2_fma(p, f, f2_pack(0.6932762265205383f, 0.6932762265205383f));
  p = f2_fma(p, f, f2_pack(0.9999289512634277f, 0.9999289512634277f));
  float q0, q1, t0, t1;
  f2_unpack(p, q0, q1);
  f2_unpack(t, t0, t1);
  // the bits of t are (0x4B400000 + round(x)); shifted by 23 only round(x) << 23 remains
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

template <int POLY_EVERY, bool TRACE>
__global__ void __launch_bounds__(kF2Threads, 1)
attn_fwd2_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                    float* __restrict__ lse, int B, int S, int Hq, int Hk, float scale_log2,
                    int causal, DeviceStatus* status, unsigned long long* __restrict__ trace) {
  // trace (TRACE builds only, [grid][kTraceSlots] ns from %globaltimer): 0 CTA
  // start; for tile x (0: A, 1: B) and key tile j = 1, 2, slots
  // 1 + 6 (2x + j - 1) + i from warp 4x lane 0: i = 0 S_j ready, 1 S_j in
  // registers, 2 row max done, 3 exponentials done, 4 P stored, 5 p_full
  // arrived; MMA thread: 25 / 27 p_full A(1) / B(1) seen, 26 / 28 PV A(1) +
  // S A(2) / PV B(1) + S B(2) issued; 29 / 30 tile A / B epilogue end, 31 key
  // tiles of B
  unsigned long long* tr = (TRACE && trace) ? trace + (size_t)blockIdx.x * kTraceSlots : nullptr;
  using L = Fwd2Smem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;     // [kF2KStages]
  uint64_t* k_empty = bars + 3;    // [kF2KStages]
  uint64_t* v_full = bars + 5;     // [kF2VStages]
  uint64_t* v_empty = bars + 7;    // [kF2VStages]
  uint64_t* s_full = bars + 9;     // [tile]
  uint64_t* p_full = bars + 11;    // [tile], one arrival per softmax warp
  uint64_t* pv_done = bars + 13;   // [tile]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nqt = S / kAttRows;
  const int npairs = nqt / 2;
  const int BH = B * Hq;
  // longest pairs first over all heads (causal), then any order
  const int pr = causal ? npairs - 1 - (int)(blockIdx.x / (unsigned)BH) : (int)(blockIdx.x / (unsigned)BH);
  const int bh = (int)(blockIdx.x % (unsigned)BH);
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hk);
  const int qt_a = 2 * pr, qt_b = 2 * pr + 1;
  const int n_a = causal ? qt_a + 1 : nqt;
  const int n_b = causal ? qt_b + 1 : nqt;

  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kF2KStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kF2VStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ TMA loader (one thread)
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * L::kTile);
      for (int x = 0; x < 2; ++x) {
        uint8_t* dst = smem + L::kQ + x * L::kTile;
        const int row0 = (x == 0 ? qt_a : qt_b) * kAttRows;
        tma_load_4d(dst, &tmQ, q_full, 0, h, row0, b);
        tma_load_4d(dst + L::kAtom, &tmQ, q_full, 64, h, row0, b);
      }
      // K_j and V_j in key order: a K stage frees when S_B(j) has read it, a V
      // stage when PV_B(j) has, and S_B(j+1) comes after PV_B(j), so loads are
      // issued in the order their stages free up
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int j = 0; j < n_b && ok; ++j) {
        for (int kv = 0; kv < 2; ++kv) {
          const int nst = kv == 0 ? kF2KStages : kF2VStages;
          const int st = j % nst;
          uint64_t* empty = kv == 0 ? k_empty : v_empty;
          uint64_t* full = kv == 0 ? k_full : v_full;
          if (!mbar_wait(&empty[st], ((j / nst) & 1) ^ 1, status, kErrAttLoad)) { ok = false; break; }
          uint8_t* dst = smem + (kv == 0 ? L::kK : L::kV) + st * L::kTile;
          const CUtensorMap* map = kv == 0 ? &tmK : &tmV;
          mbar_arrive_expect_tx(&full[st], L::kTile);
          tma_load_4d(dst, map, &full[st], 0, hk, j * kAttKeys, b);
          tma_load_4d(dst + L::kAtom, map, &full[st], 64, hk, j * kAttKeys, b);
          if (kv == 0) k_issued = j + 1; else v_issued = j + 1;
        }
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        mbar_wait(q_full, 0, nullptr, 0);
        for (int j = (k_issued > kF2KStages ? k_issued - kF2KStages : 0); j < k_issued; ++j)
          mbar_wait(&k_full[j % kF2KStages], (j / kF2KStages) & 1, nullptr, 0);
        for (int j = (v_issued > kF2VStages ? v_issued - kF2VStages : 0); j < v_issued; ++j)
          mbar_wait(&v_full[j % kF2VStages], (j / kF2VStages) & 1, nullptr, 0);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kAttRows, kAttKeys);
      constexpr uint32_t idesc_pv = umma_idesc_bf16_bmn(kAttRows, kAttD);
      auto wait_k = [&](int j) {
        return mbar_wait(&k_full[j % kF2KStages], (j / kF2KStages) & 1, status, kErrAttMma);
      };
      // S_x = Q_x K_jᵀ: both operands K-major in shared memory
      auto issue_s = [&](int x, int j) {
        const uint32_t k_addr = smem_u32(smem + L::kK + (j % kF2KStages) * L::kTile);
        const uint32_t q_addr = smem_u32(smem + L::kQ + x * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          umma_f16_ss(tmem + (uint32_t)(x * 128), umma_desc_sw128_kmajor(q_addr + off),
                      umma_desc_sw128_kmajor(k_addr + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      // O_x += P_x V_j: P from tensor memory (bf16 pairs over S_x), V read MN-major
      auto issue_pv = [&](int x, int j) {
        const uint32_t v_addr = smem_u32(smem + L::kV + (j % kF2VStages) * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttKeys / 16; ++kk)
          umma_f16_ts(tmem + 256u + (uint32_t)(x * 128), tmem + (uint32_t)(x * 128 + kk * 8),
                      umma_desc_sw128_mnmajor(v_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[x]);
      };
      bool ok = mbar_wait(q_full, 0, status, kErrAttMma) && wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_b && ok; ++j) {
        const bool a_on = j < n_a;
        if (!mbar_wait(&v_full[j % kF2VStages], (j / kF2VStages) & 1, status, kErrAttMma)) { ok = false; break; }
        bool k_next = false;   // K_{j+1} already waited for
        const bool trj = tr && j == 1;
        if (a_on) {
          if (!mbar_wait(&p_full[0], j & 1, status, kErrAttMma)) { ok = false; break; }
          if (trj) tr[25] = globaltimer();
          tc_fence_after();
          issue_pv(0, j);
          if (j + 1 < n_a) {
            if (!wait_k(j + 1)) { ok = false; break; }
            k_next = true;
            tc_fence_after();
            issue_s(0, j + 1);
          }
          if (trj) tr[26] = globaltimer();
        }
        if (!mbar_wait(&p_full[1], j & 1, status, kErrAttMma)) { ok = false; break; }
        if (trj) tr[27] = globaltimer();
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&v_empty[j % kF2VStages]);   // V_j consumed by both tiles
        if (j + 1 < n_b) {
          if (!k_next && !wait_k(j + 1)) { ok = false; break; }
          tc_fence_after();
          issue_s(1, j + 1);
          umma_commit(&k_empty[(j + 1) % kF2KStages]);   // K_{j+1} consumed by both tiles
        }
        if (trj) tr[28] = globaltimer();
      }
      // every MMA issued by this thread has completed before TMEM can be freed
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int x = warp >> 2;                        // 0: tile A, 1: tile B
    const int quad = warp & 3;                      // TMEM lane quadrant
    const int row = quad * 32 + lane;               // query row in the tile = TMEM lane
    const int qt = x == 0 ? qt_a : qt_b;
    const int n_kv = x == 0 ? n_a : n_b;
    const uint32_t t_s = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(x * 128);
    const uint32_t t_o = t_s + 256u;
    float m_used = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // every exit is decided by a warp vote: the TMEM loads/stores are warp-wide
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1, status, kErrAttSoftmax))) { ok = false; break; }
      unsigned long long* tj =
          (tr && quad == 0 && lane == 0 && (j == 1 || j == 2)) ? tr + 1 + 6 * (2 * x + j - 1) : nullptr;
      if (tj) tj[0] = globaltimer();
      tc_fence_after();
      uint32_t r[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld_32x32b_x32(t_s + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
      tmem_ld_wait();
      if (tj) tj[1] = globaltimer();
      if (causal && j == qt) {  // diagonal tile: keys after the query -> -inf
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c > row) r[c] = __float_as_uint(-INFINITY);
      }
      // row max: 8 independent chains of 3-input maxima over columns 8..119, then the rest
      float pm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int c = 8; c < 120; c += 16)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pm[i] = fmax3(pm[i], __uint_as_float(r[c + i]), __uint_as_float(r[c + 8 + i]));
      const float mx = fmax3(fmax3(pm[0], pm[1], __uint_as_float(r[120])),
                             fmax3(pm[2], pm[3], __uint_as_float(r[121])),
                             fmax3(fmax3(pm[4], pm[5], __uint_as_float(r[122])),
                                   fmax3(pm[6], pm[7], __uint_as_float(r[123])),
                                   fmax3(__uint_as_float(r[124]), __uint_as_float(r[125]),
                                         fmaxf(__uint_as_float(r[126]), __uint_as_float(r[127]))))) *
                       scale_log2;
      if (tj) tj[2] = globaltimer();
      const bool need = mx > m_used + kRescaleThreshold;
      const bool rescale = __any_sync(0xffffffffu, need);
      float factor = 1.0f;
      if (rescale) {
        const float m_new = need ? mx : m_used;
        factor = (m_used == -INFINITY) ? 0.0f : fast_exp2(m_used - m_new);
        m_used = m_new;
      }
      // P_j (bf16 pairs) over the first 64 columns of S_j; exponent arguments and
      // row sums in packed pairs
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_used, -m_used);
      uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {  // masked keys hold -inf: ex2 gives exactly 0
        float a0, a1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sc2, nm2), a0, a1);
        float p0 = 0.0f, p1 = 0.0f;
        bool poly = false;
        if constexpr (POLY_EVERY > 0) poly = (i % POLY_EVERY) == POLY_EVERY - 1;
        if (poly) {
          exp2_poly3_x2(a0, a1, p0, p1);
        } else {
          p0 = fast_exp2(a0);
          p1 = fast_exp2(a1);
        }
        ps2[i & 3] = f2_add(ps2[i & 3], f2_pack(p0, p1));
        pk[i] = pack_bf16x2(p0, p1);
      }
      if (tj) tj[3] = globaltimer();
      tmem_st_32x32b_x32(t_s, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
      tmem_st_32x32b_x32(t_s + 32u, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
      float ps[4];
      f2_unpack(f2_add(ps2[0], ps2[1]), ps[0], ps[1]);
      f2_unpack(f2_add(ps2[2], ps2[3]), ps[2], ps[3]);
      l = l * factor + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
      if (rescale && j > 0) {
        // O holds PV_0..PV_{j-1}: wait for PV_{j-1}, then scale this thread's row
        // (before the arrival below lets PV_j add into it)
        if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[x], (j - 1) & 1, status, kErrAttSoftmax))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o + (uint32_t)(c * 32), o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st_32x32b_x32(t_o + (uint32_t)(c * 32), o);
        }
      }
      tmem_st_wait();
      if (tj) tj[4] = globaltimer();
      tc_fence_before();          // TMEM loads/stores of this step ordered before the arrive
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
      if (tj) tj[5] = globaltimer();
    }
    if (ok) {
      const int jl = n_kv - 1;
      if (__all_sync(0xffffffffu, mbar_wait(&pv_done[x], jl & 1, status, kErrAttSoftmax))) {
        tc_fence_after();
        const float inv = 1.0f / l;
        const int q = qt * kAttRows + row;
        __nv_bfloat16* orow = O + (((int64_t)b * S + q) * Hq + h) * kAttD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_o + (uint32_t)(c * 32), o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + i * 8) = v;
          }
        }
        lse[((int64_t)b * Hq + h) * S + q] = (m_used + __log2f(l)) * 0.69314718055994531f;
        if (tr && quad == 0 && lane == 0) {
          tr[29 + x] = globaltimer();
          if (x == 1) tr[31] = (unsigned long long)n_b;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// Backward: dQ kernel (per query tile, also producing delta and lse2) and dK/dV
// kernel (per key tile), both on the 5th-generation tensor cores.
//
//   P  = exp(scale·Q Kᵀ - lse)            (recomputed from the saved lse)
//   dP = dO Vᵀ,   dS = P ∘ (dP - delta),   delta = rowsum(dO ∘ O)
//   dQ = scale · dS K,   dK = scale · dSᵀ Q,   dV = Pᵀ dO
//
// dQ kernel: one CTA per (128-query tile, head, batch).  Q and dO are copied
// into tensor memory once; K and V tiles stream through TMA rings.  Per key
// tile the MMA thread issues S = Q Kᵀ and dP = dO Vᵀ interleaved (two
// independent accumulation chains), eight compute warps turn them into dS
// (bf16, written over S's own columns) and the MMA thread adds dS·K into the
// dQ accumulator (K read MN-major).  dQ is written once, in bf16: no atomics.
// Before the loop the compute warps form delta = rowsum(dO ∘ O) of their rows
// (dO from the staged tile, O from global) and store delta and lse·log2(e) for
// the dK/dV kernel, which runs after this one on the same stream.
// Tensor memory: S 0-127, dP 128-255, dQ 256-383, Q 384-447, dO 448-511.
//
// dK/dV kernel: one CTA per (128-key tile, kv head, batch), looping over the
// query heads that share the kv head and over the query tiles that see the
// key tile.  Sᵀ = K Qᵀ and dPᵀ = V dOᵀ (rows = keys) are issued interleaved;
// the compute warps write Pᵀ and dSᵀ (bf16) over them, and dV += Pᵀ dO and
// dK += dSᵀ Q read them from tensor memory (dO and Q read MN-major).
// Tensor memory: dV 0-127, dK 128-255, Sᵀ 256-383, dPᵀ 384-511.
//
// In both kernels warps w and w+4 share TMEM lane quadrant w and split the 128
// columns of a row; every exit from a compute loop is decided by a vote over
// the pair, and every wait is bounded.
// ============================================================================
constexpr int kBwdThreads = 352;   // 8 compute warps, MMA warp, two loader warps
constexpr int kBwdKStages = 3;     // dQ kernel K ring
constexpr int kBwdVStages = 2;     // dQ kernel V ring
constexpr int kBwdQStages = 2;     // dK/dV kernel Q and dO rings
enum AttBwdErr { kErrBwdLoad = 311, kErrBwdMma = 312, kErrBwdCompute = 313 };

// 64 consecutive columns of one TMEM row (this thread's lane) -> registers
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
  tmem_ld_32x32b_x32(taddr + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
}

// one 128-byte row of a 128-byte-swizzled smem atom (64 bf16) -> 32 TMEM columns
__device__ __forceinline__ void copy_row_to_tmem(const uint8_t* atom_row, int row, uint32_t taddr) {
  uint32_t v[32];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(atom_row + ((c ^ (row & 7)) << 4));
    v[4 * c + 0] = u.x;
    v[4 * c + 1] = u.y;
    v[4 * c + 2] = u.z;
    v[4 * c + 3] = u.w;
  }
  tmem_st_32x32b_x32(taddr, v);
}

struct BwdDqSmem {
  static constexpr int kTile = AttSmem::kTile, kAtom = AttSmem::kAtom;
  static constexpr int kQ = 0, kDO = kTile;
  static constexpr int kK = 2 * kTile;                        // kBwdKStages stages
  static constexpr int kV = kK + kBwdKStages * kTile;         // kBwdVStages stages
  static constexpr int kX = kV + kBwdVStages * kTile;         // [2 halves][128 rows] fp32
  static constexpr int kBar = kX + 2 * 128 * 4;
  static constexpr int kBytes = kBar + 256 + 1024;
};

// One thread's half row (columns col0 .. col0 + 63 of a 128-wide head) of an fp32
// accumulator block in TMEM (tblk: this lane's column 0 of the block), times f,
// rounded to bf16 and stored.  With cs (the row position's (cos, sin) of the 64
// rotary pairs) the gradient is rotated back by the inverse RoPE first - the
// pair partners (i, i + 64) sit in the two halves, so both are read; the result
// equals the standalone RoPE kernel with sign -1 applied to the bf16 gradient.
__device__ __forceinline__ void bwd_store_half_row(uint32_t tblk, int col0, float f, const float2* cs,
                                                   __nv_bfloat16* out) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t o[32];
    tmem_ld_32x32b_x32(tblk + (uint32_t)(col0 + c * 32), o);
    if (cs == nullptr) {
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(o[8 * i + 0]) * f, __uint_as_float(o[8 * i + 1]) * f);
        v.y = pack_bf16x2(__uint_as_float(o[8 * i + 2]) * f, __uint_as_float(o[8 * i + 3]) * f);
        v.z = pack_bf16x2(__uint_as_float(o[8 * i + 4]) * f, __uint_as_float(o[8 * i + 5]) * f);
        v.w = pack_bf16x2(__uint_as_float(o[8 * i + 6]) * f, __uint_as_float(o[8 * i + 7]) * f);
        *reinterpret_cast<uint4*>(out + c * 32 + i * 8) = v;
      }
      continue;
    }
    uint32_t p[32];
    tmem_ld_32x32b_x32(tblk + (uint32_t)(64 - col0 + c * 32), p);
    const float4* cs4 = reinterpret_cast<const float4*>(cs + c * 32);
    tmem_ld_wait();
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      // bf16-rounded gradient of columns 2i, 2i + 1 in this half (m) and the partner's (q)
      const float2 m = bf16x2_to_f2(pack_bf16x2(__uint_as_float(o[2 * i]) * f, __uint_as_float(o[2 * i + 1]) * f));
      const float2 q = bf16x2_to_f2(pack_bf16x2(__uint_as_float(p[2 * i]) * f, __uint_as_float(p[2 * i + 1]) * f));
      const float4 t = __ldg(cs4 + i);   // (cos, sin) of pairs 2i and 2i + 1 of this chunk
      const float c0 = t.x, s0 = t.y * -1.0f, c1 = t.z, s1 = t.w * -1.0f;
      float r0, r1;
      if (col0 == 0) {   // this half holds x1, the partner x2
        r0 = rope_lo(m.x, q.x, c0, s0);
        r1 = rope_lo(m.y, q.y, c1, s1);
      } else {           // this half holds x2, the partner x1
        r0 = rope_hi(q.x, m.x, c0, s0);
        r1 = rope_hi(q.y, m.y, c1, s1);
      }
      w[i] = pack_bf16x2(r0, r1);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(out + c * 32 + i * 8) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

__global__ void __launch_bounds__(kBwdThreads, 1)
attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                      const float* __restrict__ lse, const __nv_bfloat16* __restrict__ o,
                      float* __restrict__ delta, float* __restrict__ lse2,
                      __nv_bfloat16* __restrict__ dq, int B, int S, int Hq, int Hk, float scale_log2,
                      float scale, int causal, const float2* __restrict__ rope_cs, DeviceStatus* status,
                      unsigned long long* __restrict__ trace) {
  // trace (optional, [grid][32] ns): 0 start; key tiles j = 1, 2 at 1 + 8(j-1) + i:
  //   compute: i = 0 S/dP seen, 1 loaded, 2 dS computed, 3 arrived;
  //   MMA: 4 K/V seen, 5 S/dP issued, 6 dS seen, 7 dQ issued;  30 end
  unsigned long long* tr = trace ? trace + (size_t)blockIdx.x * 32 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  using L = BwdDqSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;                 // Q and dO landed
  uint64_t* k_full = bars + 1;             // [kBwdKStages]
  uint64_t* k_empty = bars + 4;            // [kBwdKStages]
  uint64_t* v_full = bars + 7;             // [kBwdVStages]
  uint64_t* v_empty = bars + 9;            // [kBwdVStages]
  uint64_t* s_full = bars + 11;            // S and dP of the current key tile
  uint64_t* ds_full = bars + 12;           // dS written (one arrival per compute warp)
  uint64_t* dq_done = bars + 13;
  uint64_t* in_tmem = bars + 14;           // Q, dO copied into TMEM
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = S / kAttRows;
  const int bh = (int)(blockIdx.x / (unsigned)nqt);
  const int qt = nqt - 1 - (int)(blockIdx.x % (unsigned)nqt);
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hk);
  const int n_kv = causal ? qt + 1 : nqt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kBwdKStages; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
    for (int i = 0; i < kBwdVStages; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
    mbar_init(s_full, 1);
    mbar_init(ds_full, kSoftmaxWarps);
    mbar_init(dq_done, 1);
    mbar_init(in_tmem, kSoftmaxWarps);
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmQ); prefetch_tmap(&tmK); prefetch_tmap(&tmV); prefetch_tmap(&tmDO);
  }
  if (warp == 8) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 9) {
    // ------------------------------------------------------------ TMA loaders
    if (lane == 0) {
      const bool is_k = warp == 9;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, 2 * L::kTile);
        tma_load_4d(smem + L::kQ, &tmQ, q_full, 0, h, qt * kAttRows, b);
        tma_load_4d(smem + L::kQ + L::kAtom, &tmQ, q_full, 64, h, qt * kAttRows, b);
        tma_load_4d(smem + L::kDO, &tmDO, q_full, 0, h, qt * kAttRows, b);
        tma_load_4d(smem + L::kDO + L::kAtom, &tmDO, q_full, 64, h, qt * kAttRows, b);
      }
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint64_t* full = is_k ? k_full : v_full;
      uint8_t* ring = smem + (is_k ? L::kK : L::kV);
      const int nst = is_k ? kBwdKStages : kBwdVStages;
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % nst;
        if (!mbar_wait(&empty[st], ((j / nst) & 1) ^ 1, status, kErrBwdLoad)) { ok = false; break; }
        uint8_t* dst = ring + st * L::kTile;
        mbar_arrive_expect_tx(&full[st], L::kTile);
        tma_load_4d(dst, map, &full[st], 0, hk, j * kAttKeys, b);
        tma_load_4d(dst + L::kAtom, map, &full[st], 64, hk, j * kAttKeys, b);
        issued = j + 1;
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        if (is_k) mbar_wait(q_full, 0, nullptr, 0);
        for (int j = (issued > nst ? issued - nst : 0); j < issued; ++j)
          mbar_wait(&full[j % nst], (j / nst) & 1, nullptr, 0);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_k = umma_idesc_bf16(kAttRows, kAttKeys);   // S, dP (B K-major)
      constexpr uint32_t idesc_mn = umma_idesc_bf16_bmn(kAttRows, kAttD); // dQ (K read MN-major)
      bool ok = mbar_wait(in_tmem, 0, status, kErrBwdMma);
      for (int j = 0; j < n_kv && ok; ++j) {
        unsigned long long* tj = (tr && (j == 1 || j == 2)) ? tr + 1 + 8 * (j - 1) : nullptr;
        const int ks = j % kBwdKStages, vs = j % kBwdVStages;
        if (!mbar_wait(&k_full[ks], (j / kBwdKStages) & 1, status, kErrBwdMma)) { ok = false; break; }
        if (!mbar_wait(&v_full[vs], (j / kBwdVStages) & 1, status, kErrBwdMma)) { ok = false; break; }
        if (tj) tj[4] = globaltimer();
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kK + ks * L::kTile);
        const uint32_t v_addr = smem_u32(smem + L::kV + vs * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {   // S = Q Kᵀ and dP = dO Vᵀ, interleaved
          const uint32_t off = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          umma_f16_ts(tmem, tmem + 384u + (uint32_t)(kk * 8), umma_desc_sw128_kmajor(k_addr + off),
                      idesc_k, kk > 0 ? 1u : 0u);
          umma_f16_ts(tmem + 128u, tmem + 448u + (uint32_t)(kk * 8),
                      umma_desc_sw128_kmajor(v_addr + off), idesc_k, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(&v_empty[vs]);   // V_j consumed
        if (tj) tj[5] = globaltimer();
        if (!mbar_wait(ds_full, j & 1, status, kErrBwdMma)) { ok = false; break; }
        if (tj) tj[6] = globaltimer();
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAttKeys / 16; ++kk)   // dQ += dS K: dS in S's columns, K MN-major
          umma_f16_ts(tmem + 256u, tmem + (uint32_t)(kk * 8),
                      umma_desc_sw128_mnmajor(k_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_mn, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&k_empty[ks]);   // K_j consumed
        if (tj) tj[7] = globaltimer();
      }
      umma_commit(dq_done);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ dS + epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;                     // query row = TMEM lane
    const int col0 = half * 64;                           // this half's key (and D) columns
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int pair_bar = 1 + quad;
    const int q = qt * kAttRows + row;
    const int64_t lrow = ((int64_t)b * Hq + h) * S + q;
    const float l2 = lse[lrow] * 1.4426950408889634f;      // lse in log2 units
    // delta = rowsum(dO ∘ O) of this query row, computed here (and written for
    // the dK/dV kernel with lse2): this half's 64 columns of O from global
    // (loads issued before the tile wait), of dO from the tile in shared memory
    uint4 ov[8];
    {
      const uint4* orow = reinterpret_cast<const uint4*>(o + (((int64_t)b * S + q) * Hq + h) * kAttD + col0);
#pragma unroll
      for (int c = 0; c < 8; ++c) ov[c] = orow[c];
    }
    float dl = 0.0f;
    bool ok = named_barrier_and(pair_bar, 64, mbar_wait(q_full, 0, status, kErrBwdCompute));
    if (ok) {
      const uint8_t* drow = smem + L::kDO + half * L::kAtom + row * 128;
      float acc = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {   // dO chunk c (8 columns) sits at swizzled slot c ^ (row & 7)
        const uint4 du = *reinterpret_cast<const uint4*>(drow + ((c ^ (row & 7)) << 4));
        const uint32_t dw[4] = {du.x, du.y, du.z, du.w}, ow[4] = {ov[c].x, ov[c].y, ov[c].z, ov[c].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = bf16x2_to_f2(dw[j]), y = bf16x2_to_f2(ow[j]);
          acc = fmaf(x.x, y.x, acc);
          acc = fmaf(x.y, y.y, acc);
        }
      }
      float* xs = reinterpret_cast<float*>(smem + L::kX);
      xs[half * 128 + row] = acc;
      named_barrier(pair_bar, 64);
      dl = xs[row] + xs[128 + row];
      if (half == 0) {
        delta[lrow] = dl;
        lse2[lrow] = l2;
      }
    }
    if (ok) {  // Q and dO rows into tensor memory (A operands of S and dP)
      copy_row_to_tmem(smem + L::kQ + half * L::kAtom + row * 128, row,
                       tmem + lane_base + 384u + (uint32_t)(half * 32));
      copy_row_to_tmem(smem + L::kDO + half * L::kAtom + row * 128, row,
                       tmem + lane_base + 448u + (uint32_t)(half * 32));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(in_tmem);
    }
    for (int j = 0; j < n_kv && ok; ++j) {
      unsigned long long* tj = (tr && threadIdx.x == 0 && (j == 1 || j == 2)) ? tr + 1 + 8 * (j - 1) : nullptr;
      const bool got = mbar_wait(s_full, j & 1, status, kErrBwdCompute);
      if (!named_barrier_and(pair_bar, 64, got)) { ok = false; break; }
      if (tj) tj[0] = globaltimer();
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_ld64(tmem + lane_base + (uint32_t)col0, s);
      tmem_ld64(tmem + lane_base + 128u + (uint32_t)col0, dp);
      tmem_ld_wait();
      if (tj) tj[1] = globaltimer();
      // both halves hold their S columns before either writes dS over them
      tc_fence_before();
      named_barrier(pair_bar, 64);
      tc_fence_after();
      const bool diag = causal && j == qt;
      // dS = P (dP - delta) with P = 2^(S scale - lse): exponent arguments,
      // differences and products in packed fp32 pairs
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2), nl2 = f2_pack(-l2, -l2), dl2 = f2_pack(dl, dl);
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int c = 2 * i;
        float a0, a1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sc2, nl2), a0, a1);
        float p0 = fast_exp2(a0);
        float p1 = fast_exp2(a1);
        if (diag && col0 + c > row) p0 = 0.0f;
        if (diag && col0 + c + 1 > row) p1 = 0.0f;
        float g0, g1;
        f2_unpack(f2_mul(f2_pack(p0, p1),
                         f2_sub(f2_pack(__uint_as_float(dp[c]), __uint_as_float(dp[c + 1])), dl2)), g0, g1);
        pk[i] = pack_bf16x2(g0, g1);
      }
      if (tj) tj[2] = globaltimer();
      tmem_st_32x32b_x32(tmem + lane_base + (uint32_t)(half * 32), pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
      if (tj) tj[3] = globaltimer();
    }
    if (named_barrier_and(pair_bar, 64, ok)) {
      const bool done = mbar_wait(dq_done, 0, status, kErrBwdCompute);
      if (named_barrier_and(pair_bar, 64, done)) {
        tc_fence_after();
        __nv_bfloat16* orow = dq + (((int64_t)b * S + q) * Hq + h) * kAttD + col0;
        bwd_store_half_row(tmem + lane_base + 256u, col0, scale,
                           rope_cs != nullptr ? rope_cs + (int64_t)q * 64 : nullptr, orow);
        if (tr && threadIdx.x == 0) tr[30] = globaltimer();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

struct BwdDkvSmem {
  static constexpr int kTile = AttSmem::kTile, kAtom = AttSmem::kAtom;
  static constexpr int kK = 0, kV = kTile;
  static constexpr int kQ = 2 * kTile;                        // kBwdQStages stages
  static constexpr int kDO = kQ + kBwdQStages * kTile;        // kBwdQStages stages
  static constexpr int kLD = kDO + kBwdQStages * kTile;        // per stage: lse2[128], delta[128]
  static constexpr int kBar = kLD + kBwdQStages * 1024;
  static constexpr int kBytes = kBar + 256 + 1024;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
attn_bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const float* __restrict__ lse2, const float* __restrict__ delta,
                       __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int B, int S,
                       int Hq, int Hk, float scale_log2, float scale, int causal,
                       const float2* __restrict__ rope_cs, DeviceStatus* status,
                       unsigned long long* __restrict__ trace, int64_t ld_dk, int64_t ld_dv) {
  // ld_dk / ld_dv: elements between consecutive tokens of dK / dV (Hk * 128 when
  // contiguous; wider when the output is a column slice of a fused gradient)
  // trace (optional, [grid][32] ns): 0 start; iterations t = 1, 2 at 1 + 8(t-1) + i:
  //   compute: i = 0 Sᵀ/dPᵀ seen, 1 loaded, 2 Pᵀ/dSᵀ computed, 3 arrived;
  //   MMA: 4 Q/dO seen, 5 Sᵀ/dPᵀ issued, 6 Pᵀ/dSᵀ seen, 7 dV/dK issued;  30 end
  unsigned long long* tr = trace ? trace + (size_t)blockIdx.x * 32 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  using L = BwdDkvSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bars;                // K_j and V_j landed
  uint64_t* q_full = bars + 1;             // [kBwdQStages]
  uint64_t* q_empty = bars + 3;            // [kBwdQStages]
  uint64_t* o_full = bars + 5;             // [kBwdQStages] dO
  uint64_t* o_empty = bars + 7;            // [kBwdQStages]
  uint64_t* s_full = bars + 9;             // Sᵀ and dPᵀ of the current query tile
  uint64_t* p_full = bars + 10;            // Pᵀ, dSᵀ written (one arrival per compute warp)
  uint64_t* acc_done = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = S / kAttKeys, nqt = S / kAttRows;
  const int bhk = (int)(blockIdx.x / (unsigned)nkt);
  const int kt = (int)(blockIdx.x % (unsigned)nkt);        // key tile 0 (most work) first
  const int b = bhk / Hk, hk = bhk % Hk;
  const int group = Hq / Hk;
  const int i0 = causal ? kt : 0;                           // first query tile that sees this key tile
  const int per_head = nqt - i0;
  const int n_it = group * per_head;                        // (query head, query tile) iterations

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kBwdQStages; ++i) {
      mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1);
      mbar_init(&o_full[i], 1); mbar_init(&o_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmQ); prefetch_tmap(&tmK); prefetch_tmap(&tmV); prefetch_tmap(&tmDO);
  }
  if (warp == 8) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 9) {
    // ------------------------------------------------------------ TMA loaders
    if (lane == 0) {
      const bool is_q = warp == 9;
      if (is_q) {
        mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
        tma_load_4d(smem + L::kK, &tmK, kv_full, 0, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kK + L::kAtom, &tmK, kv_full, 64, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kV, &tmV, kv_full, 0, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kV + L::kAtom, &tmV, kv_full, 64, hk, kt * kAttKeys, b);
      }
      const CUtensorMap* map = is_q ? &tmQ : &tmDO;
      uint64_t* empty = is_q ? q_empty : o_empty;
      uint64_t* full = is_q ? q_full : o_full;
      uint8_t* ring = smem + (is_q ? L::kQ : L::kDO);
      int issued = 0;
      bool ok = true;
      for (int t = 0; t < n_it; ++t) {
        const int st = t % kBwdQStages;
        const int h = hk * group + t / per_head, it = i0 + t % per_head;
        if (!mbar_wait(&empty[st], ((t / kBwdQStages) & 1) ^ 1, status, kErrBwdLoad)) { ok = false; break; }
        uint8_t* dst = ring + st * L::kTile;
        mbar_arrive_expect_tx(&full[st], L::kTile + (is_q ? 0 : 1024));
        tma_load_4d(dst, map, &full[st], 0, h, it * kAttRows, b);
        tma_load_4d(dst + L::kAtom, map, &full[st], 64, h, it * kAttRows, b);
        if (!is_q) {  // this query tile's lse2 and delta rows (512 B each)
          const int64_t li = ((int64_t)b * Hq + h) * S + it * kAttRows;
          bulk_load(smem + L::kLD + st * 1024, lse2 + li, 512, &full[st]);
          bulk_load(smem + L::kLD + st * 1024 + 512, delta + li, 512, &full[st]);
        }
        issued = t + 1;
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        if (is_q) mbar_wait(kv_full, 0, nullptr, 0);
        for (int t = (issued > kBwdQStages ? issued - kBwdQStages : 0); t < issued; ++t)
          mbar_wait(&full[t % kBwdQStages], (t / kBwdQStages) & 1, nullptr, 0);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_k = umma_idesc_bf16(kAttKeys, kAttRows);   // Sᵀ, dPᵀ
      constexpr uint32_t idesc_mn = umma_idesc_bf16_bmn(kAttKeys, kAttD); // dV, dK
      bool ok = mbar_wait(kv_full, 0, status, kErrBwdMma);
      const uint32_t k_addr = smem_u32(smem + L::kK), v_addr = smem_u32(smem + L::kV);
      for (int t = 0; t < n_it && ok; ++t) {
        unsigned long long* tj = (tr && (t == 1 || t == 2)) ? tr + 1 + 8 * (t - 1) : nullptr;
        const int st = t % kBwdQStages;
        const uint32_t ph = (t / kBwdQStages) & 1;
        if (!mbar_wait(&q_full[st], ph, status, kErrBwdMma)) { ok = false; break; }
        if (!mbar_wait(&o_full[st], ph, status, kErrBwdMma)) { ok = false; break; }
        if (tj) tj[4] = globaltimer();
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + L::kQ + st * L::kTile);
        const uint32_t o_addr = smem_u32(smem + L::kDO + st * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {   // Sᵀ = K Qᵀ and dPᵀ = V dOᵀ, interleaved
          const uint32_t off = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          umma_f16_ss(tmem + 256u, umma_desc_sw128_kmajor(k_addr + off),
                      umma_desc_sw128_kmajor(q_addr + off), idesc_k, kk > 0 ? 1u : 0u);
          umma_f16_ss(tmem + 384u, umma_desc_sw128_kmajor(v_addr + off),
                      umma_desc_sw128_kmajor(o_addr + off), idesc_k, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (tj) tj[5] = globaltimer();
        if (!mbar_wait(p_full, t & 1, status, kErrBwdMma)) { ok = false; break; }
        if (tj) tj[6] = globaltimer();
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAttRows / 16; ++kk) {   // dV += Pᵀ dO and dK += dSᵀ Q, interleaved
          umma_f16_ts(tmem, tmem + 256u + (uint32_t)(kk * 8),
                      umma_desc_sw128_mnmajor(o_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_mn, (t > 0 || kk > 0) ? 1u : 0u);
          umma_f16_ts(tmem + 128u, tmem + 384u + (uint32_t)(kk * 8),
                      umma_desc_sw128_mnmajor(q_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_mn, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&q_empty[st]);
        umma_commit(&o_empty[st]);
        if (tj) tj[7] = globaltimer();
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ Pᵀ, dSᵀ + epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;                     // key row = TMEM lane
    const int col0 = half * 64;                           // this half's query (and D) columns
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int pair_bar = 1 + quad;
    const int key = kt * kAttKeys + row;
    bool ok = true;
    for (int t = 0; t < n_it && ok; ++t) {
      const int h = hk * group + t / per_head, it = i0 + t % per_head;
      // lse2 / delta of this query tile, staged with dO (s_full implies they landed)
      const float* sl = reinterpret_cast<const float*>(smem + L::kLD + (t % kBwdQStages) * 1024) + col0;
      unsigned long long* tj = (tr && threadIdx.x == 0 && (t == 1 || t == 2)) ? tr + 1 + 8 * (t - 1) : nullptr;
      // the staged lse2/delta completed o_full; wait on it too so the bulk copy's
      // data is visible to these threads (it has completed by now)
      const bool got = mbar_wait(s_full, t & 1, status, kErrBwdCompute) &&
                       mbar_wait(&o_full[t % kBwdQStages], (t / kBwdQStages) & 1, status, kErrBwdCompute);
      if (!named_barrier_and(pair_bar, 64, got)) { ok = false; break; }
      if (tj) tj[0] = globaltimer();
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_ld64(tmem + lane_base + 256u + (uint32_t)col0, s);
      tmem_ld64(tmem + lane_base + 384u + (uint32_t)col0, dp);
      tmem_ld_wait();
      if (tj) tj[1] = globaltimer();
      tc_fence_before();
      named_barrier(pair_bar, 64);   // both halves hold their columns before either overwrites
      tc_fence_after();
      const bool diag = causal && it == kt;
      uint32_t pp[32], dsp[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {   // 4 queries per step: shared-memory broadcasts
        const float4 l4 = reinterpret_cast<const float4*>(sl)[i];
        const float4 d4 = reinterpret_cast<const float4*>(sl + 128)[i];
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
        float p[4], ds[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = 4 * i + u;
          p[u] = fast_exp2(fmaf(__uint_as_float(s[c]), scale_log2, -lv[u]));
          if (diag && key > it * kAttRows + col0 + c) p[u] = 0.0f;
          ds[u] = p[u] * (__uint_as_float(dp[c]) - dv4[u]);
        }
        pp[2 * i] = pack_bf16x2(p[0], p[1]);
        pp[2 * i + 1] = pack_bf16x2(p[2], p[3]);
        dsp[2 * i] = pack_bf16x2(ds[0], ds[1]);
        dsp[2 * i + 1] = pack_bf16x2(ds[2], ds[3]);
      }
      if (tj) tj[2] = globaltimer();
      tmem_st_32x32b_x32(tmem + lane_base + 256u + (uint32_t)(half * 32), pp);
      tmem_st_32x32b_x32(tmem + lane_base + 384u + (uint32_t)(half * 32), dsp);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (tj) tj[3] = globaltimer();
    }
    if (named_barrier_and(pair_bar, 64, ok)) {
      const bool done = mbar_wait(acc_done, 0, status, kErrBwdCompute);
      if (named_barrier_and(pair_bar, 64, done)) {
        tc_fence_after();
        const int64_t tok = (int64_t)b * S + key, hoff = (int64_t)hk * kAttD + col0;
#pragma unroll 1
        for (int w = 0; w < 2; ++w) {   // w = 0: dV (scale 1), w = 1: dK (scale)
          __nv_bfloat16* out = w == 0 ? dv + tok * ld_dv + hoff : dk + tok * ld_dk + hoff;
          const float f = w == 0 ? 1.0f : scale;
          // dK of rotary-embedded keys: rotated back (dV never is)
          bwd_store_half_row(tmem + lane_base + (uint32_t)(w * 128), col0, f,
                             (w == 1 && rope_cs != nullptr) ? rope_cs + (int64_t)key * 64 : nullptr, out);
        }
        if (tr && threadIdx.x == 0) tr[30] = globaltimer();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

// ============================================================================
// dK/dV backward with 64-query iterations and double-buffered Sᵀ / dPᵀ.
//
// Per key tile (one CTA), iterating over (query head, 64-query tile):
//   Sᵀ_t  = K Q_tᵀ,  dPᵀ_t = V dO_tᵀ       M = 128 keys, N = 64 queries (SS MMAs)
//   Pᵀ_t  = exp2(Sᵀ·scale·log2e - lse2),  dSᵀ_t = Pᵀ ⊙ (dPᵀ - delta)   (compute warps)
//   dV   += Pᵀ_t dO_t,  dK += dSᵀ_t Q_t     A = Pᵀ / dSᵀ from TMEM, B MN-major
// Tensor memory: dV 0-127, dK 128-255, buffer b (= t & 1): Sᵀ at 256 + 128 b
// (64 columns, then Pᵀ packed in its first 32) and dPᵀ at 320 + 128 b.
// The MMA thread issues Sᵀ/dPᵀ of iteration t + 1 before it waits for the
// compute warps' Pᵀ/dSᵀ of iteration t, so the score MMAs of the next tile run
// while the exponentials of this one are computed; buffer b is rewritten only
// by MMAs issued after the dV/dK MMAs that read it (tcgen05 MMAs of one CTA
// execute in issue order).  Q and dO stream through 4-stage rings of 64-query
// tiles (16 KB each), each dO stage with its 64 lse2 / delta values.
// ============================================================================
constexpr int kBwd64Q = 64;
constexpr int kBwd64Stages = 4;

struct BwdDkv64Smem {
  static constexpr int kTile = AttSmem::kTile, kAtom = AttSmem::kAtom;  // 128-key K / V tiles
  static constexpr int kQTile = kBwd64Q * kAttD * 2;                  // 16 KB
  static constexpr int kQAtom = kQTile / 2;                            // 64 rows x 64 D, 8 KB
  static constexpr int kK = 0, kV = kTile;
  static constexpr int kQ = 2 * kTile;
  static constexpr int kDO = kQ + kBwd64Stages * kQTile;
  static constexpr int kLD = kDO + kBwd64Stages * kQTile;              // per stage: lse2[64], delta[64]
  static constexpr int kBar = kLD + kBwd64Stages * 512;
  static constexpr int kBytes = kBar + 256 + 1024;
};

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__global__ void __launch_bounds__(kBwdThreads, 1)
attn_bwd_dkv64_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                         const float* __restrict__ lse2, const float* __restrict__ delta,
                         __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int B, int S,
                         int Hq, int Hk, float scale_log2, float scale, int causal,
                         const float2* __restrict__ rope_cs, DeviceStatus* status, int64_t ld_dk,
                         int64_t ld_dv, unsigned long long* __restrict__ trace) {
  // tmQ / tmDO: 4-D maps with a box of 64 D x 1 head x 64 rows x 1 batch
  // trace (optional, [grid][32] ns): 0 start; iterations t = 1, 2 at 1 + 8(t-1) + i:
  //   compute: i = 0 Sᵀ/dPᵀ seen, 1 loaded, 2 Pᵀ/dSᵀ computed, 3 arrived;
  //   MMA: 4 Q/dO of t seen, 5 Sᵀ/dPᵀ of t issued, 6 Pᵀ/dSᵀ seen, 7 dV/dK issued;  30 end
  unsigned long long* tr = trace ? trace + (size_t)blockIdx.x * 32 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();
  using L = BwdDkv64Smem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bars;                          // K and V landed
  uint64_t* q_full = bars + 1;                       // [kBwd64Stages]
  uint64_t* q_empty = q_full + kBwd64Stages;
  uint64_t* o_full = q_empty + kBwd64Stages;         // dO + lse2/delta
  uint64_t* o_empty = o_full + kBwd64Stages;
  uint64_t* s_full = o_empty + kBwd64Stages;         // [2] Sᵀ / dPᵀ of buffer b
  uint64_t* p_full = s_full + 2;                     // [2] Pᵀ / dSᵀ written (8 arrivals)
  uint64_t* acc_done = p_full + 2;
  uint64_t* drain = acc_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = S / kAttKeys, nq64 = S / kBwd64Q;
  const int bhk = (int)(blockIdx.x / (unsigned)nkt);
  const int kt = (int)(blockIdx.x % (unsigned)nkt);
  const int b = bhk / Hk, hk = bhk % Hk;
  const int group = Hq / Hk;
  const int i0 = causal ? 2 * kt : 0;        // first 64-query tile that sees this key tile
  const int per_head = nq64 - i0;
  const int n_it = group * per_head;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kBwd64Stages; ++i) {
      mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1);
      mbar_init(&o_full[i], 1); mbar_init(&o_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftmaxWarps);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmQ); prefetch_tmap(&tmK); prefetch_tmap(&tmV); prefetch_tmap(&tmDO);
  }
  if (warp == 8) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 9) {
    // ------------------------------------------------------------ TMA loaders
    if (lane == 0) {
      const bool is_q = warp == 9;
      if (is_q) {
        mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
        tma_load_4d(smem + L::kK, &tmK, kv_full, 0, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kK + L::kAtom, &tmK, kv_full, 64, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kV, &tmV, kv_full, 0, hk, kt * kAttKeys, b);
        tma_load_4d(smem + L::kV + L::kAtom, &tmV, kv_full, 64, hk, kt * kAttKeys, b);
      }
      const CUtensorMap* map = is_q ? &tmQ : &tmDO;
      uint64_t* empty = is_q ? q_empty : o_empty;
      uint64_t* full = is_q ? q_full : o_full;
      uint8_t* ring = smem + (is_q ? L::kQ : L::kDO);
      int issued = 0;
      bool ok = true;
      for (int t = 0; t < n_it; ++t) {
        const int st = t % kBwd64Stages;
        const int h = hk * group + t / per_head, it = i0 + t % per_head;
        if (!mbar_wait(&empty[st], ((t / kBwd64Stages) & 1) ^ 1, status, kErrBwdLoad)) { ok = false; break; }
        uint8_t* dst = ring + st * L::kQTile;
        mbar_arrive_expect_tx(&full[st], L::kQTile + (is_q ? 0 : 512));
        tma_load_4d(dst, map, &full[st], 0, h, it * kBwd64Q, b);
        tma_load_4d(dst + L::kQAtom, map, &full[st], 64, h, it * kBwd64Q, b);
        if (!is_q) {  // this query tile's lse2 and delta (256 B each)
          const int64_t li = ((int64_t)b * Hq + h) * S + it * kBwd64Q;
          bulk_load(smem + L::kLD + st * 512, lse2 + li, 256, &full[st]);
          bulk_load(smem + L::kLD + st * 512 + 256, delta + li, 256, &full[st]);
        }
        issued = t + 1;
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        if (is_q) mbar_wait(kv_full, 0, nullptr, 0);
        for (int t = (issued > kBwd64Stages ? issued - kBwd64Stages : 0); t < issued; ++t)
          mbar_wait(&full[t % kBwd64Stages], (t / kBwd64Stages) & 1, nullptr, 0);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_k = umma_idesc_bf16(kAttKeys, kBwd64Q);     // Sᵀ, dPᵀ
      constexpr uint32_t idesc_mn = umma_idesc_bf16_bmn(kAttKeys, kAttD);  // dV, dK
      const uint32_t k_addr = smem_u32(smem + L::kK), v_addr = smem_u32(smem + L::kV);
      bool ok = mbar_wait(kv_full, 0, status, kErrBwdMma);
      // Sᵀ_t and dPᵀ_t into buffer t & 1
      auto issue_scores = [&](int t) -> bool {
        unsigned long long* tj = (tr && (t == 1 || t == 2)) ? tr + 1 + 8 * (t - 1) : nullptr;
        const int st = t % kBwd64Stages;
        const uint32_t ph = (t / kBwd64Stages) & 1;
        if (!mbar_wait(&q_full[st], ph, status, kErrBwdMma)) return false;
        if (!mbar_wait(&o_full[st], ph, status, kErrBwdMma)) return false;
        if (tj) tj[4] = globaltimer();
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + L::kQ + st * L::kQTile);
        const uint32_t o_addr = smem_u32(smem + L::kDO + st * L::kQTile);
        const uint32_t sc = 256u + 128u * (uint32_t)(t & 1);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {
          const uint32_t ka = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          const uint32_t qa = (uint32_t)((kk >> 2) * L::kQAtom + (kk & 3) * 32);
          umma_f16_ss(tmem + sc, umma_desc_sw128_kmajor(k_addr + ka), umma_desc_sw128_kmajor(q_addr + qa),
                      idesc_k, kk > 0 ? 1u : 0u);
          umma_f16_ss(tmem + sc + 64u, umma_desc_sw128_kmajor(v_addr + ka),
                      umma_desc_sw128_kmajor(o_addr + qa), idesc_k, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t & 1]);
        if (tj) tj[5] = globaltimer();
        return true;
      };
      if (ok && n_it > 0) ok = issue_scores(0);
      for (int t = 0; t < n_it && ok; ++t) {
        unsigned long long* tj = (tr && (t == 1 || t == 2)) ? tr + 1 + 8 * (t - 1) : nullptr;
        if (t + 1 < n_it && !issue_scores(t + 1)) { ok = false; break; }
        if (!mbar_wait(&p_full[t & 1], (t >> 1) & 1, status, kErrBwdMma)) { ok = false; break; }
        if (tj) tj[6] = globaltimer();
        tc_fence_after();
        const int st = t % kBwd64Stages;
        const uint32_t q_addr = smem_u32(smem + L::kQ + st * L::kQTile);
        const uint32_t o_addr = smem_u32(smem + L::kDO + st * L::kQTile);
        const uint32_t sc = 256u + 128u * (uint32_t)(t & 1);
#pragma unroll
        for (int kk = 0; kk < kBwd64Q / 16; ++kk) {   // dV += Pᵀ dO and dK += dSᵀ Q, interleaved
          umma_f16_ts(tmem, tmem + sc + (uint32_t)(kk * 8),
                      umma_desc_sw128_mnmajor(o_addr + (uint32_t)kk * 2048u, (uint32_t)L::kQAtom), idesc_mn,
                      (t > 0 || kk > 0) ? 1u : 0u);
          umma_f16_ts(tmem + 128u, tmem + sc + 64u + (uint32_t)(kk * 8),
                      umma_desc_sw128_mnmajor(q_addr + (uint32_t)kk * 2048u, (uint32_t)L::kQAtom), idesc_mn,
                      (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&q_empty[st]);
        umma_commit(&o_empty[st]);
        if (tj) tj[7] = globaltimer();
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ Pᵀ, dSᵀ + epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;                     // key row = TMEM lane
    const int col0 = half * 32;                           // this half's 32 query columns
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int pair_bar = 1 + quad;
    const int key = kt * kAttKeys + row;
    bool ok = true;
    for (int t = 0; t < n_it && ok; ++t) {
      const int st = t % kBwd64Stages;
      const int it = i0 + t % per_head;
      const uint32_t sc = 256u + 128u * (uint32_t)(t & 1);
      const float* sl = reinterpret_cast<const float*>(smem + L::kLD + st * 512) + col0;
      // o_full also covers the staged lse2/delta (the bulk copies completed on it)
      unsigned long long* tj = (tr && threadIdx.x == 0 && (t == 1 || t == 2)) ? tr + 1 + 8 * (t - 1) : nullptr;
      const bool got = mbar_wait(&s_full[t & 1], (t >> 1) & 1, status, kErrBwdCompute) &&
                       mbar_wait(&o_full[st], (t / kBwd64Stages) & 1, status, kErrBwdCompute);
      if (!named_barrier_and(pair_bar, 64, got)) { ok = false; break; }
      if (tj) tj[0] = globaltimer();
      tc_fence_after();
      uint32_t sv[32], dp[32];
      tmem_ld_32x32b_x32(tmem + lane_base + sc + (uint32_t)col0, sv);
      tmem_ld_32x32b_x32(tmem + lane_base + sc + 64u + (uint32_t)col0, dp);
      tmem_ld_wait();
      if (tj) tj[1] = globaltimer();
      tc_fence_before();
      named_barrier(pair_bar, 64);   // both halves hold their columns before either overwrites
      tc_fence_after();
      const bool diag = causal && it <= 2 * kt + 1;   // some key of this tile is after some query
      const int q0 = it * kBwd64Q + col0;
      uint32_t pp[16], dsp[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {   // 4 queries per step: shared-memory broadcasts
        const float4 l4 = reinterpret_cast<const float4*>(sl)[i];
        const float4 d4 = reinterpret_cast<const float4*>(sl + 64)[i];
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
        float p[4], ds[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = 4 * i + u;
          p[u] = fast_exp2(fmaf(__uint_as_float(sv[c]), scale_log2, -lv[u]));
          if (diag && key > q0 + c) p[u] = 0.0f;
          ds[u] = p[u] * (__uint_as_float(dp[c]) - dv4[u]);
        }
        pp[2 * i] = pack_bf16x2(p[0], p[1]);
        pp[2 * i + 1] = pack_bf16x2(p[2], p[3]);
        dsp[2 * i] = pack_bf16x2(ds[0], ds[1]);
        dsp[2 * i + 1] = pack_bf16x2(ds[2], ds[3]);
      }
      if (tj) tj[2] = globaltimer();
      tmem_st_32x32b_x16(tmem + lane_base + sc + (uint32_t)(half * 16), pp);
      tmem_st_32x32b_x16(tmem + lane_base + sc + 64u + (uint32_t)(half * 16), dsp);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t & 1]);
      if (tj) tj[3] = globaltimer();
    }
    if (named_barrier_and(pair_bar, 64, ok)) {
      const bool done = mbar_wait(acc_done, 0, status, kErrBwdCompute);
      if (named_barrier_and(pair_bar, 64, done)) {
        tc_fence_after();
        const int ecol0 = half * 64;                      // epilogue: this half's 64 D columns
        const int64_t tok = (int64_t)b * S + key, hoff = (int64_t)hk * kAttD + ecol0;
#pragma unroll 1
        for (int w = 0; w < 2; ++w) {   // w = 0: dV (scale 1), w = 1: dK (scale)
          __nv_bfloat16* out = w == 0 ? dv + tok * ld_dv + hoff : dk + tok * ld_dk + hoff;
          const float f = w == 0 ? 1.0f : scale;
          bwd_store_half_row(tmem + lane_base + (uint32_t)(w * 128), ecol0, f,
                             (w == 1 && rope_cs != nullptr) ? rope_cs + (int64_t)key * 64 : nullptr, out);
        }
        if (tr && threadIdx.x == 0) tr[30] = globaltimer();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

}  // namespace zq

using namespace zq;

// [B, S, H, D] bf16 as a 4-D tensor map (dims innermost first: D, H, S, B) with a
// box of 64 D x 1 head x 128 rows x 1 batch and the 128-byte swizzle: one box is
// one 128 x 64 operand atom.
// With bhsd = true the tensor is [B, H, S, D] (heads outermost); the map keeps
// the same coordinate order (D, H, S, B), only the strides differ, so the kernel
// addresses both layouts alike.
static CUtensorMap make_tmap_bshd(const at::Tensor& t, bool bhsd = false, int box_rows = kAttRows) {
  const int64_t B = t.size(0), S = bhsd ? t.size(2) : t.size(1), H = bhsd ? t.size(1) : t.size(2),
                D = t.size(3);
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "attention: 16-byte aligned tensors");
  // any strides with unit D stride and 16-byte multiples (e.g. q/k/v as column
  // slices of one fused projection output)
  const int64_t sH = bhsd ? t.stride(1) : t.stride(2), sS = bhsd ? t.stride(2) : t.stride(1),
                sB = t.stride(0);
  TORCH_CHECK(t.stride(3) == 1 && sH % 8 == 0 && sS % 8 == 0 && sB % 8 == 0,
              "attention: unit head-dim stride and 16-byte multiple strides");
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sH * 2), (cuuint64_t)(sS * 2), (cuuint64_t)(sB * 2)};
  cuuint32_t box[4] = {64u, 1u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention: cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

// kv_bhsd: k and v are given as [B, Hk, S, D] (heads outermost) instead of
// [B, S, Hk, D]; q and o keep [B, S, Hq, D].
void attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, bool causal,
                 double scale, c10::optional<at::Tensor> trace, bool kv_bhsd) {
  for (const at::Tensor* t : {&q, &k, &v, &o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4,
                "attention: bf16 [B, S, H, D] CUDA tensors");
  }
  TORCH_CHECK(o.is_contiguous(), "attention: o must be contiguous (q/k/v may be strided)");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), D = q.size(3),
                Hk = kv_bhsd ? k.size(1) : k.size(2);
  TORCH_CHECK(D == kAttD, "attention (tcgen05): head dim 128");
  TORCH_CHECK(S % kAttRows == 0 && S > 0, "attention: S must be a multiple of 128");
  TORCH_CHECK(Hk > 0 && Hq % Hk == 0, "attention: Hq must be a multiple of Hk");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == B && k.size(kv_bhsd ? 2 : 1) == S &&
                  k.size(3) == D,
              "attention: k/v shape");
  TORCH_CHECK(o.sizes() == q.sizes(), "attention: o shape");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == B * Hq * S,
              "attention: lse [B, Hq, S] fp32");
  TORCH_CHECK(B * Hq * (S / kAttRows) < (1LL << 31), "attention: grid too large");
  const at::cuda::CUDAGuard guard(q.device());
  const int dev = q.get_device();
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        AttSmem::kBytes));
    configured[dev] = true;
  }
  const CUtensorMap tq = make_tmap_bshd(q), tk = make_tmap_bshd(k, kv_bhsd),
                    tv = make_tmap_bshd(v, kv_bhsd);
  const bool want_trace = trace.has_value() && trace->defined();
  // two query tiles per CTA when S is a multiple of 256 (ZEROQ_ATTN_FWD1=1: the
  // one-tile kernel); ZEROQ_ATTN_POLY = 0 / 4: every how many column pairs the
  // polynomial exponential takes (default 4)
  static const bool fwd1 = [] {
    const char* e = std::getenv("ZEROQ_ATTN_FWD1");
    return e != nullptr && e[0] == '1';
  }();
  static const int poly = [] {
    const char* e = std::getenv("ZEROQ_ATTN_POLY");
    return e == nullptr ? 4 : std::atoi(e);
  }();
  if (!fwd1 && S % (2 * kAttRows) == 0) {
    static bool configured2[64] = {false};
    if (!configured2[dev]) {
      for (auto k2 : {attn_fwd2_tc_kernel<0, false>, attn_fwd2_tc_kernel<4, false>,
                      attn_fwd2_tc_kernel<0, true>, attn_fwd2_tc_kernel<4, true>})
        C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, Fwd2Smem::kBytes));
      configured2[dev] = true;
    }
    const unsigned grid2 = (unsigned)(B * Hq * (S / (2 * kAttRows)));
    unsigned long long* trp2 = nullptr;
    if (want_trace) {
      TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                      trace->numel() >= (int64_t)grid2 * kTraceSlots,
                  "attention trace: int64 CUDA tensor of [grid, 32]");
      trp2 = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
    }
    auto kern = want_trace ? (poly == 4 ? attn_fwd2_tc_kernel<4, true> : attn_fwd2_tc_kernel<0, true>)
                           : (poly == 4 ? attn_fwd2_tc_kernel<4, false> : attn_fwd2_tc_kernel<0, false>);
    kern<<<grid2, kF2Threads, Fwd2Smem::kBytes, at::cuda::getCurrentCUDAStream()>>>(
        tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(o.data_ptr<at::BFloat16>()), lse.data_ptr<float>(),
        (int)B, (int)S, (int)Hq, (int)Hk, (float)(scale * 1.4426950408889634), causal ? 1 : 0,
        status_buffer(dev), trp2);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const unsigned grid = (unsigned)(B * Hq * (S / kAttRows));
  unsigned long long* trp = nullptr;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= (int64_t)grid * kTraceSlots,
                "attention trace: int64 CUDA tensor of [grid, 32]");
    trp = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  attn_fwd_tc_kernel<<<grid, kAttThreads, AttSmem::kBytes, at::cuda::getCurrentCUDAStream()>>>(
      tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(o.data_ptr<at::BFloat16>()), lse.data_ptr<float>(),
      (int)B, (int)S, (int)Hq, (int)Hk, (float)(scale * 1.4426950408889634), causal ? 1 : 0,
      status_buffer(dev), trp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward of attn_fwd_tc: dq, dk, dv [B, S, H, D] bf16 from dout, q, k, v, o and
// the forward's lse.  Two launches: dQ (per query tile; writes delta and lse2 too),
// then dK/dV (per key tile).
// trace (optional): int64 [dQ grid + dK/dV grid, 32] per-CTA timestamps.
void attn_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                 at::Tensor lse, at::Tensor dq, at::Tensor dk, at::Tensor dv, bool causal,
                 double scale, c10::optional<at::Tensor> trace, c10::optional<at::Tensor> rope_cs) {
  for (const at::Tensor* t : {&dout, &q, &k, &v, &o, &dq, &dk, &dv}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4,
                "attention backward: bf16 [B, S, H, D] CUDA tensors");
  }
  for (const at::Tensor* t : {&dout, &o, &dq})
    TORCH_CHECK(t->is_contiguous(), "attention backward: dout, o, dq must be contiguous");
  // dK / dV: [B, S, H, D] with unit head-dim stride, D between heads and any
  // 16-byte-multiple token pitch (a column slice of a wider gradient buffer)
  for (const at::Tensor* t : {&dk, &dv})
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == t->size(3) && t->stride(1) >= t->size(2) * t->size(3) &&
                    t->stride(1) % 8 == 0 && t->stride(0) == t->size(1) * t->stride(1) &&
                    (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0,
                "attention backward: dk / dv must be [B, S, H, D] rows of a token-pitched buffer");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), D = q.size(3), Hk = k.size(2);
  TORCH_CHECK(D == kAttD, "attention backward (tcgen05): head dim 128");
  TORCH_CHECK(S % kAttRows == 0 && S > 0, "attention backward: S must be a multiple of 128");
  TORCH_CHECK(Hk > 0 && Hq % Hk == 0, "attention backward: Hq must be a multiple of Hk");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == B && k.size(1) == S && k.size(3) == D &&
                  dk.sizes() == k.sizes() && dv.sizes() == v.sizes() && dq.sizes() == q.sizes() &&
                  o.sizes() == q.sizes() && dout.sizes() == q.sizes(),
              "attention backward: shapes");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == B * Hq * S,
              "attention backward: lse [B, Hq, S] fp32");
  const at::cuda::CUDAGuard guard(q.device());
  const int dev = q.get_device();
  auto stream = at::cuda::getCurrentCUDAStream();
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BwdDqSmem::kBytes));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_dkv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BwdDkvSmem::kBytes));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_dkv64_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BwdDkv64Smem::kBytes));
    configured[dev] = true;
  }
  const float2* rcs = nullptr;
  if (rope_cs.has_value() && rope_cs->defined()) {
    const at::Tensor& t = *rope_cs;
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.dim() == 3 &&
                    t.size(0) == S && t.size(1) == 64 && t.size(2) == 2,
                "attention backward: rope table must be fp32 [S, 64, 2]");
    rcs = reinterpret_cast<const float2*>(t.data_ptr<float>());
  }
  auto delta = at::empty({B, Hq, S}, q.options().dtype(at::kFloat));
  auto lse2 = at::empty({B, Hq, S}, q.options().dtype(at::kFloat));
  // delta = rowsum(dO ∘ O) and lse2 = lse·log2(e) are produced by the dQ kernel
  // (each query row by the CTA that owns it) for the dK/dV kernel launched after it
  const CUtensorMap tq = make_tmap_bshd(q), tk = make_tmap_bshd(k), tv = make_tmap_bshd(v),
                    tdo = make_tmap_bshd(dout);
  const float sl2 = (float)(scale * 1.4426950408889634);
  DeviceStatus* st = status_buffer(dev);
  const int64_t g_dq = B * Hq * (S / kAttRows), g_dkv = B * Hk * (S / kAttKeys);
  unsigned long long* trp = nullptr;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= (g_dq + g_dkv) * 32,
                "attention backward trace: int64 [dQ grid + dK/dV grid, 32]");
    trp = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  attn_bwd_dq_tc_kernel<<<(unsigned)g_dq, kBwdThreads, BwdDqSmem::kBytes, stream>>>(
      tq, tk, tv, tdo, lse.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(o.data_ptr<at::BFloat16>()), delta.data_ptr<float>(),
      lse2.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dq.data_ptr<at::BFloat16>()), (int)B, (int)S, (int)Hq, (int)Hk, sl2,
      (float)scale, causal ? 1 : 0, rcs, st, trp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // dK/dV: 64-query iterations with double-buffered scores (overlapping the score
  // MMAs of the next tile with this tile's exponentials); ZEROQ_ATTN_DKV128=1 or a
  // trace request selects the 128-query kernel
  static const bool dkv128 = [] {
    const char* e = std::getenv("ZEROQ_ATTN_DKV128");
    return e != nullptr && e[0] == '1';
  }();
  if (dkv128) {
    attn_bwd_dkv_tc_kernel<<<(unsigned)g_dkv, kBwdThreads, BwdDkvSmem::kBytes, stream>>>(
        tq, tk, tv, tdo, lse2.data_ptr<float>(), delta.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dk.data_ptr<at::BFloat16>()),
        reinterpret_cast<__nv_bfloat16*>(dv.data_ptr<at::BFloat16>()), (int)B, (int)S, (int)Hq, (int)Hk, sl2,
        (float)scale, causal ? 1 : 0, rcs, st, trp ? trp + g_dq * 32 : nullptr, dk.stride(1), dv.stride(1));
  } else {
    const CUtensorMap tq64 = make_tmap_bshd(q, false, kBwd64Q), tdo64 = make_tmap_bshd(dout, false, kBwd64Q);
    attn_bwd_dkv64_tc_kernel<<<(unsigned)g_dkv, kBwdThreads, BwdDkv64Smem::kBytes, stream>>>(
        tq64, tk, tv, tdo64, lse2.data_ptr<float>(), delta.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dk.data_ptr<at::BFloat16>()),
        reinterpret_cast<__nv_bfloat16*>(dv.data_ptr<at::BFloat16>()), (int)B, (int)S, (int)Hq, (int)Hk, sl2,
        (float)scale, causal ? 1 : 0, rcs, st, dk.stride(1), dv.stride(1), trp ? trp + g_dq * 32 : nullptr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

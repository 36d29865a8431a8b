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

}  // namespace zq

using namespace zq;

// [B, S, H, D] bf16 as a 4-D tensor map (dims innermost first: D, H, S, B) with a
// box of 64 D x 1 head x 128 rows x 1 batch and the 128-byte swizzle: one box is
// one 128 x 64 operand atom.
// With bhsd = true the tensor is [B, H, S, D] (heads outermost); the map keeps
// the same coordinate order (D, H, S, B), only the strides differ, so the kernel
// addresses both layouts alike.
static CUtensorMap make_tmap_bshd(const at::Tensor& t, bool bhsd = false) {
  const int64_t B = t.size(0), S = bhsd ? t.size(2) : t.size(1), H = bhsd ? t.size(1) : t.size(2),
                D = t.size(3);
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "attention: 16-byte aligned tensors");
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(bhsd ? S * D * 2 : D * 2), (cuuint64_t)(bhsd ? D * 2 : H * D * 2),
                           (cuuint64_t)(S * H * D * 2)};
  cuuint32_t box[4] = {64u, 1u, (cuuint32_t)kAttRows, 1u};
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
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4,
                "attention: contiguous bf16 [B, S, H, D] CUDA tensors");
  }
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

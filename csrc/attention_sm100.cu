// Flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// q, k, v, o: [B, S, H, D] bf16 (projection layout, no transposes), D = 128,
// S % 128 == 0, GQA (Hq a multiple of Hk); lse [B, Hq, S] fp32, natural log of
// the softmax denominator of the scaled scores (what the backward expects).
//
// One CTA per (128-query tile, head, batch); 192 threads:
//   warps 0-3  softmax + epilogue: thread t owns query row t = TMEM lane t.
//   warp 4     MMA issuer (one thread) and TMEM owner (512 columns:
//              S double buffer at columns 0 / 128, O at 256).
//   warp 5     TMA loader (one thread): Q once, K/V tiles of 128 keys into a
//              two-stage ring (4-D tensor maps over [B, S, H, D], 128-byte swizzle).
// Per key tile j:
//   S_j = Q K_jᵀ            tcgen05.mma, A = Q (smem, K-major), B = K_j (smem, K-major)
//   softmax_j (registers)   row max; P_j = exp2(S_j·scale·log2e - m) as bf16 into a
//                           swizzled smem tile; row sums in fp32
//   O += P_j V_j            tcgen05.mma, A = P_j (smem, K-major), B = V_j read MN-major
// The MMA thread issues S_{j+1} before PV_j so softmax_{j+1} overlaps PV_j.  The
// running max m only moves when a row's new max exceeds it by more than 8 (log2
// units): exponentials stay <= 2^8 and O (in TMEM) is rescaled only then, which
// after the first tiles is rare.  The final O / l and lse use the same m, so the
// result is exact softmax attention.
//
// Causal: query tile qt visits key tiles 0..qt; only the diagonal tile is masked.
// CTAs are numbered so the largest qt (most work) start first.
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
constexpr int kAttThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum AttErr { kErrAttLoad = 301, kErrAttMma = 302, kErrAttSoftmax = 303 };

struct AttSmem {
  // a 128 x 128 bf16 tile = two 128-byte-swizzled atoms of 128 rows x 64 columns
  static constexpr int kTile = kAttRows * kAttD * 2;   // 32 KB
  static constexpr int kAtom = kTile / 2;              // 16 KB
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;                 // 2 stages
  static constexpr int kV = kK + 2 * kTile;             // 2 stages
  static constexpr int kP = kV + 2 * kTile;             // 2 buffers
  static constexpr int kBar = kP + 2 * kTile;           // 224 KB
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
                   int causal, DeviceStatus* status) {
  using L = AttSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;     // [2]
  uint64_t* pv_done = bars + 11;   // [2]
  uint64_t* drain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nqt = S / kAttRows;
  const int qt = nqt - 1 - (int)(blockIdx.x / (unsigned)(B * Hq));
  const int bh = (int)(blockIdx.x % (unsigned)(B * Hq));
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hk);
  const int n_kv = causal ? qt + 1 : nqt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
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
  if (warp == 4) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint8_t* sQ = smem + L::kQ;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA loader
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kTile);
      tma_load_4d(sQ, &tmQ, q_full, 0, h, qt * kAttRows, b);
      tma_load_4d(sQ + L::kAtom, &tmQ, q_full, 64, h, qt * kAttRows, b);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, status, kErrAttLoad)) { ok = false; break; }
        uint8_t* sK = smem + L::kK + st * L::kTile;
        uint8_t* sV = smem + L::kV + st * L::kTile;
        mbar_arrive_expect_tx(&k_full[st], L::kTile);
        tma_load_4d(sK, &tmK, &k_full[st], 0, hk, j * kAttKeys, b);
        tma_load_4d(sK + L::kAtom, &tmK, &k_full[st], 64, hk, j * kAttKeys, b);
        mbar_arrive_expect_tx(&v_full[st], L::kTile);
        tma_load_4d(sV, &tmV, &v_full[st], 0, hk, j * kAttKeys, b);
        tma_load_4d(sV + L::kAtom, &tmV, &v_full[st], 64, hk, j * kAttKeys, b);
        issued = j + 1;
      }
      if (!ok) {  // let every copy this thread issued land before the CTA can exit
        mbar_wait(q_full, 0, nullptr, 0);
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, 0);
          mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, 0);
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kAttRows, kAttKeys);
      constexpr uint32_t idesc_pv = umma_idesc_bf16_bmn(kAttRows, kAttD);
      bool ok = mbar_wait(q_full, 0, status, kErrAttMma);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, status, kErrAttMma)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kK + st * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttD / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          umma_f16_ss(tmem + (uint32_t)(st * kAttKeys), umma_desc_sw128_kmajor(q_addr + off),
                      umma_desc_sw128_kmajor(k_addr + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        const int st = j & 1;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1, status, kErrAttMma)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, status, kErrAttMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + L::kP + st * L::kTile);
        const uint32_t v_addr = smem_u32(smem + L::kV + st * L::kTile);
#pragma unroll
        for (int kk = 0; kk < kAttKeys / 16; ++kk) {
          const uint32_t poff = (uint32_t)((kk >> 2) * L::kAtom + (kk & 3) * 32);
          // V tile: two 64-column (D) atoms of 128 key rows; 16 keys = 2048 B
          umma_f16_ss(tmem + 256u, umma_desc_sw128_kmajor(p_addr + poff),
                      umma_desc_sw128_mnmajor(v_addr + (uint32_t)kk * 2048u, (uint32_t)L::kAtom),
                      idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[st]);
        umma_commit(&pv_done[st]);
      }
      // every MMA issued by this thread has completed before TMEM can be freed
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int row = warp * 32 + lane;               // query row in the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_used = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int st = j & 1;
      const bool got = mbar_wait(&s_full[st], (j >> 1) & 1, status, kErrAttSoftmax);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[kAttKeys];
#pragma unroll
      for (int c = 0; c < kAttKeys / 32; ++c)
        tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(st * kAttKeys + c * 32),
                           *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_ld_wait();
      const bool diag = causal && j == qt;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAttKeys; ++c) {
        const float sv = __uint_as_float(r[c]);
        if (!diag || c <= row) mx = fmaxf(mx, sv);
      }
      mx *= scale_log2;
      const bool need = mx > m_used + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_used;
        const float factor = (m_used == -INFINITY) ? 0.0f : fast_exp2(m_used - m_new);
        if (j > 0) {
          // O holds PV_0..PV_{j-1}: wait for PV_{j-1}, then scale the rows in TMEM
          const bool pv = mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, status, kErrAttSoftmax);
          if (!__all_sync(0xffffffffu, pv)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kAttD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tmem + lane_base + 256u + (uint32_t)(c * 32), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            tmem_st_32x32b_x32(tmem + lane_base + 256u + (uint32_t)(c * 32), o);
          }
          tmem_st_wait();
        }
        l *= factor;
        m_used = m_new;
      }
      // P buffer st was last read by PV_{j-2}
      if (j >= 2) {
        const bool pf = mbar_wait(&pv_done[st], ((j - 2) >> 1) & 1, status, kErrAttSoftmax);
        if (!__all_sync(0xffffffffu, pf)) { ok = false; break; }
      }
      uint8_t* prow = smem + L::kP + st * L::kTile + row * 128;
      float sum = 0.0f;
#pragma unroll
      for (int ch = 0; ch < kAttKeys / 8; ++ch) {  // 16 chunks of 8 keys
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c0 = ch * 8 + 2 * i;
          float p0 = fast_exp2(__uint_as_float(r[c0]) * scale_log2 - m_used);
          float p1 = fast_exp2(__uint_as_float(r[c0 + 1]) * scale_log2 - m_used);
          if (diag && c0 > row) p0 = 0.0f;
          if (diag && c0 + 1 > row) p1 = 0.0f;
          sum += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        // atom ch/8 (keys 0-63 | 64-127), 16-byte chunk ch%8 swizzled by the row
        *reinterpret_cast<uint4*>(prow + (ch >> 3) * L::kAtom + (((ch & 7) ^ (row & 7)) << 4)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += sum;
      fence_proxy_async_smem();   // P stores -> visible to the tensor core
      tc_fence_before();          // TMEM loads/stores of this step ordered before the arrive
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    if (ok) {
      const int jl = n_kv - 1;
      const bool done = mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, status, kErrAttSoftmax);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float inv = 1.0f / l;
        const int q = qt * kAttRows + row;
        __nv_bfloat16* orow = O + (((int64_t)b * S + q) * Hq + h) * kAttD;
#pragma unroll 1
        for (int c = 0; c < kAttD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256u + (uint32_t)(c * 32), o);
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
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace zq

using namespace zq;

// [B, S, H, D] bf16 as a 4-D tensor map (dims innermost first: D, H, S, B) with a
// box of 64 D x 1 head x 128 rows x 1 batch and the 128-byte swizzle: one box is
// one 128 x 64 operand atom.
static CUtensorMap make_tmap_bshd(const at::Tensor& t) {
  const int64_t B = t.size(0), S = t.size(1), H = t.size(2), D = t.size(3);
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "attention: 16-byte aligned tensors");
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2), (cuuint64_t)(S * H * D * 2)};
  cuuint32_t box[4] = {64u, 1u, (cuuint32_t)kAttRows, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention: cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

void attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse, bool causal,
                 double scale) {
  for (const at::Tensor* t : {&q, &k, &v, &o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4,
                "attention: contiguous bf16 [B, S, H, D] CUDA tensors");
  }
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), D = q.size(3), Hk = k.size(2);
  TORCH_CHECK(D == kAttD, "attention (tcgen05): head dim 128");
  TORCH_CHECK(S % kAttRows == 0 && S > 0, "attention: S must be a multiple of 128");
  TORCH_CHECK(Hk > 0 && Hq % Hk == 0, "attention: Hq must be a multiple of Hk");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == B && k.size(1) == S && k.size(3) == D,
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
  const CUtensorMap tq = make_tmap_bshd(q), tk = make_tmap_bshd(k), tv = make_tmap_bshd(v);
  const unsigned grid = (unsigned)(B * Hq * (S / kAttRows));
  attn_fwd_tc_kernel<<<grid, kAttThreads, AttSmem::kBytes, at::cuda::getCurrentCUDAStream()>>>(
      tq, tk, tv, reinterpret_cast<__nv_bfloat16*>(o.data_ptr<at::BFloat16>()), lse.data_ptr<float>(),
      (int)B, (int)S, (int)Hq, (int)Hk, (float)(scale * 1.4426950408889634), causal ? 1 : 0,
      status_buffer(dev));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Peer-memory collectives over NVLink / NVSwitch, one process per GPU.
//
// Buffers are plain cudaMalloc allocations shared between the ranks of one node
// with CUDA IPC handles (exchanged by the Python side over the process group);
// every kernel below addresses peers' buffers directly with ordinary 16-byte
// loads and stores (no TMA).
//
// Synchronisation between ranks uses per-rank flag words in peer memory with
// system-scope release/acquire and a monotonically increasing epoch.  Every
// wait is bounded (kPeerWaitNs); a timeout records an error in the rank's
// status word and the kernel stops working and exits, so a missing peer turns
// into an error the host reads, not a hung GPU.
//
// Kernels:
//   rs_adamw   - reduce-scatter of a flat gradient fused with the AdamW update
//                of this rank's shard and (optionally) the all-gather of the
//                updated shard into every peer's parameter buffer.
//   gather     - assemble a flat buffer whose pieces are laid out on the ranks
//                by an arbitrary (weighted / uneven) shard plan.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <string>
#include <vector>

#include "common.cuh"
#include "peer_gather.cuh"

namespace zq {

constexpr unsigned long long kPeerWaitNsDefault = 10000000000ull;  // 10 s
constexpr int kMaxRanks = 8;

// Flag block of one rank (int32 words, in IPC memory):
//   [0 .. 7]    start-barrier epochs written by rank q into slot q
//   [8 .. 15]   end-barrier epochs
//   [16]        local "go" word (this rank's CTAs wait on it)
//   [17]        local arrival counter for the end barrier
//   [18..19]    status (code, detail)
constexpr int kFlagStart = 0, kFlagEnd = 8, kFlagGo = 16, kFlagCount = 17, kFlagStatus = 18;
constexpr int kFlagWords = 32;

struct PeerTable {
  int64_t ptr[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void peer_status(int* flags, int code, int detail) {
  if (atomicCAS(flags + kFlagStatus, 0, code) == 0) flags[kFlagStatus + 1] = detail;
}

// Signal `slot_base + rank` = epoch in every rank's flag block, then wait until
// this rank's block has `epoch` from every rank.  Returns false on timeout.
__device__ bool cross_rank_barrier(const PeerTable& flags, int rank, int world, int slot_base,
                                   int epoch, unsigned long long wait_ns) {
  __threadfence_system();
  for (int q = 0; q < world; ++q) {
    int* f = reinterpret_cast<int*>(flags.ptr[q]);
    st_release_sys(f + slot_base + rank, epoch);
  }
  const int* mine = reinterpret_cast<const int*>(flags.ptr[rank]);
  const unsigned long long t0 = globaltimer();
  for (int q = 0; q < world; ++q) {
    while (ld_acquire_sys(mine + slot_base + q) < epoch) {
      if (globaltimer() - t0 > wait_ns) {
        peer_status(reinterpret_cast<int*>(flags.ptr[rank]), 201 + slot_base, q);
        return false;
      }
    }
  }
  return true;
}

// All CTAs: the grid's CTA 0 runs the start barrier and publishes "go"; the
// others wait for it (the grid is sized to be fully resident).
// epoch 0: no cross-rank synchronisation (the data read is static)
__device__ bool grid_start(const PeerTable& flags, int rank, int world, int epoch,
                           unsigned long long wait_ns) {
  if (epoch == 0) return true;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int* mine = reinterpret_cast<int*>(flags.ptr[rank]);
    ok = 1;
    if (blockIdx.x == 0) {
      if (!cross_rank_barrier(flags, rank, world, kFlagStart, epoch, wait_ns)) {
        ok = 0;
        st_release_gpu(mine + kFlagGo, -epoch);
      } else {
        st_release_gpu(mine + kFlagGo, epoch);
      }
    } else {
      const unsigned long long t0 = globaltimer();
      int g;
      while ((g = ld_acquire_gpu(mine + kFlagGo)) != epoch && g != -epoch) {
        if (globaltimer() - t0 > wait_ns + 1000000000ull) {
          peer_status(mine, 210, blockIdx.x);
          g = -epoch;
          break;
        }
      }
      ok = (g == epoch);
    }
  }
  __syncthreads();
  return ok != 0;
}

// All CTAs: count arrivals; the last CTA runs the end barrier (so no rank
// reuses its buffers while a peer still reads or writes them).
__device__ void grid_end(const PeerTable& flags, int rank, int world, int epoch,
                         unsigned long long wait_ns) {
  if (epoch == 0) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    int* mine = reinterpret_cast<int*>(flags.ptr[rank]);
    __threadfence_system();
    const int prev = atomicAdd(mine + kFlagCount, 1);
    if (prev == (int)gridDim.x - 1) {
      mine[kFlagCount] = 0;
      cross_rank_barrier(flags, rank, world, kFlagEnd, epoch, wait_ns);
    }
  }
}

template <typename G>
__device__ __forceinline__ float4 load4(const G* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// grads[q] + lo .. lo+n: rank q's full flat gradient (only our shard is read);
// params[q]: rank q's flat fp32 parameter buffer; master = params[rank] + lo.
template <typename G>
__global__ void __launch_bounds__(256) rs_adamw_kernel(PeerTable grads, PeerTable params, PeerTable flags,
                                                       int rank, int world, int epoch, int64_t lo,
                                                       int64_t n, float* __restrict__ m,
                                                       float* __restrict__ v, float lr, float b1,
                                                       float b2, float eps, float wd, float bc1,
                                                       float bc2, float gscale, int push,
                                                       unsigned long long wait_ns,
                                                       const int64_t* __restrict__ clk,
                                                       const float* __restrict__ bcp,
                                                       const float* __restrict__ clip_sq, float max_norm,
                                                       int epoch_mul, int epoch_add) {
  // device-side optimizer clock (CUDA-graph replays): epoch and bias corrections
  // written by opt_tick earlier on this stream instead of launch arguments (a
  // step that runs two peer kernels takes epochs clk * 2 and clk * 2 + 1)
  if (clk != nullptr) epoch = (int)clk[1] * epoch_mul + epoch_add;
  if (bcp != nullptr) {
    bc1 = bcp[0];
    bc2 = bcp[1];
  }
  // gradient clipping: clip_sq holds the squared norm of the averaged gradient
  // (rs_sumsq, then summed over the ranks); scale by min(1, max_norm / norm)
  if (clip_sq != nullptr) gscale *= fminf(1.0f, max_norm / (sqrtf(*clip_sq) + 1e-6f));
  const bool ok = grid_start(flags, rank, world, epoch, wait_ns);
  if (ok) {
    const float step_size = lr / bc1;
    const float inv_sqrt_bc2 = rsqrtf(bc2);
    float* master = reinterpret_cast<float*>(params.ptr[rank]) + lo;
    const int64_t n4 = n >> 2;
    constexpr int U = 4;  // independent 4-element groups in flight per thread
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < n4; base += stride * U) {
      float4 g[U];
#pragma unroll
      for (int u = 0; u < U; ++u) g[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      // issue every peer load of the U groups before using any of them
      for (int q = 0; q < world; ++q) {
        const G* gq = reinterpret_cast<const G*>(grads.ptr[q]) + lo;
        float4 t[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = base + u * stride;
          t[u] = i < n4 ? load4<G>(gq + i * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          g[u].x += t[u].x; g[u].y += t[u].y; g[u].z += t[u].z; g[u].w += t[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = base + u * stride;
        if (i >= n4) break;
        const int64_t e = i * 4;
        float4 p = *reinterpret_cast<const float4*>(master + e);
        float4 mm = *reinterpret_cast<const float4*>(m + e);
        float4 vv = *reinterpret_cast<const float4*>(v + e);
        float* pp = &p.x;
        float* mp = &mm.x;
        float* vp = &vv.x;
        const float* gp = &g[u].x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float gi = gp[j] * gscale;
          float pi = pp[j] * (1.0f - lr * wd);
          mp[j] = b1 * mp[j] + (1.0f - b1) * gi;
          vp[j] = b2 * vp[j] + (1.0f - b2) * gi * gi;
          pi -= step_size * mp[j] / (sqrtf(vp[j]) * inv_sqrt_bc2 + eps);
          pp[j] = pi;
        }
        *reinterpret_cast<float4*>(m + e) = mm;
        *reinterpret_cast<float4*>(v + e) = vv;
        *reinterpret_cast<float4*>(master + e) = p;
        if (push) {
          for (int q = 0; q < world; ++q) {
            if (q == rank) continue;
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(params.ptr[q]) + lo + e) = p;
          }
        }
      }
    }
  }
  grid_end(flags, rank, world, epoch, wait_ns);
}

// sq[0] += sum over this rank's shard [lo, lo + n) of (gscale * sum_q grads[q][i])^2:
// the squared norm of the averaged gradient's shard, read over NVLink like
// rs_adamw reads it (same barriers), for gradient clipping without a host sync.
template <typename G>
__global__ void __launch_bounds__(256) rs_sumsq_kernel(PeerTable grads, PeerTable flags, int rank, int world,
                                                       int epoch, int64_t lo, int64_t n, float gscale,
                                                       float* __restrict__ sq, unsigned long long wait_ns,
                                                       const int64_t* __restrict__ clk, int epoch_mul,
                                                       int epoch_add) {
  if (clk != nullptr) epoch = (int)clk[1] * epoch_mul + epoch_add;
  __shared__ float red[8];
  const bool ok = grid_start(flags, rank, world, epoch, wait_ns);
  float acc = 0.0f;
  if (ok) {
    const int64_t n4 = n >> 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < world; ++q) {
        const float4 t = load4<G>(reinterpret_cast<const G*>(grads.ptr[q]) + lo + i * 4);
        g.x += t.x; g.y += t.y; g.z += t.z; g.w += t.w;
      }
      g.x *= gscale; g.y *= gscale; g.z *= gscale; g.w *= gscale;
      acc += g.x * g.x + g.y * g.y + g.z * g.z + g.w * g.w;
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    v = warp_sum(v);
    if (threadIdx.x == 0 && v != 0.0f) atomicAdd(sq, v);
  }
  grid_end(flags, rank, world, epoch, wait_ns);
}

// out[0 .. total): for every rank q, its piece src[q][0 .. len_q) lands at
// out[off_q ..).  Works for any plan (uneven or weighted); bytes, 16-byte chunks
// where aligned.
__global__ void __launch_bounds__(256) plan_gather_kernel(PeerTable src, PeerTable flags, int rank,
                                                          int world, int epoch, PeerTable offs,
                                                          PeerTable lens, uint8_t* __restrict__ out,
                                                          unsigned long long wait_ns) {
  const bool ok = grid_start(flags, rank, world, epoch, wait_ns);
  if (ok) {
    for (int q = 0; q < world; ++q) {
      const uint8_t* s = reinterpret_cast<const uint8_t*>(src.ptr[q]);
      const int64_t off = offs.ptr[q], len = lens.ptr[q];
      uint8_t* d = out + off;
      const bool vec = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0;
      const int64_t nv = vec ? len / 16 : 0;
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
           i += (int64_t)gridDim.x * blockDim.x)
        reinterpret_cast<uint4*>(d)[i] = reinterpret_cast<const uint4*>(s)[i];
      for (int64_t i = nv * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len;
           i += (int64_t)gridDim.x * blockDim.x)
        d[i] = s[i];
    }
  }
  grid_end(flags, rank, world, epoch, wait_ns);
}

// Gather + dequantise in one pass: element e of the [rows, cols] NF4 weight
// takes its packed byte from the rank that owns byte e/2 under `pplan` and its
// scale from the rank that owns block e/blocksize under `aplan` (the two plans
// are independent, as in the weighted split).  Each thread expands 16 elements
// and writes them as bf16, either as [rows, cols] or transposed [cols, rows]
// (through a 64x64 shared-memory tile).
__constant__ float c_p2p_code[2][16] = {
    {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
     -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
     0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
     0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f},
    {0.0f, 0.005208333333f, 0.66666667f, 1.0f, 0.33333333f, 0.5f, 0.16666667f, 0.25f, -0.0f,
     -0.005208333333f, -0.66666667f, -1.0f, -0.33333333f, -0.5f, -0.16666667f, -0.25f}};

__device__ __forceinline__ int plan_owner(const PeerTable& starts, int world, int64_t idx) {
  int q = 0;
  for (int r = 1; r < world; ++r)
    if (idx >= starts.ptr[r]) q = r;
  return q;
}

__device__ __forceinline__ uint8_t peer_byte(const PeerTable& src, const PeerTable& starts, int world,
                                             int64_t idx) {
  const int q = plan_owner(starts, world, idx);
  return reinterpret_cast<const uint8_t*>(src.ptr[q])[idx - starts.ptr[q]];
}

__global__ void __launch_bounds__(256) plan_gather_dequant_kernel(
    PeerTable psrc, PeerTable pstart, PeerTable asrc, PeerTable astart, int world, int rows,
    int cols, int64_t row0, int blocksize, int qtype, int transpose, __nv_bfloat16* __restrict__ out) {
  __shared__ float lut[16];
  __shared__ __align__(16) __nv_bfloat16 tile[64][64 + 8];
  if (threadIdx.x < 16) lut[threadIdx.x] = c_p2p_code[qtype][threadIdx.x];
  __syncthreads();
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const int tr = threadIdx.x >> 2, tc = (threadIdx.x & 3) * 16;
  const int r = r0 + tr, c = c0 + tc;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = 0.0f;
  if (r < rows && c < cols) {
    const int64_t e0 = (row0 + r) * (int64_t)cols + c;
    const int64_t b0 = e0 >> 1;
    const int qa = plan_owner(astart, world, e0 / blocksize);
    const float s = reinterpret_cast<const float*>(asrc.ptr[qa])[e0 / blocksize - astart.ptr[qa]];
    const int q0 = plan_owner(pstart, world, b0);
    const int64_t local0 = b0 - pstart.ptr[q0];
    const bool one_owner = (q0 == world - 1 || b0 + 8 <= pstart.ptr[q0 + 1]);
    const uint8_t* sp = reinterpret_cast<const uint8_t*>(psrc.ptr[q0]) + local0;
    uint32_t w[2];
    if (c + 16 <= cols && one_owner && (reinterpret_cast<uintptr_t>(sp) & 7) == 0) {
      const uint2 pk = *reinterpret_cast<const uint2*>(sp);
      w[0] = pk.x;
      w[1] = pk.y;
    } else {
      w[0] = w[1] = 0;
      for (int i = 0; i < 8 && c + 2 * i < cols; ++i)
        w[i >> 2] |= (uint32_t)peer_byte(psrc, pstart, world, b0 + i) << (8 * (i & 3));
    }
    // blocks never straddle a 16-element chunk when blocksize >= 16 and cols % 16 == 0
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFF;
      v[2 * i] = lut[byte >> 4] * s;
      v[2 * i + 1] = lut[byte & 0xF] * s;
    }
  }
  if (!transpose) {
    if (r < rows && c + 16 <= cols) {
      uint4 o0, o1;
      o0.x = pack_bf16x2(v[0], v[1]);   o0.y = pack_bf16x2(v[2], v[3]);
      o0.z = pack_bf16x2(v[4], v[5]);   o0.w = pack_bf16x2(v[6], v[7]);
      o1.x = pack_bf16x2(v[8], v[9]);   o1.y = pack_bf16x2(v[10], v[11]);
      o1.z = pack_bf16x2(v[12], v[13]); o1.w = pack_bf16x2(v[14], v[15]);
      uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)r * cols + c);
      dst[0] = o0;
      dst[1] = o1;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) tile[tc + i][tr] = __float2bfloat16_rn(v[i]);
  __syncthreads();
  const int oc = c0 + tr, orow0 = r0 + tc;
  if (oc < cols && orow0 + 16 <= rows) {
    const uint32_t* sv = reinterpret_cast<const uint32_t*>(&tile[tr][tc]);
    uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)oc * rows + orow0);
    dst[0] = make_uint4(sv[0], sv[1], sv[2], sv[3]);
    dst[1] = make_uint4(sv[4], sv[5], sv[6], sv[7]);
  }
}

// Non-transposed peer gather + dequantise, one warp per item of 8 rows x 1024
// columns (16-byte loads, 8 in flight per lane): rows [row0, row0 + rows) of
// W [*, K] into out_base + r * K (out_base = output - row0 * K).
__global__ void __launch_bounds__(256) ag_dequant_kernel(AgSource s, int K, int row0, int rows,
                                                         int blocksize, int qtype,
                                                         __nv_bfloat16* out_base) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = c_p2p_code[qtype][threadIdx.x];
  __syncthreads();
  const int kchunks = (K + kAgCols - 1) / kAgCols;
  const int64_t total = (int64_t)((rows + kAgRows - 1) / kAgRows) * kchunks;
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t it = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < total; it += nw) {
    const int rg = (int)(it / kchunks), kc = (int)(it - (int64_t)rg * kchunks);
    ag_item(s, lut, row0 + rows, K, blocksize, row0 + rg * kAgRows, kc * kAgCols, out_base, lane);
  }
}

}  // namespace zq

using namespace zq;

static PeerTable table_from(const std::vector<int64_t>& v) {
  TORCH_CHECK((int)v.size() <= kMaxRanks, "at most 8 ranks per node");
  PeerTable t{};
  for (size_t i = 0; i < v.size(); ++i) t.ptr[i] = v[i];
  return t;
}

// ---------------------------------------------------------------- IPC plumbing
std::vector<int64_t> peer_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  return {reinterpret_cast<int64_t>(p)};
}

at::Tensor peer_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t peer_open(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void peer_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

void peer_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel},
                       at::TensorOptions().dtype(dtype).device(at::kCUDA, device));
}

std::vector<int64_t> peer_status_read(int64_t flags_ptr) {
  int st[2] = {0, 0};
  C10_CUDA_CHECK(cudaMemcpy(st, reinterpret_cast<int*>(flags_ptr) + kFlagStatus, sizeof(st),
                            cudaMemcpyDeviceToHost));
  int zero[2] = {0, 0};
  C10_CUDA_CHECK(cudaMemcpy(reinterpret_cast<int*>(flags_ptr) + kFlagStatus, zero, sizeof(zero),
                            cudaMemcpyHostToDevice));
  return {st[0], st[1]};
}

int64_t peer_flag_words() { return kFlagWords; }

static unsigned long long wait_ns(int64_t timeout_ms) {
  return timeout_ms > 0 ? (unsigned long long)timeout_ms * 1000000ull : kPeerWaitNsDefault;
}

// Largest grid whose CTAs are all resident at once (the kernels' CTAs wait on
// CTA 0's barrier, so every CTA must be running).
template <typename K>
static int resident_grid(K kernel, int threads) {
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  int per_sm = 0;
  C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0));
  return sms * std::max(1, std::min(per_sm, 4));
}

void rs_adamw(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
              int64_t rank, int64_t epoch, int64_t lo, int64_t n, at::Tensor m, at::Tensor v,
              int64_t grad_is_bf16, double lr, double b1, double b2, double eps, double wd,
              double bc1, double bc2, double gscale, bool push, int64_t timeout_ms,
              c10::optional<at::Tensor> clk, c10::optional<at::Tensor> bc,
              c10::optional<at::Tensor> clip_sq, double max_norm, int64_t epoch_mul, int64_t epoch_add,
              int64_t max_ctas) {
  const int world = (int)grads.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && (int)params.size() == world &&
                  (int)flags.size() == world, "rs_adamw: one pointer per rank");
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0, "rs_adamw: shard offset/length must be multiples of 4");
  TORCH_CHECK(m.numel() >= n && v.numel() >= n, "rs_adamw: moments too small");
  const at::cuda::CUDAGuard guard(m.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t* clkp = nullptr;
  const float* bcp = nullptr;
  if (clk.has_value() && clk->defined()) {
    TORCH_CHECK(clk->scalar_type() == at::kLong && clk->numel() >= 2 && clk->is_cuda(), "rs_adamw: clk int64[2]");
    TORCH_CHECK(bc.has_value() && bc->defined() && bc->scalar_type() == at::kFloat && bc->numel() >= 2,
                "rs_adamw: bc fp32[2] with clk");
    clkp = clk->data_ptr<int64_t>();
    bcp = bc->data_ptr<float>();
  }
  const float* sqp = nullptr;
  if (clip_sq.has_value() && clip_sq->defined()) {
    TORCH_CHECK(clip_sq->is_cuda() && clip_sq->scalar_type() == at::kFloat && clip_sq->numel() >= 1,
                "rs_adamw: clip_sq fp32[1]");
    TORCH_CHECK(max_norm > 0.0, "rs_adamw: max_norm must be positive");
    sqp = clip_sq->data_ptr<float>();
  }
  // max_ctas > 0 caps the grid: a launch that runs beside other kernels (a
  // bucket synchronised during the backward) takes a few CTAs, which share SMs
  // with the compute kernels instead of filling them (CTA 0 runs the cross-rank
  // barrier and the others wait for its flag, so a partly resident grid is fine)
  int grid = grad_is_bf16 ? resident_grid(rs_adamw_kernel<__nv_bfloat16>, 256)
                          : resident_grid(rs_adamw_kernel<float>, 256);
  if (max_ctas > 0) grid = std::max(1, std::min(grid, (int)max_ctas));
  if (grad_is_bf16) {
    rs_adamw_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        table_from(grads), table_from(params), table_from(flags), (int)rank, world, (int)epoch, lo, n,
        m.data_ptr<float>(), v.data_ptr<float>(), (float)lr, (float)b1, (float)b2, (float)eps,
        (float)wd, (float)bc1, (float)bc2, (float)gscale, push ? 1 : 0, wait_ns(timeout_ms), clkp, bcp,
        sqp, (float)max_norm, (int)epoch_mul, (int)epoch_add);
  } else {
    rs_adamw_kernel<float><<<grid, 256, 0, stream>>>(
        table_from(grads), table_from(params), table_from(flags), (int)rank, world, (int)epoch, lo, n,
        m.data_ptr<float>(), v.data_ptr<float>(), (float)lr, (float)b1, (float)b2, (float)eps,
        (float)wd, (float)bc1, (float)bc2, (float)gscale, push ? 1 : 0, wait_ns(timeout_ms), clkp, bcp,
        sqp, (float)max_norm, (int)epoch_mul, (int)epoch_add);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// sq[0] += squared norm of this rank's shard of the averaged gradient (see
// rs_sumsq_kernel); sq must be zeroed by the caller.  clk: device clock epochs.
void rs_sumsq(std::vector<int64_t> grads, std::vector<int64_t> flags, int64_t rank, int64_t epoch, int64_t lo,
              int64_t n, at::Tensor sq, int64_t grad_is_bf16, double gscale, int64_t timeout_ms,
              c10::optional<at::Tensor> clk, int64_t epoch_mul, int64_t epoch_add) {
  const int world = (int)grads.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && (int)flags.size() == world, "rs_sumsq: one pointer per rank");
  TORCH_CHECK(n % 4 == 0 && lo % 4 == 0, "rs_sumsq: shard offset/length must be multiples of 4");
  TORCH_CHECK(sq.is_cuda() && sq.scalar_type() == at::kFloat && sq.numel() >= 1, "rs_sumsq: sq fp32[1]");
  const at::cuda::CUDAGuard guard(sq.device());
  const int64_t* clkp = nullptr;
  if (clk.has_value() && clk->defined()) {
    TORCH_CHECK(clk->scalar_type() == at::kLong && clk->numel() >= 2 && clk->is_cuda(), "rs_sumsq: clk int64[2]");
    clkp = clk->data_ptr<int64_t>();
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  if (grad_is_bf16) {
    const int grid = resident_grid(rs_sumsq_kernel<__nv_bfloat16>, 256);
    rs_sumsq_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        table_from(grads), table_from(flags), (int)rank, world, (int)epoch, lo, n, (float)gscale,
        sq.data_ptr<float>(), wait_ns(timeout_ms), clkp, (int)epoch_mul, (int)epoch_add);
  } else {
    const int grid = resident_grid(rs_sumsq_kernel<float>, 256);
    rs_sumsq_kernel<float><<<grid, 256, 0, stream>>>(
        table_from(grads), table_from(flags), (int)rank, world, (int)epoch, lo, n, (float)gscale,
        sq.data_ptr<float>(), wait_ns(timeout_ms), clkp, (int)epoch_mul, (int)epoch_add);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void plan_gather(std::vector<int64_t> src, std::vector<int64_t> flags, int64_t rank, int64_t epoch,
                 std::vector<int64_t> offsets, std::vector<int64_t> lengths, at::Tensor out,
                 int64_t timeout_ms) {
  const int world = (int)src.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && (int)offsets.size() == world &&
                  (int)lengths.size() == world && (int)flags.size() == world,
              "plan_gather: one entry per rank");
  int64_t total = 0;
  for (int q = 0; q < world; ++q) total = std::max(total, offsets[q] + lengths[q]);
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() * out.element_size() >= total,
              "plan_gather: output too small");
  const at::cuda::CUDAGuard guard(out.device());
  plan_gather_kernel<<<resident_grid(plan_gather_kernel, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      table_from(src), table_from(flags), (int)rank, world, (int)epoch, table_from(offsets),
      table_from(lengths), reinterpret_cast<uint8_t*>(out.data_ptr()), wait_ns(timeout_ms));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Peer NF4 shards -> bf16 operand: rows [row0, row0+rows) of the [*, cols] weight as
// [rows, cols] (or transposed [cols, rows]).
// pstarts/astarts: global start index of each rank's packed bytes / absmax values.
void plan_gather_dequant(std::vector<int64_t> psrc, std::vector<int64_t> pstarts,
                         std::vector<int64_t> asrc, std::vector<int64_t> astarts, int64_t rows,
                         int64_t cols, int64_t row0, int64_t blocksize, int64_t qtype, bool transpose,
                         at::Tensor out) {
  const int world = (int)psrc.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && (int)pstarts.size() == world &&
                  (int)asrc.size() == world && (int)astarts.size() == world,
              "plan_gather_dequant: one entry per rank");
  TORCH_CHECK(cols % 16 == 0 && (!transpose || rows % 16 == 0) && blocksize >= 16,
              "plan_gather_dequant: cols (and rows when transposing) must be multiples of 16");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == rows * cols,
              "plan_gather_dequant: bf16 output of rows*cols");
  const at::cuda::CUDAGuard guard(out.device());
  if (!transpose && cols % 32 == 0 && blocksize % 32 == 0 && rows > 0) {
    AgSource s{};
    s.world = world;
    for (int q = 0; q < kAgMaxRanks; ++q) {
      s.packed[q] = q < world ? reinterpret_cast<const uint8_t*>(psrc[q]) : nullptr;
      s.absmax[q] = q < world ? reinterpret_cast<const float*>(asrc[q]) : nullptr;
      // the last rank's piece is unbounded here (the totals are not passed)
      s.pstart[q] = q < world ? pstarts[q] : INT64_MAX;
      s.astart[q] = q < world ? astarts[q] : INT64_MAX;
    }
    s.pstart[kAgMaxRanks] = s.astart[kAgMaxRanks] = INT64_MAX;
    const int64_t items = ((rows + kAgRows - 1) / kAgRows) * ((cols + kAgCols - 1) / kAgCols);
    const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, (int64_t)sms * 8));
    ag_dequant_kernel<<<(unsigned)grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        s, (int)cols, (int)row0, (int)rows, (int)blocksize, (int)qtype,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()) - row0 * cols);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  plan_gather_dequant_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      table_from(psrc), table_from(pstarts), table_from(asrc), table_from(astarts), world, (int)rows,
      (int)cols, row0, (int)blocksize, (int)qtype, transpose ? 1 : 0,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

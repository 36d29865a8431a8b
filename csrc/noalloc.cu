// Allocation-free RMSNorm backward entry point (see noalloc.cuh for the rules).
// No counterpart in the reference.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "noalloc.cuh"

namespace zq {
// defined in elementwise.cu: per-CTA partial weight gradients into dw_part[grid][D],
// grid <= max_grid returned in *grid_out; allocates nothing
cudaError_t launch_rmsnorm_bwd(const __nv_bfloat16* gy, const __nv_bfloat16* x, const float* w,
                               const float* rstd, const __nv_bfloat16* gh, __nv_bfloat16* dx,
                               float* dw_part, int64_t M, int D, int64_t max_grid,
                               cudaStream_t stream, int64_t* grid_out);
}  // namespace zq

namespace {

constexpr long long kNoAllocScratchBytes = 4ll << 20;
constexpr int kScratchFloats = (int)(kNoAllocScratchBytes / 4);
constexpr int kMaxD = 8192;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

std::mutex g_mu;
float* g_scratch_addr[kMaxDevices] = {nullptr};
thread_local const char* g_last_error = "";

// dw[c] = sum over rows r < rows of part[r][c]
__global__ void sum_partial_rows_kernel(const float* __restrict__ part, int rows, int D,
                                        float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float s = 0.0f;
  for (int r = 0; r < rows; ++r) s += part[(int64_t)r * D + c];
  dw[c] = s;
}

int fail(cudaError_t e, const char* msg) {
  g_last_error = msg;
  return (int)e;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" const char* zq_noalloc_error_string(void) { return g_last_error; }

extern "C" int zq_rmsnorm_bwd_noalloc(const void* gy, const void* x, const float* w,
                                      const float* rstd, const void* gh, void* dx, float* dw,
                                      long long M, int D, void* stream) {
  if (M < 1 || D < 8 || D % 8 != 0)
    return fail(cudaErrorInvalidValue, "zq_rmsnorm_bwd_noalloc: need M >= 1 and D a multiple of 8");
  if (D > kMaxD)
    return fail(cudaErrorInvalidValue,
                "zq_rmsnorm_bwd_noalloc: D exceeds the maximum of 8192 supported by the 4 MiB "
                "static scratch");
  if (!gy || !x || !w || !rstd || !dx || !dw)
    return fail(cudaErrorInvalidValue, "zq_rmsnorm_bwd_noalloc: a required pointer is NULL");
  if (!aligned16(gy) || !aligned16(x) || !aligned16(dx) || (gh && !aligned16(gh)) || !aligned16(w))
    return fail(cudaErrorInvalidValue, "zq_rmsnorm_bwd_noalloc: buffers must be 16-byte aligned");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "zq_rmsnorm_bwd_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "zq_rmsnorm_bwd_noalloc: device index too large");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return fail(e, "zq_rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed");
      g_scratch_addr[dev] = static_cast<float*>(p);
    }
    scratch = g_scratch_addr[dev];
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fail(e, "zq_rmsnorm_bwd_noalloc: cudaDeviceGetAttribute failed");
  long long max_grid = 2ll * sms;
  const long long cap = kScratchFloats / D;  // partial rows that fit in the scratch
  if (max_grid > cap) max_grid = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t grid = 0;
  e = zq::launch_rmsnorm_bwd(
      static_cast<const __nv_bfloat16*>(gy), static_cast<const __nv_bfloat16*>(x), w, rstd,
      static_cast<const __nv_bfloat16*>(gh), static_cast<__nv_bfloat16*>(dx), scratch, (int64_t)M, D,
      max_grid, s, &grid);
  if (e != cudaSuccess) return fail(e, "zq_rmsnorm_bwd_noalloc: kernel launch failed");
  sum_partial_rows_kernel<<<(unsigned)((D + 255) / 256), 256, 0, s>>>(scratch, (int)grid, D, dw);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(e, "zq_rmsnorm_bwd_noalloc: kernel launch failed");
  g_last_error = "";
  return 0;
}

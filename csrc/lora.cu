// LoRA support for the NF4 linear layer:
//  * lora_pack: the padded, pre-scaled bf16 operands that ride as the extra
//    64-wide K slab of the tcgen05 GEMM, plus the transposed B that the
//    rank-space product V = dY·B reads (one launch per module per optimizer
//    step, rows/columns past the rank stay zero); the LoRA products themselves
//    are the tcgen05 kernels of lora_sm100.cu;
//  * matmul_accum_f32: C (fp32) = beta * C + alpha * A @ B for bf16 A, B - a
//    plain library GEMM (cuBLAS, bf16 inputs, fp32 accumulate and output) kept
//    for the full-size weight gradient of train-from-scratch layers.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cublas_v2.h>

#include "common.cuh"

namespace zq {

// a_pad[i, k] = s * A[i, k] for i < r; b_pad[n, j] = B[n, j] for j < r; and,
// when b_t is given, b_t[j, n] = B[n, j] (the K-major operand of V = dY·B),
// each output written in its own index order so every store is coalesced.
__global__ void lora_pack_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                 __nv_bfloat16* __restrict__ a_pad, int64_t a_ld,
                                 __nv_bfloat16* __restrict__ b_pad, int64_t b_ld,
                                 __nv_bfloat16* __restrict__ b_t, int64_t t_ld, int r, int64_t K,
                                 int64_t N, float s) {
  const int64_t na = (int64_t)r * K, nb = N * r, nt = b_t != nullptr ? N * r : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb + nt;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < na) {
      const int64_t row = i / K, col = i % K;
      a_pad[row * a_ld + col] = __float2bfloat16_rn(s * A[i]);
    } else if (i < na + nb) {
      const int64_t j = i - na, row = j / r, col = j % r;
      b_pad[row * b_ld + col] = __float2bfloat16_rn(B[j]);
    } else {
      const int64_t j = i - na - nb, row = j / N, col = j % N;  // b_t[row, col] = B[col, row]
      b_t[row * t_ld + col] = __float2bfloat16_rn(B[col * r + row]);
    }
  }
}

// Many lora_pack jobs in one launch: job j = blockIdx.y reads its row of `table`
// (kPackFields int64 words: A, B, a_pad, a_ld, b_pad, b_ld, b_t, t_ld, r, K, N,
// scaling as fp32 bits; b_t may be 0) and runs the same element loop.
constexpr int kPackFields = 12;

__global__ void lora_pack_many_kernel(const int64_t* __restrict__ table) {
  const int64_t* e = table + (int64_t)blockIdx.y * kPackFields;
  const float* A = reinterpret_cast<const float*>(e[0]);
  const float* B = reinterpret_cast<const float*>(e[1]);
  __nv_bfloat16* a_pad = reinterpret_cast<__nv_bfloat16*>(e[2]);
  __nv_bfloat16* b_pad = reinterpret_cast<__nv_bfloat16*>(e[4]);
  __nv_bfloat16* b_t = reinterpret_cast<__nv_bfloat16*>(e[6]);
  const int64_t a_ld = e[3], b_ld = e[5], t_ld = e[7], K = e[9], N = e[10];
  const int r = (int)e[8];
  const float s = __int_as_float((int)e[11]);
  const int64_t na = (int64_t)r * K, nb = N * r, nt = b_t != nullptr ? N * r : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb + nt;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i < na) {
      const int64_t row = i / K, col = i % K;
      a_pad[row * a_ld + col] = __float2bfloat16_rn(s * A[i]);
    } else if (i < na + nb) {
      const int64_t j = i - na, row = j / r, col = j % r;
      b_pad[row * b_ld + col] = __float2bfloat16_rn(B[j]);
    } else {
      const int64_t j = i - na - nb, row = j / N, col = j % N;
      b_t[row * t_ld + col] = __float2bfloat16_rn(B[col * r + row]);
    }
  }
}

}  // namespace zq

using namespace zq;

// table: int64 CUDA tensor [jobs, 12] (see lora_pack_many_kernel); max_elems: the
// largest job's element count (sizes the grid).  The caller validated every job
// the way lora_pack does.
void lora_pack_many(at::Tensor table, int64_t max_elems) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kLong && table.is_contiguous() &&
                  table.dim() == 2 && table.size(1) == kPackFields,
              "lora_pack_many: table must be a contiguous int64 CUDA tensor [jobs, 12]");
  const int64_t jobs = table.size(0);
  if (jobs == 0 || max_elems <= 0) return;
  TORCH_CHECK(jobs <= 65535, "lora_pack_many: at most 65535 jobs");
  const at::cuda::CUDAGuard guard(table.device());
  const int64_t bx = std::min<int64_t>((max_elems + 255) / 256, 16);
  lora_pack_many_kernel<<<dim3((unsigned)bx, (unsigned)jobs), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      table.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lora_pack(at::Tensor A, at::Tensor B, double scaling, at::Tensor a_pad, at::Tensor b_pad,
               c10::optional<at::Tensor> b_t) {
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kFloat && A.is_contiguous() && A.dim() == 2,
              "lora_pack: A must be contiguous fp32 [r, K]");
  TORCH_CHECK(B.is_cuda() && B.scalar_type() == at::kFloat && B.is_contiguous() && B.dim() == 2,
              "lora_pack: B must be contiguous fp32 [N, r]");
  const int64_t r = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == r, "lora_pack: rank mismatch");
  TORCH_CHECK(a_pad.scalar_type() == at::kBFloat16 && a_pad.dim() == 2 && a_pad.size(0) >= r &&
                  a_pad.size(1) == K && a_pad.stride(1) == 1,
              "lora_pack: a_pad must be bf16 [>= r, K] with unit column stride");
  TORCH_CHECK(b_pad.scalar_type() == at::kBFloat16 && b_pad.dim() == 2 && b_pad.size(0) == N &&
                  b_pad.size(1) >= r && b_pad.stride(1) == 1,
              "lora_pack: b_pad must be bf16 [N, >= r] with unit column stride");
  __nv_bfloat16* btp = nullptr;
  int64_t t_ld = 0;
  if (b_t.has_value() && b_t->defined()) {
    TORCH_CHECK(b_t->scalar_type() == at::kBFloat16 && b_t->dim() == 2 && b_t->size(0) >= r &&
                    b_t->size(1) == N && b_t->stride(1) == 1,
                "lora_pack: b_t must be bf16 [>= r, N] with unit column stride");
    btp = reinterpret_cast<__nv_bfloat16*>(b_t->data_ptr());
    t_ld = b_t->stride(0);
  }
  const at::cuda::CUDAGuard guard(A.device());
  const int64_t total = r * K + N * r + (btp != nullptr ? N * r : 0);
  if (total == 0) return;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
  lora_pack_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      A.data_ptr<float>(), B.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(a_pad.data_ptr()), a_pad.stride(0),
      reinterpret_cast<__nv_bfloat16*>(b_pad.data_ptr()), b_pad.stride(0), btp, t_ld, (int)r, K, N,
      (float)scaling);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Operand of a row-major product as cuBLAS (column-major) sees it: a matrix
// whose last dimension is contiguous is "row-major" with leading dimension
// stride(0); one whose first dimension is contiguous is "column-major" with
// leading dimension stride(1).
static bool row_major(const at::Tensor& t, int64_t* ld) {
  if (t.stride(1) == 1 && t.stride(0) >= std::max<int64_t>(1, t.size(1))) {
    *ld = t.stride(0);
    return true;
  }
  TORCH_CHECK(t.stride(0) == 1 && t.stride(1) >= std::max<int64_t>(1, t.size(0)),
              "matmul_accum_f32: operands must have one unit stride");
  *ld = t.stride(1);
  return false;
}

// C[m, n] (fp32, row-major contiguous) = beta * C + alpha * A[m, k] @ B[k, n].
void matmul_accum_f32(at::Tensor A, at::Tensor B, at::Tensor C, double alpha, double beta) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "matmul_accum_f32: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "matmul_accum_f32: A and B must be bf16");
  TORCH_CHECK(C.scalar_type() == at::kFloat && C.is_contiguous(), "matmul_accum_f32: C fp32 contiguous");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "matmul_accum_f32: 2-D operands");
  const int64_t m = A.size(0), k = A.size(1), n = B.size(1);
  TORCH_CHECK(B.size(0) == k && C.size(0) == m && C.size(1) == n, "matmul_accum_f32: shapes");
  if (m == 0 || n == 0) return;
  const at::cuda::CUDAGuard guard(C.device());
  if (k == 0) {
    C.mul_(beta);
    return;
  }
  int64_t lda = 0, ldb = 0;
  const bool a_rm = row_major(A, &lda);
  const bool b_rm = row_major(B, &ldb);
  // row-major C = column-major C^T [n, m] = B^T [n, k] @ A^T [k, m]
  const cublasOperation_t opB = b_rm ? CUBLAS_OP_N : CUBLAS_OP_T;
  const cublasOperation_t opA = a_rm ? CUBLAS_OP_N : CUBLAS_OP_T;
  const float al = (float)alpha, be = (float)beta;
  cublasHandle_t h = at::cuda::getCurrentCUDABlasHandle();
  TORCH_CHECK(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "matmul_accum_f32: size");
  const cublasStatus_t st = cublasGemmEx(
      h, opB, opA, (int)n, (int)m, (int)k, &al, B.data_ptr(), CUDA_R_16BF, (int)ldb, A.data_ptr(),
      CUDA_R_16BF, (int)lda, &be, C.data_ptr(), CUDA_R_32F, (int)n, CUBLAS_COMPUTE_32F,
      CUBLAS_GEMM_DEFAULT);
  TORCH_CHECK(st == CUBLAS_STATUS_SUCCESS, "matmul_accum_f32: cublasGemmEx failed with status ",
              (int)st);
}

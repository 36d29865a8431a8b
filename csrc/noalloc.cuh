// No counterpart in the reference.
//
// An allocation-free entry point for the RMSNorm backward pass, for callers that
// cannot allocate device memory themselves: code that runs while another
// component owns every byte of the device (a fixed-pool serving runtime, a
// framework with its own allocator that forbids cudaMalloc behind its back),
// or code that must not trigger the implicit device synchronisation that
// cudaMalloc/cudaFree can cause in the middle of a pipelined step.
//
// The backward pass needs scratch memory for per-block partial sums of the
// weight gradient.  Here that scratch is a file-scope __device__ array of
// kNoAllocScratchBytes (4 MiB) that every GPU loading this library keeps until
// the process exits.  The caller passes every input and output buffer; the
// entry point itself calls no cudaMalloc, cudaFree or allocating library
// routine.
//
// Calling rules:
//  * The first call on a device looks up the device address of the scratch
//    array (cudaGetSymbolAddress) with that device current; make that first
//    call before any stream capture on the device.
//  * All calls on a device share the one scratch array and it keeps whatever
//    the previous call left there.  Calls whose executions overlap on the GPU
//    (different streams without ordering between them) race on it and give
//    wrong results; order them on one stream or with events.
//  * D must be a multiple of 8 and at most 8192; M >= 1.  Larger problems are
//    rejected with cudaErrorInvalidValue and a message from
//    zq_noalloc_error_string().
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// dx[M,D] (bf16) and dw[D] (fp32, overwritten) from gy[M,D], x[M,D] (bf16),
// w[D] and rstd[M] (fp32), plus an optional residual gradient gh[M,D] (bf16,
// may be NULL) that is added to dx.  Pointers to bf16 data and w must be
// 16-byte aligned.  `stream` is a cudaStream_t (NULL = legacy default stream).
// Returns 0 on success or a cudaError_t code.
int zq_rmsnorm_bwd_noalloc(const void* gy, const void* x, const float* w, const float* rstd,
                           const void* gh, void* dx, float* dw, long long M, int D, void* stream);

// Human-readable reason for the last non-zero return of this thread's call.
const char* zq_noalloc_error_string(void);

#ifdef __cplusplus
}
#endif

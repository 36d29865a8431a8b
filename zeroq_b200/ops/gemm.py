"""Dense bf16 GEMMs on tcgen05 (``csrc/gemm_sm100.cu``).

``gemm_bt``: ``C[M,N] = A[M,K] · B[N,K]ᵀ``, both operands K-major.
``gemm_nn``: ``C[M,N] = A[M,K] · B[K,N]``, ``B`` read MN-major by the tensor
core straight from its row-major layout (no transposed copy).

Operands are staged by TMA into 128-byte-swizzled shared memory; the
accumulator lives in TMEM.  Requirements: bf16, contiguous, ``K % 64 == 0``,
``N % 8 == 0`` (``gemm_nn``: ``N % 64 == 0`` and ``M >= 256``).  Anything else,
and all CPU tensors, uses ``torch.matmul``.
"""

from __future__ import annotations

import torch

from . import _ext


def gemm_ok(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
            and a.dim() == 2 and b.dim() == 2 and a.shape[1] == b.shape[1]
            and a.shape[1] % 64 == 0 and b.shape[0] % 8 == 0 and a.is_contiguous()
            and b.is_contiguous())


def gemm_bt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """``a @ b.T`` with ``a [M,K]``, ``b [N,K]``."""
    if gemm_ok(a, b):
        M, N = a.shape[0], b.shape[0]
        if out is None:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
        _ext.ext().gemm_bf16_tn(a, b, out)
        return out
    r = a @ b.t()
    if out is not None:
        out.copy_(r)
        return out
    return r


def gemm_nn_ok(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
            and a.dim() == 2 and b.dim() == 2 and a.shape[1] == b.shape[0]
            and a.shape[0] >= 256 and a.shape[1] % 64 == 0 and b.shape[1] % 64 == 0
            and a.is_contiguous() and b.is_contiguous())


def gemm_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """``a @ b`` with ``a [M,K]``, ``b [K,N]`` (both row-major)."""
    if gemm_nn_ok(a, b):
        if out is None:
            out = torch.empty(a.shape[0], b.shape[1], dtype=torch.bfloat16, device=a.device)
        _ext.ext().gemm_bf16_nn(a, b, out, None, None)
        return out
    r = a @ b
    if out is not None:
        out.copy_(r)
        return out
    return r


class LMHeadFunction(torch.autograd.Function):
    """``logits = h · Eᵀ`` for a (frozen or trainable) embedding matrix ``E [V, d]``.

    The input gradient ``dh = dlogits · E`` reads ``E`` MN-major in place, so no
    transposed copy of the head matrix is kept.
    """

    @staticmethod
    def forward(ctx, h, E):
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        logits = gemm_bt(h2, E)
        ctx.save_for_backward(h2, E)
        ctx.hshape = h.shape
        return logits

    @staticmethod
    def backward(ctx, g):
        h2, E = ctx.saved_tensors
        g = g.contiguous()
        dh = gemm_nn(g, E.detach().to(g.dtype) if E.dtype != g.dtype else E.detach())
        dE = None
        if ctx.needs_input_grad[1]:
            dE = (g.t() @ h2).to(E.dtype)
        return dh.view(ctx.hshape), dE

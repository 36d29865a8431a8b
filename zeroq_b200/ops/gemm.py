"""Dense bf16 GEMM ``C[M,N] = A[M,K] · B[N,K]ᵀ`` on tcgen05 (``csrc/gemm_sm100.cu``).

Both operands are K-major (row-major ``A`` and row-major ``B`` with K
contiguous) and staged by TMA into 128-byte-swizzled shared memory; the
accumulator lives in TMEM.  Requirements: bf16, contiguous, ``K % 64 == 0``,
``N % 8 == 0`` (16-byte row pitch for the TMA store).  Anything else, and all
CPU tensors, uses ``torch.matmul``.
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


class LMHeadFunction(torch.autograd.Function):
    """``logits = h · Eᵀ`` for a (frozen or trainable) embedding matrix ``E [V, d]``.

    ``Et`` is a cached ``Eᵀ`` (``[d, V]``, contiguous) so the input gradient
    ``dh = dlogits · E`` is also a K-major GEMM; it is refreshed by the model
    when ``E`` changes.
    """

    @staticmethod
    def forward(ctx, h, E, Et):
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        logits = gemm_bt(h2, E)
        ctx.save_for_backward(h2, E, Et)
        ctx.hshape = h.shape
        return logits

    @staticmethod
    def backward(ctx, g):
        h2, E, Et = ctx.saved_tensors
        g = g.contiguous()
        dh = gemm_bt(g, Et) if Et is not None else g @ E
        dE = None
        if ctx.needs_input_grad[1]:
            dE = (g.t() @ h2).to(E.dtype)
        return dh.view(ctx.hshape), dE, None

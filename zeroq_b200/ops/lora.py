"""Rank-space products of LoRA adapters (``csrc/lora_sm100.cu``).

For a projection ``y = x Wᵀ + s (x Aᵀ) Bᵀ`` training needs four skinny products
per step, each reading one activation-sized operand once:

* ``U = x·(sA)ᵀ`` (forward) and ``V = dY·B`` (backward) - :func:`down`;
* ``dA += s·Vᵀ·x`` and ``dB += dYᵀ·U`` - :func:`wgrad`, accumulated in fp32
  straight into the gradient buffers.

The reference computes them with PEFT's ``nn.Linear`` adapters on cuBLAS
(``examples/train_32b_maxwell.py:345-354``).  On CUDA tensors these are the
tcgen05 kernels of ``csrc/lora_sm100.cu``; CPU tensors take the fp32 PyTorch
oracle below.

Rank-space layouts: ``down`` returns ``U [T, upad]`` row-major with the columns
past ``nq`` zero (the 64-wide extra K slab the main GEMM multiplies against the
padded ``B``) and ``Ut [nq, T]`` (the K-major operand ``wgrad`` reads).  Several
adapters that share an input (the fused q/k/v projection) pack their ranks side
by side, ``g`` columns each.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import _ext


def round16(r: int) -> int:
    return (r + 15) // 16 * 16


def down(p: torch.Tensor, w: torch.Tensor, upad: int = 64, transposed: bool = True
         ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """``U = P·Wᵀ`` as ``[T, upad]`` bf16 (columns past ``W.shape[0]`` zero) and,
    with ``transposed``, ``Ut = Uᵀ`` as ``[nq, T']`` (T' = T rounded up to 8)."""
    T = p.shape[0]
    nq = w.shape[0]
    if p.is_cuda:
        u = torch.empty(T, upad, dtype=torch.bfloat16, device=p.device)
        ut = None
        if transposed:
            ut = torch.empty(nq, (T + 7) // 8 * 8, dtype=torch.bfloat16, device=p.device)
        _ext.ext().lora_down(p, w, u, ut)
        return u, ut
    prod = (p.float() @ w.float().t()).to(torch.bfloat16)
    u = torch.zeros(T, upad, dtype=torch.bfloat16)
    u[:, :nq] = prod
    return u, (prod.t().contiguous() if transposed else None)


def wgrad(p: torch.Tensor, qt: torch.Tensor, nq: int,
          jobs: Sequence[Tuple[int, int, int, float]], outs: List[torch.Tensor], gsz: int,
          rvalid: int, transposed: bool) -> None:
    """For each job ``(i_begin, i_count, q_row, alpha)`` and group ``g`` of ``gsz``
    rank columns (``outs`` job-major, ``nq // gsz`` per job):

    * ``transposed``: ``out[jj, i] += alpha · Σ_t P[t, i_begin+i] · Qt[q_row+g·gsz+jj, t]``
      (an ``A`` gradient ``[r, in]``);
    * else ``out[i, jj] += ...`` (a ``B`` gradient ``[out, r]``),

    for ``i < i_count`` and ``jj < rvalid``.
    """
    if p.is_cuda:
        _ext.ext().lora_wgrad(p, qt, nq, [j[0] for j in jobs], [j[1] for j in jobs],
                              [j[2] for j in jobs], [float(j[3]) for j in jobs], list(outs),
                              gsz, rvalid, transposed)
        return
    T = p.shape[0]
    ng = nq // gsz
    pf = p.float()
    qf = qt[:, :T].float()
    for b, (i0, ni, q0, alpha) in enumerate(jobs):
        for g in range(ng):
            o = outs[b * ng + g]
            rows = qf[q0 + g * gsz: q0 + g * gsz + rvalid]           # [rvalid, T]
            prod = alpha * (rows @ pf[:, i0:i0 + ni])                  # [rvalid, ni]
            if transposed:
                o[:rvalid, :ni] += prod
            else:
                o[:ni, :rvalid] += prod.t()


def vdb(g: torch.Tensor, bt: torch.Tensor, ut: torch.Tensor, upad: int,
        segs: Sequence[Tuple[int, int, int]], outs: List[torch.Tensor], nqb: int, rvalid: int
        ) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """The backward's two products over ``dY`` (``g [T, N]``) in one pass:
    ``V = dY·Btᵀ`` returned as ``(V [T, upad], Vt)`` like :func:`down`, and for each
    segment ``(n_begin, n_count, q_row)`` of ``dY``'s columns
    ``out[n, jj] += Σ_t dY[t, n_begin+n] · Ut[q_row+jj, t]`` (``jj < rvalid``).
    Returns None when the shape does not fit the fused kernel (CUDA only); the
    caller then uses :func:`down` and :func:`wgrad`."""
    T = g.shape[0]
    nqv = bt.shape[0]
    if g.is_cuda:
        v = torch.empty(T, upad, dtype=torch.bfloat16, device=g.device)
        vt = torch.empty(nqv, (T + 7) // 8 * 8, dtype=torch.bfloat16, device=g.device)
        ok = _ext.ext().lora_vdb(g, bt, ut, v, vt, nqb, [s[0] for s in segs],
                                 [s[1] for s in segs], [s[2] for s in segs], list(outs), rvalid)
        return (v, vt) if ok else None
    v, vt = down(g, bt, upad)
    wgrad(g, ut, nqb, [(s[0], s[1], s[2], 1.0) for s in segs], outs, nqb, rvalid, False)
    return v, vt

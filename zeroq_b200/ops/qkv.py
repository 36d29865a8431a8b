"""Fused q/k/v projection of an attention block (NF4 weights, optional LoRA).

The three frozen NF4 weights are decoded into one bf16 operand ``[Nq+Nk+Nv, d]``
and multiplied in ONE tcgen05 GEMM (one wave-quantised grid instead of three).
The three LoRA up-projections ride in the same MMA chain as three 64-wide extra
K slabs: ``U = x·[sA_q; sA_k; sA_v]ᵀ`` (one skinny GEMM reading ``x`` once)
against a block-diagonal ``[B_q, B_k, B_v]``.  The GEMM epilogue applies the
rotary embedding to the q and k columns (``csrc/gemm_sm100.cu`` ``kEpiRope``).
q, k and v are returned as column slices of the one output, which the tcgen05
attention reads through strided TMA maps.

Backward: dQ and dK are rotated back straight into the column slices of one
``[M, Nq+Nk+Nv]`` gradient and dV is copied into the third, so the input
gradient is one MN-major GEMM (no residual-gradient adds) with the LoRA term
``V·[sA]`` folded in the same way (``V = dY·B_blk``, one skinny GEMM), and the
three ``dA`` products are one skinny GEMM.  The reference runs three separate
projections (``transformers`` q_proj/k_proj/v_proj modules around
``bnb.matmul_4bit``, see ``src/hetero/zeroq_hetero.py:477-500``).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _ext
from .nf4 import QUANT_TYPE_ID


def _decode_into(mods, w: torch.Tensor):
    E = _ext.ext()
    off = 0
    for m in mods:
        n, d = m.out_features, m.in_features
        E.nf4_to_bf16(m.weight_packed, m.weight_absmax, w[off:off + n].view(-1), n, d,
                      m.blocksize, QUANT_TYPE_ID[m.quant_type], False)
        off += n


def _lora_blocks(mods, cache: dict):
    """``A_cat [64·3, d]`` (the modules' cached scaled, padded A operands stacked)
    and the block-diagonal ``B_blk [Nq+Nk+Nv, 64·3]``, rebuilt only when a
    module's LoRA operands change."""
    ops = [m._lora_operands() for m in mods]
    key = tuple(m._lora_key for m in mods)
    if cache.get("key") != key:
        Nt = sum(m.out_features for m in mods)
        A_cat = torch.cat([o[0] for o in ops], 0)
        B_blk = torch.zeros(Nt, 64 * len(mods), dtype=torch.bfloat16, device=A_cat.device)
        off = 0
        for i, (m, o) in enumerate(zip(mods, ops)):
            B_blk[off:off + m.out_features, 64 * i:64 * (i + 1)] = o[1]
            off += m.out_features
        cache.update(key=key, A_cat=A_cat, B_blk=B_blk)
    return cache["A_cat"], cache["B_blk"]


def _direct(p) -> bool:
    return (p is not None and getattr(p, "_zq_flat_grad", False) and p.grad is not None
            and p.grad.dtype == torch.float32 and p.grad.is_contiguous())


class QKVFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, qA, qB, kA, kB, vA, vB, mods, cs, cache):
        d = mods[0].in_features
        Ns = [m.out_features for m in mods]
        Nt = sum(Ns)
        x2 = x.reshape(-1, d)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M = x2.shape[0]
        E = _ext.ext()
        w = torch.empty(Nt, d, dtype=torch.bfloat16, device=x2.device)
        _decode_into(mods, w)
        lora = mods[0].lora_r > 0
        U = A_cat = B_blk = None
        if lora:
            A_cat, B_blk = _lora_blocks(mods, cache)
            U = x2 @ A_cat.t()                      # [M, 192]: x read once for all three
        y = torch.empty(M, Nt, dtype=torch.bfloat16, device=x2.device)
        E.gemm_rope(x2, w, y, cs, U, B_blk, Ns[0] + Ns[1])
        del w
        ctx.save_for_backward(x2 if lora else None, U, A_cat, B_blk)
        ctx.mods, ctx.cs, ctx.meta = mods, cs, (x.shape, Ns, lora)
        S = cs.shape[0]
        B = M // S
        o1, o2 = Ns[0], Ns[0] + Ns[1]
        q = y[:, :o1].view(B, S, Ns[0] // 128, 128)
        k = y[:, o1:o2].view(B, S, Ns[1] // 128, 128)
        v = y[:, o2:].view(B, S, Ns[2] // 128, 128)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x2, U, A_cat, B_blk = ctx.saved_tensors
        shp, Ns, lora = ctx.meta
        mods, cs = ctx.mods, ctx.cs
        E = _ext.ext()
        Nt = sum(Ns)
        o1, o2 = Ns[0], Ns[0] + Ns[1]
        ref = dq if dq is not None else (dk if dk is not None else dv)
        M = ref.shape[0] * ref.shape[1]
        dev = ref.device
        g = torch.empty(M, Nt, dtype=torch.bfloat16, device=dev)
        for grad, lo, hi, rot in ((dq, 0, o1, True), (dk, o1, o2, True), (dv, o2, Nt, False)):
            if grad is None:
                g[:, lo:hi].zero_()
            elif rot:   # gradient of the pre-rotation columns, straight into its slice
                E.rope_into(grad.contiguous(), g[:, lo:hi], cs, -1.0)
            else:
                g[:, lo:hi].copy_(grad.reshape(M, hi - lo))
        d = mods[0].in_features
        gx = None
        V = None
        if lora:
            V = g @ B_blk                          # [M, 192], unscaled dY·B per projection
        if ctx.needs_input_grad[0]:
            w = torch.empty(Nt, d, dtype=torch.bfloat16, device=dev)
            _decode_into(mods, w)
            gx = torch.empty(M, d, dtype=torch.bfloat16, device=dev)
            E.gemm_bf16_nn(g, w, gx, V, A_cat)     # dX = dY·W + V·[sA] in one GEMM
            del w
            gx = gx.view(*shp[:-1], d)
        grads = [None] * 6
        if lora:
            dA_cat = torch.empty(A_cat.shape[0], d, dtype=torch.float32, device=dev)
            E.matmul_accum_f32(V.t(), x2, dA_cat, 1.0, 0.0)   # all three dA in one product
            off = 0
            for i, m in enumerate(mods):
                r = m.lora_r
                A, Bm = m.lora_A, m.lora_B
                if ctx.needs_input_grad[1 + 2 * i]:
                    gA = dA_cat[64 * i:64 * i + r] * m.scaling
                    if _direct(A):
                        A.grad.add_(gA)
                    else:
                        grads[2 * i] = gA.to(A.dtype)
                if ctx.needs_input_grad[2 + 2 * i]:
                    gy_i = g[:, off:off + m.out_features]
                    if _direct(Bm):
                        E.matmul_accum_f32(gy_i.t(), U[:, 64 * i:64 * i + r], Bm.grad, 1.0, 1.0)
                    else:
                        gB = torch.empty(m.out_features, r, dtype=torch.float32, device=dev)
                        E.matmul_accum_f32(gy_i.t(), U[:, 64 * i:64 * i + r], gB, 1.0, 0.0)
                        grads[2 * i + 1] = gB.to(Bm.dtype)
                off += m.out_features
        return (gx, *grads, None, None, None)


def qkv_fusable(mods: Sequence, x: torch.Tensor, S: int) -> bool:
    """The fused path applies: resident NF4 (no bias, no peer or master source),
    128-wide heads, equal input width, LoRA on all three (rank <= 64) or on none,
    a CUDA bf16 input of at least 256 rows, and a fused backend."""
    from .qlinear import IN_KERNEL_DECODE

    if IN_KERNEL_DECODE or not (x.is_cuda and x.dtype == torch.bfloat16):
        return False
    d = mods[0].in_features
    M = x.numel() // d if x.numel() else 0
    if M < 256 or d % 128 or M % S:
        return False
    ranks = {m.lora_r for m in mods}
    if len(ranks) != 1 or next(iter(ranks)) > 64:
        return False
    for m in mods:
        if (m.weight_packed is None or m.bias is not None or m.in_features != d
                or m.out_features % 128 or m.backend == "torch" or m.blocksize % 64
                or getattr(m, "_peer", None) is not None or getattr(m, "_master", None) is not None):
            return False
    return True


def qkv_projection(x: torch.Tensor, mods: Sequence, cs: torch.Tensor, cache: Optional[dict] = None):
    """``(q, k, v)`` of ``x [B, S, d]`` with q and k rotary-embedded by ``cs``,
    each ``[B, S, H, 128]`` (column slices of one fused output)."""
    q_, k_, v_ = mods
    cache = cache if cache is not None else {}
    return QKVFunction.apply(x, q_.lora_A, q_.lora_B, k_.lora_A, k_.lora_B, v_.lora_A, v_.lora_B,
                             tuple(mods), cs, cache)

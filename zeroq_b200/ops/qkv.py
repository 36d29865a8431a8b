"""Fused q/k/v projection of an attention block (NF4 weights, optional LoRA).

The three frozen NF4 weights are decoded into one bf16 operand ``[Nq+Nk+Nv, d]``
and multiplied in ONE tcgen05 GEMM (one wave-quantised grid instead of three).
The three LoRA up-projections ride in the same MMA chain as extra K slabs:
``U = x·[sA_q; sA_k; sA_v]ᵀ`` (one rank-space kernel reading ``x`` once, from
``csrc/lora_sm100.cu``) against a block-diagonal ``[B_q, B_k, B_v]``.  With
ranks up to 21 the three adapters pack side by side into ONE 64-wide slab
(columns ``[g·i, g·i + r)`` of adapter ``i``, ``g`` = rank rounded up to 16);
larger ranks take one 64-wide slab each.  The GEMM epilogue applies the
rotary embedding to the q and k columns (``csrc/gemm_sm100.cu`` ``kEpiRope``).
q, k and v are returned as column slices of the one output, which the tcgen05
attention reads through strided TMA maps.

Backward: dQ and dK are rotated back straight into the column slices of one
``[M, Nq+Nk+Nv]`` gradient and dV is copied into the third, so the input
gradient is one MN-major GEMM (no residual-gradient adds) with the LoRA term
``V·[sA]`` folded in the same way (``V = dY·B_blk``, one rank-space kernel), the
three ``dA`` products are one pass over ``x`` and the three ``dB`` one launch.  The reference runs three separate
projections (``transformers`` q_proj/k_proj/v_proj modules around
``bnb.matmul_4bit``, see ``src/hetero/zeroq_hetero.py:477-500``).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _ext
from . import lora as lora_k
from .nf4 import QUANT_TYPE_ID
from .qlinear import KEEP_OPERANDS


def _decode_into(mods, w: torch.Tensor):
    """The modules' 4-bit weights, one after the other, into ``w`` (one launch when
    they share block size and code)."""
    E = _ext.ext()
    if (len({m.blocksize for m in mods}) == 1 and len({m.quant_type for m in mods}) == 1
            and len(mods) <= 4 and w.is_contiguous()):
        E.nf4_to_bf16_segments([m.weight_packed for m in mods], [m.weight_absmax for m in mods],
                               [m.out_features * m.in_features for m in mods], w,
                               mods[0].blocksize, QUANT_TYPE_ID[mods[0].quant_type])
        return
    off = 0
    for m in mods:
        n, d = m.out_features, m.in_features
        E.nf4_to_bf16(m.weight_packed, m.weight_absmax, w[off:off + n].view(-1), n, d,
                      m.blocksize, QUANT_TYPE_ID[m.quant_type], False)
        off += n


def _lora_blocks(mods, cache: dict):
    """``(g, A_cat [W, d], B_blk [Nq+Nk+Nv, W], B_catT [3g, Nq+Nk+Nv])`` with ``g`` the
    per-adapter column stride in rank space and ``W`` the slab width (64 when the
    three ranks pack into one slab, else 3 x 64).  The three buffers persist (their
    padding stays zero); when an adapter changes (every optimizer step) each one
    is packed straight into its slices from the fp32 parameters - one pack kernel
    per adapter, no per-step allocation or slice copies."""
    key = lora_blocks_key(mods)
    if cache.get("key") != key:
        r = mods[0].lora_r
        g = lora_k.round16(r)
        if 3 * g > 64:
            g = 64
        W = 64 if 3 * g <= 64 else 3 * 64
        Nt = sum(m.out_features for m in mods)
        d = mods[0].in_features
        dev = mods[0].lora_A.device
        if cache.get("shape") != (g, W, Nt, d, r, dev):
            cache.update(shape=(g, W, Nt, d, r, dev),
                         A_cat=torch.zeros(W, d, dtype=torch.bfloat16, device=dev),
                         B_blk=torch.zeros(Nt, W, dtype=torch.bfloat16, device=dev),
                         B_catT=torch.zeros(3 * g, Nt, dtype=torch.bfloat16, device=dev))
        cache["g"] = g
        with torch.no_grad():
            for m, a_v, b_v, t_v in lora_block_views(mods, cache):
                A, B = m.lora_A.detach(), m.lora_B.detach()
                if A.is_cuda and A.dtype == torch.float32 and B.dtype == torch.float32:
                    _ext.ext().lora_pack(A.contiguous(), B.contiguous(), float(m.scaling), a_v, b_v, t_v)
                else:
                    a_v.copy_(A.float() * m.scaling)
                    b_v.copy_(B)
                    t_v.copy_(B.t())
        cache.update(key=key, g=g)
    return cache["g"], cache["A_cat"], cache["B_blk"], cache["B_catT"]


def lora_blocks_key(mods):
    """What the cached q/k/v block operands were packed from."""
    return tuple((m.lora_A._version, m.lora_B._version, m.lora_A.data_ptr(), m.lora_B.data_ptr(),
                  float(m.scaling)) for m in mods)


def lora_block_views(mods, cache: dict):
    """``(module, s·A slice, B slice, Bᵀ slice)`` of each adapter inside the cached
    block buffers (their layout is fixed by ``_lora_blocks``)."""
    g, r = cache["g"], mods[0].lora_r
    A_cat, B_blk, B_catT = cache["A_cat"], cache["B_blk"], cache["B_catT"]
    out, off = [], 0
    for i, m in enumerate(mods):
        n = m.out_features
        out.append((m, A_cat[g * i:g * i + r], B_blk[off:off + n, g * i:g * i + r],
                    B_catT[g * i:g * i + r, off:off + n]))
        off += n
    return out


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
        U = Ut = A_cat = B_blk = B_catT = None
        g = 0
        if lora:
            g, A_cat, B_blk, B_catT = _lora_blocks(mods, cache)
            # x read once for all three adapters: U [M, slab width] and Ut [3g, M]
            U, Ut = lora_k.down(x2, A_cat[:3 * g], upad=A_cat.shape[0])
        y = torch.empty(M, Nt, dtype=torch.bfloat16, device=x2.device)
        E.gemm_rope(x2, w, y, cs, U, B_blk, Ns[0] + Ns[1])
        # the input-gradient GEMM reads the same operand (see qlinear.KEEP_OPERANDS)
        ctx.w_kept = w if (KEEP_OPERANDS and ctx.needs_input_grad[0]) else None
        del w, U
        ctx.save_for_backward(x2 if lora else None, Ut, A_cat, B_blk, B_catT)
        ctx.g = g
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
        x2, Ut, A_cat, B_blk, B_catT = ctx.saved_tensors
        gw = ctx.g
        shp, Ns, lora = ctx.meta
        mods, cs = ctx.mods, ctx.cs
        E = _ext.ext()
        Nt = sum(Ns)
        o1, o2 = Ns[0], Ns[0] + Ns[1]
        ref = dq if dq is not None else (dk if dk is not None else dv)
        M = ref.shape[0] * ref.shape[1]
        dev = ref.device
        # the attention backward writes dV in the layout of the fused output (a
        # column slice of a [M, Nt] buffer): that buffer becomes the gradient
        in_place = (dv is not None and dv.dtype == torch.bfloat16 and dv.dim() == 4
                    and dv.stride(3) == 1 and dv.stride(2) == dv.shape[3] and dv.stride(1) == Nt
                    and dv.stride(0) == dv.shape[1] * Nt and dv.storage_offset() == o2
                    and dv.untyped_storage().nbytes() == M * Nt * 2)
        if in_place:
            g = torch.empty(0, dtype=torch.bfloat16, device=dev).set_(
                dv.untyped_storage(), 0, (M, Nt), (Nt, 1))
        else:
            g = torch.empty(M, Nt, dtype=torch.bfloat16, device=dev)
        both = dq is not None and dk is not None
        if both:   # gradients of the pre-rotation q and k columns: one launch
            E.rope_into2(dq.contiguous(), g[:, :o1], dk.contiguous(), g[:, o1:o2], cs, -1.0)
        for grad, lo, hi, rot in ((dq, 0, o1, True), (dk, o1, o2, True), (dv, o2, Nt, False)):
            if grad is None:
                g[:, lo:hi].zero_()
            elif rot:   # gradient of the pre-rotation columns, straight into its slice
                if not both:
                    E.rope_into(grad.contiguous(), g[:, lo:hi], cs, -1.0)
            elif not in_place:
                g[:, lo:hi].copy_(grad.reshape(M, hi - lo))
        d = mods[0].in_features
        gx = None
        V = Vt = None
        b_outs = None
        if lora:
            # unscaled dY·B per projection: V [M, slab width] and Vt [3g, M]; with
            # the three dB (each from its column slice of dY) in the same pass
            r = mods[0].lora_r
            res = None
            if any(ctx.needs_input_grad[2 + 2 * i] for i in range(3)):
                b_outs = [m.lora_B.grad if _direct(m.lora_B) else
                          torch.zeros(m.out_features, r, dtype=torch.float32, device=dev)
                          for m in mods]
                segs = [(0, Ns[0], 0), (o1, Ns[1], gw), (o2, Ns[2], 2 * gw)]
                # (None: nothing launched, the outputs are untouched)
                res = lora_k.vdb(g, B_catT, Ut, A_cat.shape[0], segs, b_outs, gw, r)
            vdb_done = res is not None
            if res is None:
                res = lora_k.down(g, B_catT, upad=A_cat.shape[0])
            V, Vt = res
        if ctx.needs_input_grad[0]:
            w = ctx.w_kept
            if w is None:
                w = torch.empty(Nt, d, dtype=torch.bfloat16, device=dev)
                _decode_into(mods, w)
            ctx.w_kept = None
            gx = torch.empty(M, d, dtype=torch.bfloat16, device=dev)
            E.gemm_bf16_nn(g, w, gx, V, A_cat)     # dX = dY·W + V·[sA] in one GEMM
            del w
            gx = gx.view(*shp[:-1], d)
        grads = [None] * 6
        if lora:
            r = mods[0].lora_r
            scal = {m.scaling for m in mods}
            want_a = [ctx.needs_input_grad[1 + 2 * i] for i in range(3)]
            want_b = [ctx.needs_input_grad[2 + 2 * i] for i in range(3)]
            # dA of all three adapters: one pass over x (groups of gw rank columns)
            if any(want_a):
                one = len(scal) == 1
                outs = [m.lora_A.grad if (one and _direct(m.lora_A)) else
                        torch.zeros(r, d, dtype=torch.float32, device=dev) for m in mods]
                alpha = next(iter(scal)) if one else 1.0
                lora_k.wgrad(x2, Vt, 3 * gw, [(0, d, 0, alpha)], outs, gw, r, True)
                for i, m in enumerate(mods):
                    if want_a[i] and outs[i] is not m.lora_A.grad:
                        gA = outs[i] if one else outs[i] * m.scaling
                        if _direct(m.lora_A):
                            m.lora_A.grad.add_(gA)
                        else:
                            grads[2 * i] = gA.to(m.lora_A.dtype)
            # dB of each adapter from its own column slice of dY: three jobs, one
            # launch (unless the fused pass above already added them)
            if any(want_b):
                if not vdb_done:
                    jobs, off = [], 0
                    for i, m in enumerate(mods):
                        jobs.append((off, m.out_features, gw * i, 1.0))
                        off += m.out_features
                    lora_k.wgrad(g, Ut, gw, jobs, b_outs, gw, r, False)
                for i, m in enumerate(mods):
                    if want_b[i] and b_outs[i] is not m.lora_B.grad:
                        grads[2 * i + 1] = b_outs[i].to(m.lora_B.dtype)
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

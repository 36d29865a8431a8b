"""NF4 linear layer with a fused LoRA path (4-bit compute mode).

``Linear4bit`` replaces bitsandbytes' ``Linear4bit``/``matmul_4bit`` that the
reference relies on (``src/hetero/zeroq_hetero.py:477-500``).  Its frozen weight
``W [out, in]`` is stored as NF4 (packed bytes + fp32 absmax, bitsandbytes
layout); no full-precision copy of it is kept between uses.

CUDA path, per call (``csrc/gemm_sm100.cu``):

* the NF4 operand kernel expands ``W`` once per use into a transient bf16
  ``[N, K]`` operand (a flat, fully coalesced decode) that stays L2-resident for
  the GEMM that follows.  The alternative ``gemm_nf4`` decodes ``W`` inside the
  GEMM (four decode warps per CTA write the bf16 B tile straight into the
  tensor-core operand layout, no bf16 copy of ``W`` at all) and gives bit-identical
  results, but it re-decodes every weight tile once per 256 rows of ``X`` and
  measured 2.4-3.4x slower than decode-once at every M from 256 to 8192 on B200,
  so it is off by default (``ZEROQ_IN_KERNEL_DECODE=1`` enables it);
* the tcgen05/TMEM pair GEMM computes ``Y = X Wᵀ`` and, in the same MMA chain, the
  LoRA up-projection as one extra 64-wide K slab (``U = s·X Aᵀ`` against
  ``B``, both zero-padded to rank 64); the input gradient
  ``dX = dY W + (s·dY B) A`` reads the same ``[N, K]`` operand MN-major
  (``gemm_bf16_nn``), so no transposed operand is produced;
* the rank-space products ``U = x·(sA)ᵀ``, ``V = dY·B`` and the ``A``/``B`` weight
  gradients (contractions over tokens) are the tcgen05 kernels of
  ``csrc/lora_sm100.cu`` (:mod:`zeroq_b200.ops.lora`): ``U``/``V`` are computed at
  the rank rounded up to 16 and written zero-padded to the 64-wide slab plus a
  transposed copy, and the weight gradients accumulate in fp32 straight into the
  ``.grad`` buffers bound by ``FlatParams``.

The padded bf16 LoRA operands (``s·A`` as ``[64, in]``, ``B`` as ``[out, 64]``
and ``Bᵀ`` as ``[r16, out]``) are cached per module and rebuilt by one kernel when the
parameters' version counters change (every in-place update by an optimizer
bumps them; ``ShardedAdamW`` bumps them after its kernels).  Writes through
``.data`` bypass the counters: call :meth:`Linear4bit.refresh_lora_cache`
after those.

LoRA parameter names follow PEFT (``lora_A [r, in]``, ``lora_B [out, r]``,
``scaling = alpha / r``, ``B`` zero-initialised) so ``prepare_model_for_zeroq``'s
``'lora_'`` rule trains them.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn as nn

from . import _ext
from . import lora as lora_k
from .nf4 import QUANT_TYPE_ID, QuantState, dequantize_4bit, quantize_4bit


# in-kernel decode of the 4-bit weight inside the GEMM (off by default, see above)
IN_KERNEL_DECODE = os.environ.get("ZEROQ_IN_KERNEL_DECODE", "0") == "1"

# Peer-sourced weights: up to this many rows of x, the two-kernel form (peer
# gather + dequantise into a bf16 operand, then the GEMM) is faster than the
# one-kernel gather-GEMM (measured on 2 B200s at M = 1024: 0.055 / 0.159 /
# 0.483 ms against 0.071 / 0.182 / 0.538 ms for K = N = 4096 / 8192 / 12288;
# equal or slower from M = 4096 on).
AG_ONE_KERNEL_MIN_M = int(os.environ.get("ZEROQ_AG_ONE_KERNEL_MIN_M", "2049"))


def _in_kernel_ok(M: int, K: int, N: int) -> bool:
    return IN_KERNEL_DECODE and M >= 256 and K % 128 == 0 and N % 64 == 0


def _fused_ok(x: torch.Tensor, K: int, N: int, blocksize: int) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and K % 64 == 0 and N % 64 == 0
            and blocksize % 64 == 0)


def _dequant_weight(packed, absmax, N, K, blocksize, quant_type, dtype):
    st = QuantState(absmax=absmax, shape=torch.Size([N, K]), dtype=dtype, blocksize=blocksize,
                    quant_type=quant_type)
    return dequantize_4bit(packed, st, out_dtype=dtype)


# The bf16 operand a resident projection decodes for its forward GEMM is the one
# its input-gradient GEMM reads (W [N, K], MN-major there): keeping it from the
# forward to the backward halves the decode launches of a step, for the memory of
# one bf16 copy of the resident weights held between the two (4.7B: ~9.4 GB).
# The weights stay NF4-resident and are decoded every step.  Peer-sourced
# operands are never kept (that would pin every gathered layer).
# ZEROQ_KEEP_OPERANDS=0 decodes again in the backward.
KEEP_OPERANDS = os.environ.get("ZEROQ_KEEP_OPERANDS", "1") != "0"


def _nf4_operand(packed, absmax, N, K, blocksize, quant_type, transpose: bool):
    """bf16 GEMM operand from NF4: ``W [N, K]`` or ``Wᵀ [K, N]`` (``csrc/gemm_sm100.cu``)."""
    w = torch.empty(N * K, dtype=torch.bfloat16, device=packed.device)
    _ext.ext().nf4_to_bf16(packed, absmax, w, N, K, blocksize, QUANT_TYPE_ID[quant_type],
                           transpose)
    return w.view(K, N) if transpose else w.view(N, K)


def _pad_cols(t: torch.Tensor, width: int = 64) -> torch.Tensor:
    out = torch.zeros(t.shape[0], width, dtype=torch.bfloat16, device=t.device)
    out[:, : t.shape[1]] = t
    return out


def _pad_rows(t: torch.Tensor, height: int = 64) -> torch.Tensor:
    out = torch.zeros(height, t.shape[1], dtype=torch.bfloat16, device=t.device)
    out[: t.shape[0]] = t
    return out


def _direct_grad(p: Optional[torch.Tensor]) -> bool:
    """True when ``p``'s gradient is accumulated in place into its bound fp32
    ``.grad`` (parameters bound by ``FlatParams``) instead of returned to autograd."""
    return (p is not None and getattr(p, "_zq_flat_grad", False) and p.grad is not None
            and p.grad.dtype == torch.float32 and p.grad.is_contiguous())


class NF4LinearFunction(torch.autograd.Function):
    """``y = x Wᵀ + s (x Aᵀ) Bᵀ (+ bias)`` with ``W`` frozen NF4.

    CUDA path: the NF4 operand is produced in the tcgen05 operand layout and the
    LoRA up-projection rides as the extra 64-wide K slab of the same GEMM
    (``U = x·(s·A)ᵀ`` against ``B``, zero-padded to rank 64).  ``lora_ops`` is
    the cached triple ``(s·A padded [64, K], B padded [N, 64], Bᵀ [r16, N])`` in
    bf16.

    GELU MLP fusion (``act_out`` / ``pre``):

    * ``act_out="gelu"``: returns ``(h, gelu(h))`` with ``h`` the layer output; the
      GEMM epilogue writes both (no separate GELU kernel), ``gelu(h)`` is
      non-differentiable and the gradient flows through ``h``;
    * ``pre=h``: ``x`` is ``gelu(h)`` (no gradient of its own) and the gradient is
      returned for ``h`` - the input-gradient GEMM's epilogue multiplies by
      ``gelu'(h)``, so the gradient of ``gelu(h)`` is never stored.
    Off the fused path both fall back to the GELU kernels with the same results.

    SwiGLU MLP fusion (``act_out="swiglu"`` with ``gate`` / ``pre`` with ``pre_u``):

    * the up-projection with ``act_out="swiglu", gate=g`` returns ``(u, silu(g)·u)``:
      its GEMM epilogue reads ``g`` and writes both; ``silu(g)·u`` carries no
      gradient of its own (nor does ``gate`` through this function);
    * the down-projection with ``pre=g, pre_u=u``: ``x`` is ``silu(g)·u`` and the
      gradients are returned for ``g`` and ``u`` - the input-gradient GEMM's
      epilogue writes ``dg`` and ``du`` and the gradient of the activation is
      never stored.
    Off the fused path both fall back to the SwiGLU kernels with the same results.

    ``rope=cs`` (a ``[S, D/2, 2]`` cos/sin table, D = 128): the output is returned
    rotary-embedded (row m at position m % S); the GEMM epilogue applies the
    rotation, and the backward un-rotates the incoming gradient first.
    """

    @staticmethod
    def forward(ctx, x, packed, absmax, lora_A, lora_B, bias, N, K, blocksize, quant_type,
                scaling, backend, lora_ops=None, peer=None, act_out=None, pre=None, rope=None,
                pre_u=None, gate=None):
        shp = x.shape
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M = x2.shape[0]
        has_lora = lora_A is not None and lora_B is not None
        r = lora_A.shape[0] if has_lora else 0
        fused = backend != "torch" and _fused_ok(x2, K, N, blocksize) and r <= 64
        # peer = (PeerShardPool, ZeroQParameter): W stays in its owners' shards and
        # the fused gather + dequantise + GEMM kernel reads it there
        peer_fused = peer is not None and fused and _peer_ag_ok(M, N, K, blocksize)
        w_peer = None
        if peer_fused and M < AG_ONE_KERNEL_MIN_M:
            # short inputs: dequantise straight from the owners' shards (one
            # kernel), then the regular GEMM paths (epilogues included)
            w_peer = peer[0].gather_dequant(peer[1], N, K)
            peer_fused = False
        elif peer is not None and not peer_fused:
            packed, absmax = peer[0].gather(peer[1]).wait()

        # the backward reads the same W [N, K] for inputs of at least 256 rows
        keep_ok = (KEEP_OPERANDS and peer is None and M >= 256
                   and (ctx.needs_input_grad[0] or pre is not None))
        kept = []

        def operand():  # bf16 W [N, K] for the GEMM paths below
            if w_peer is not None:
                return w_peer
            w_ = _nf4_operand(packed, absmax, N, K, blocksize, quant_type, False)
            if keep_ok:
                kept.append(w_)
            return w_
        U = None
        Ut = None
        a_pad = b_pad = b_t = None
        act = None
        rope_done = False
        rope_cs = None
        if rope is not None:
            from .rope import rope_table_of

            rope_cs = rope_table_of(rope)
        if act_out not in (None, "gelu", "swiglu"):
            raise ValueError(f"unsupported fused activation {act_out!r}")
        gate2 = None
        if act_out == "swiglu":
            if gate is None:
                raise ValueError('act_out="swiglu" needs the gate projection\'s output')
            gate2 = gate.reshape(-1, N)
            if not gate2.is_contiguous():
                gate2 = gate2.contiguous()
        if fused:
            E = _ext.ext()
            y = torch.empty(M, N, dtype=x2.dtype, device=x2.device)
            if has_lora:
                if lora_ops is None:
                    lora_ops = _pack_lora(lora_A.detach(), lora_B.detach(), scaling)
                a_pad, b_pad, b_t = lora_ops
                # U [M, 64] (zero past the rank) for the GEMM slab, Ut [r16, M] for dB
                U, Ut = lora_k.down(x2, a_pad[:lora_k.round16(r)])
            if peer_fused:
                sw = None
                if act_out == "swiglu" and bias is None and gate2.dtype == torch.bfloat16:
                    act = torch.empty_like(y)
                    sw = (gate2, act)
                _, wbuf = peer[0].ag_gemm(peer[1], x2, out=y,
                                          extra=(U, b_pad) if has_lora else None, swiglu=sw)
                del wbuf
            elif (rope is not None and bias is None and _epi_ok(M, K) and N % 128 == 0
                  and rope_cs.shape[1] == 64 and M % rope_cs.shape[0] == 0
                  and not _in_kernel_ok(M, K, N)):
                w = operand()
                E.gemm_rope(x2, w, y, rope_cs, U, b_pad)
                rope_done = True
                del w
            elif act_out == "gelu" and bias is None and _epi_ok(M, K) and not _in_kernel_ok(M, K, N):
                w = operand()
                act = torch.empty_like(y)
                E.gemm_gelu(x2, w, y, act, False, U, b_pad)
                del w
            elif (act_out == "swiglu" and bias is None and _epi_ok(M, K)
                  and gate2.dtype == torch.bfloat16 and not _in_kernel_ok(M, K, N)):
                w = operand()
                act = torch.empty_like(y)
                E.gemm_swiglu(x2, w, y, act, gate2, None, False, U, b_pad)
                del w
            elif _in_kernel_ok(M, K, N) and w_peer is None:
                E.gemm_nf4(x2, packed, absmax, N, K, blocksize, QUANT_TYPE_ID[quant_type], False, y,
                           U, b_pad)
            else:
                w = operand()
                if has_lora:
                    E.gemm_bf16_tn_extra(x2, w, y, U, b_pad)
                else:
                    E.gemm_bf16_tn(x2, w, y)
                del w
        else:
            w = _dequant_weight(packed, absmax, N, K, blocksize, quant_type, torch.float32)
            y = x2.float() @ w.t()
            if has_lora:
                U = (x2.float() @ lora_A.float().t()) * scaling
                y = y + U @ lora_B.float().t()
            y = y.to(x2.dtype)
        if bias is not None:
            y = y + bias.to(y.dtype)
        if rope is not None and not rope_done:
            from .rope import rope_rows

            y = rope_rows(y, rope_cs, 1.0)
        ctx.rope = rope
        ctx.w_kept = kept[0] if kept else None
        if peer is not None:
            packed = absmax = None  # re-read from the owners in backward
        pre2 = preu2 = None
        if pre is not None:
            pre2 = pre.reshape(-1, K)
            if not pre2.is_contiguous():
                pre2 = pre2.contiguous()
        if pre_u is not None:
            preu2 = pre_u.reshape(-1, K)
            if not preu2.is_contiguous():
                preu2 = preu2.contiguous()
        # fused path: the transposed rank-space product is what the backward reads
        ctx.save_for_backward(x2 if has_lora else None, packed, absmax, lora_A, lora_B,
                              Ut if fused else U, a_pad, b_pad, b_t, pre2, preu2)
        ctx.meta = (shp, N, K, blocksize, quant_type, scaling, fused, bias is not None, has_lora, r)
        ctx.peer = peer
        y = y.view(*shp[:-1], N)
        if act_out in ("gelu", "swiglu"):
            if act is None:
                act = _gelu_kernel(y) if act_out == "gelu" else _swiglu_kernel(gate2, y.view(-1, N))
            act = act.view(*shp[:-1], N)
            ctx.mark_non_differentiable(act)
            # no zero-filled gradient for gelu(h) (it never has one): saves a
            # full-size fill per layer
            ctx.set_materialize_grads(False)
            return y, act
        return y

    @staticmethod
    def backward(ctx, gy, g_act=None):
        if gy is None:  # (grads are not materialised for the act_out form)
            ctx.w_kept = None
            return (None,) * 19
        x2, packed, absmax, lora_A, lora_B, U, a_pad, b_pad, b_t, pre2, preu2 = ctx.saved_tensors
        swiglu_in = preu2 is not None
        shp, N, K, blocksize, quant_type, scaling, fused, has_bias, has_lora, r = ctx.meta
        gy2 = gy.reshape(-1, N)
        if not gy2.is_contiguous():
            gy2 = gy2.contiguous()
        if ctx.rope is not None:  # gradient of the pre-rotation output
            from .rope import rope_grad_done, rope_rows, rope_table_of

            if not rope_grad_done(ctx.rope):  # (else the attention backward did it)
                gy2 = rope_rows(gy2, rope_table_of(ctx.rope), -1.0)
        M = gy2.shape[0]
        gx = gA = gB = gbias = None
        # with pre=h the input gradient is taken for h (through gelu'(h)); with
        # pre=g, pre_u=u for g and u (through the SwiGLU derivative)
        if swiglu_in:
            want_gx = ctx.needs_input_grad[15] or ctx.needs_input_grad[17]
        else:
            want_gx = ctx.needs_input_grad[15] if pre2 is not None else ctx.needs_input_grad[0]
        peer = ctx.peer
        peer_operand = (peer is not None and fused and M >= 256 and want_gx
                        and not _in_kernel_ok(M, N, K))
        if peer is not None and not peer_operand and want_gx:
            packed, absmax = peer[0].gather(peer[1]).wait()
        gelu_done = False
        g_swiglu = None   # (dg, du) from the SwiGLU-gradient epilogue
        if fused:
            E = _ext.ext()
            gy2 = gy2.to(torch.bfloat16)
            V = Vt = None
            b_done = False
            if has_lora:
                r16 = lora_k.round16(r)
                res = None
                if ctx.needs_input_grad[4]:
                    # V = dY·B and dB += dYᵀ·U in one pass over dY
                    direct_b = _direct_grad(lora_B)
                    out_b = lora_B.grad if direct_b else torch.zeros(N, r, dtype=torch.float32,
                                                                     device=gy2.device)
                    res = lora_k.vdb(gy2, b_t, U, 64, [(0, N, 0)], [out_b], r16, r)
                    if res is not None:
                        b_done = True
                        if not direct_b:
                            gB = out_b.to(lora_B.dtype)
                if res is None:
                    res = lora_k.down(gy2, b_t)  # [M, 64] = dY·B (unscaled), and Vᵀ
                V, Vt = res
            if want_gx:
                gx = torch.empty(M, K, dtype=torch.bfloat16, device=gy2.device)
                if (pre2 is not None and _epi_ok(M, N) and not _in_kernel_ok(M, N, K)
                        and pre2.dtype == torch.bfloat16
                        and (not swiglu_in or preu2.dtype == torch.bfloat16)):
                    if ctx.w_kept is not None:
                        w = ctx.w_kept
                    elif peer_operand:
                        w = peer[0].gather_dequant(peer[1], N, K)
                    else:
                        w = _nf4_operand(packed, absmax, N, K, blocksize, quant_type, False)
                    if swiglu_in:
                        # D = dY·W + V·(s·A); dg = D·u·silu'(g), du = D·silu(g) in the epilogue
                        du = torch.empty_like(gx)
                        E.gemm_swiglu(gy2, w, gx, du, pre2, preu2, True, V, a_pad)
                        g_swiglu = (gx.view(*shp[:-1], K), du.view(*shp[:-1], K))
                    else:
                        # dH = (dY·W + V·(s·A)) * gelu'(H) in the GEMM epilogue
                        E.gemm_gelu(gy2, w, gx, pre2, True, V, a_pad)
                        gelu_done = True
                    del w
                elif _in_kernel_ok(M, N, K):  # dX = dY·W + V·(s·A), W decoded in the kernel
                    E.gemm_nf4(gy2, packed, absmax, N, K, blocksize, QUANT_TYPE_ID[quant_type],
                               True, gx, V, a_pad)
                elif M >= 256:  # W [N, K] read MN-major from the operand kernel's copy
                    if ctx.w_kept is not None:   # the forward's operand
                        w = ctx.w_kept
                    elif peer_operand:  # straight from the owners' shards (one kernel)
                        w = peer[0].gather_dequant(peer[1], N, K)
                    else:
                        w = _nf4_operand(packed, absmax, N, K, blocksize, quant_type, False)
                    E.gemm_bf16_nn(gy2, w, gx, V, a_pad)
                    del w
                else:  # short inputs: single-CTA kernel on the transposed operand
                    w = _nf4_operand(packed, absmax, N, K, blocksize, quant_type, True)
                    if has_lora:
                        E.gemm_bf16_tn_extra(gy2, w, gx, V, a_pad.t().contiguous())
                    else:
                        E.gemm_bf16_tn(gy2, w, gx)
                    del w
                gx = gx.view(*shp[:-1], K)
            ctx.w_kept = None
            if has_lora:
                # dA += s·Vᵀ·X, dB += dYᵀ·U: bf16 operands, fp32 accumulation straight
                # into the bound gradient (or a zeroed buffer), U read as Ut [r16, M]
                if ctx.needs_input_grad[3]:
                    direct = _direct_grad(lora_A)
                    out = lora_A.grad if direct else torch.zeros(r, K, dtype=torch.float32,
                                                                 device=gy2.device)
                    lora_k.wgrad(x2, Vt, r16, [(0, K, 0, scaling)], [out], r16, r, True)
                    if not direct:
                        gA = out.to(lora_A.dtype)
                if ctx.needs_input_grad[4] and not b_done:
                    direct = _direct_grad(lora_B)
                    out = lora_B.grad if direct else torch.zeros(N, r, dtype=torch.float32,
                                                                 device=gy2.device)
                    lora_k.wgrad(gy2, U, r16, [(0, N, 0, 1.0)], [out], r16, r, False)
                    if not direct:
                        gB = out.to(lora_B.dtype)
        else:
            Vf = None
            if has_lora:
                Vf = (gy2.float() @ lora_B.float()) * scaling
            if want_gx:
                w = _dequant_weight(packed, absmax, N, K, blocksize, quant_type, torch.float32)
                g = gy2.float() @ w
                if has_lora:
                    g = g + Vf @ lora_A.float()
                gx = g.to(gy.dtype).view(*shp[:-1], K)
            if has_lora:
                if ctx.needs_input_grad[3]:
                    gA = (Vf.t() @ x2.float()).to(lora_A.dtype)
                if ctx.needs_input_grad[4]:
                    gB = (gy2.float().t() @ U.float()).to(lora_B.dtype)
        if has_bias and ctx.needs_input_grad[5]:
            gbias = gy2.float().sum(0)
        if swiglu_in:
            dg = du = None
            if gx is not None:
                if g_swiglu is None:
                    g_swiglu = _swiglu_grad_kernel(gx, pre2.view(gx.shape), preu2.view(gx.shape))
                dg, du = g_swiglu
            return (None, None, None, gA, gB, gbias, None, None, None, None, None, None, None,
                    None, None, dg, None, du, None)
        if pre2 is not None:
            g_pre = None
            if gx is not None:
                g_pre = gx if gelu_done else _gelu_grad_kernel(gx, pre2.view(gx.shape))
            return (None, None, None, gA, gB, gbias, None, None, None, None, None, None, None,
                    None, None, g_pre, None, None, None)
        return (gx, None, None, gA, gB, gbias, None, None, None, None, None, None, None, None,
                None, None, None, None, None)


def _epi_ok(M: int, K: int) -> bool:
    """Shapes the GELU-epilogue GEMMs take (pair kernel, 128-wide K stages)."""
    return M >= 256 and K % 128 == 0


def _gelu_kernel(h: torch.Tensor) -> torch.Tensor:
    from .activations import gelu

    with torch.no_grad():
        return gelu(h)


def _swiglu_kernel(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """``silu(g)·u`` with no autograd graph (the standalone SwiGLU kernel on CUDA)."""
    with torch.no_grad():
        if g.is_cuda and g.dtype == torch.bfloat16 and u.dtype == torch.bfloat16:
            out = torch.empty_like(u)
            _ext.ext().swiglu_fwd(g.contiguous(), u.contiguous(), out)
            return out
        return (torch.nn.functional.silu(g.float()) * u.float()).to(u.dtype)


def _swiglu_grad_kernel(d: torch.Tensor, g: torch.Tensor, u: torch.Tensor):
    """``(d·u·silu'(g), d·silu(g))``: the gradients of ``silu(g)·u`` for ``g`` and ``u``."""
    if d.is_cuda and d.dtype == torch.bfloat16 and g.dtype == torch.bfloat16:
        dg = torch.empty_like(g)
        du = torch.empty_like(u)
        _ext.ext().swiglu_bwd(d.contiguous(), g.contiguous(), u.contiguous(), dg, du)
        return dg, du
    gf, uf, df = g.float(), u.float(), d.float()
    sg = torch.sigmoid(gf)
    return ((df * uf * sg * (1.0 + gf * (1.0 - sg))).to(g.dtype), (df * gf * sg).to(u.dtype))


def _gelu_grad_kernel(g: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    if g.is_cuda and g.dtype == torch.bfloat16:
        out = torch.empty_like(g)
        _ext.ext().gelu_bwd(g.contiguous(), h.contiguous(), out)
        return out
    hf = h.float()
    cdf = 0.5 * (1.0 + torch.erf(hf * 0.7071067811865476))
    pdf = torch.exp(-0.5 * hf * hf) * 0.3989422804014327
    return (g.float() * (cdf + hf * pdf)).to(g.dtype)


def _peer_ag_ok(M: int, N: int, K: int, blocksize: int) -> bool:
    from ..parallel.peer import ag_gemm_ok

    return ag_gemm_ok(M, N, K, blocksize)


class MasterGatherLinearFunction(torch.autograd.Function):
    """``y = x · bf16(W)ᵀ (+ bias)`` for a trainable weight whose fp32 masters are
    sharded over the ranks (train-from-scratch): the forward gathers every rank's
    master shard over NVLink, casts it to bf16 and multiplies in one kernel
    (:meth:`~zeroq_b200.parallel.peer.PeerMasterPool.ag_gemm`); the backward
    reuses the assembled bf16 weight for ``dX``, forms ``dW = dYᵀ X`` in fp32 and
    reduce-scatters it straight into the master shard's gradient (the reference
    all-gathers the fp32 masters and reduce-scatters the gradient in a tensor
    hook, ``src/coordinator.py:606-611`` and ``:349-359``).
    """

    @staticmethod
    def forward(ctx, x, master_shard, bias, pool, zq):
        N, K = zq.original_shape
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, wbuf = pool.ag_gemm(zq, x2)
        if bias is not None:
            y = y + bias.to(y.dtype)
        ctx.save_for_backward(x2, wbuf)
        ctx.meta = (x.shape, N, K, bias is not None)
        ctx.zq = zq
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, gy):
        from ..parallel.gradient_sync import reduce_scatter_grads

        x2, wbuf = ctx.saved_tensors
        shp, N, K, has_bias = ctx.meta
        zq = ctx.zq
        gy2 = gy.reshape(-1, N).to(torch.bfloat16).contiguous()
        M = gy2.shape[0]
        E = _ext.ext()
        gx = gshard = gbias = None
        if ctx.needs_input_grad[0]:
            if M >= 256 and N % 64 == 0 and K % 64 == 0:
                gx = torch.empty(M, K, dtype=torch.bfloat16, device=gy2.device)
                E.gemm_bf16_nn(gy2, wbuf, gx, None, None)
            else:
                gx = gy2 @ wbuf
            gx = gx.view(*shp[:-1], K)
        if ctx.needs_input_grad[1]:
            gW = torch.empty(N, K, dtype=torch.float32, device=gy2.device)
            E.matmul_accum_f32(gy2.t(), x2, gW, 1.0, 0.0)
            gshard = reduce_scatter_grads(gW, zq.world_size, zq.rank, group=zq.process_group)
            gshard = gshard[: zq.master_shard.numel()].to(zq.master_shard.dtype)
        if has_bias and ctx.needs_input_grad[2]:
            gbias = gy2.float().sum(0)
        return gx, gshard, gbias, None, None


def _master_fused_ok(x: torch.Tensor, N: int, K: int) -> bool:
    from ..parallel.peer import ag_gemm_ok

    M = x.numel() // K if x.numel() else 0
    return (x.is_cuda and x.dtype == torch.bfloat16 and ag_gemm_ok(M, N, K, 32)
            and N % 64 == 0 and K % 64 == 0)


def _pack_lora(A: torch.Tensor, B: torch.Tensor, scaling: float, out=None):
    """``(s·A padded to [64, K], B padded to [N, 64], Bᵀ padded to [r16, N])`` in
    bf16; ``out`` reuses buffers whose padding is already zero."""
    r, K = A.shape
    N = B.shape[0]
    if out is None:
        out = (torch.zeros(64, K, dtype=torch.bfloat16, device=A.device),
               torch.zeros(N, 64, dtype=torch.bfloat16, device=A.device),
               torch.zeros(lora_k.round16(r), N, dtype=torch.bfloat16, device=A.device))
    a_pad, b_pad, b_t = out
    if A.is_cuda and A.dtype == torch.float32 and B.dtype == torch.float32:
        _ext.ext().lora_pack(A.contiguous(), B.contiguous(), float(scaling), a_pad, b_pad, b_t)
    else:
        a_pad[:r].copy_(A.float() * scaling)
        b_pad[:, :r].copy_(B)
        b_t[:r].copy_(B.t())
    return a_pad, b_pad, b_t


class LoraPackBatch:
    """Repack many adapters' bf16 operands in one launch (``lora_pack_many``).

    ``run(jobs)``: each job is ``(A, B, scaling, a_view, b_view, bt_view, done)``
    with the same shapes ``lora_pack`` takes; ``done()`` marks the owner's cache as
    current.  The job table lives on the device and is rebuilt only when a pointer
    or shape changes; a rebuild needs a host-to-device copy, so during stream
    capture a changed table makes ``run`` return False without launching (the
    owners then pack themselves on first use, as without the batch)."""

    def __init__(self):
        self._sig = None
        self._table = None
        self._max = 0

    @staticmethod
    def _check(A, B, a, b, t):
        r, K = A.shape
        N = B.shape[0]
        ok = (A.is_cuda and A.dtype == torch.float32 and A.is_contiguous()
              and B.dtype == torch.float32 and B.is_contiguous() and B.shape[1] == r
              and a.dtype == torch.bfloat16 and a.shape[0] >= r and a.shape[1] == K and a.stride(1) == 1
              and b.dtype == torch.bfloat16 and b.shape[0] == N and b.shape[1] >= r and b.stride(1) == 1
              and (t is None or (t.dtype == torch.bfloat16 and t.shape[0] >= r and t.shape[1] == N
                                 and t.stride(1) == 1)))
        if not ok:
            raise ValueError("LoraPackBatch: a job's operands do not have lora_pack's shapes")

    def run(self, jobs) -> bool:
        import struct

        if not jobs:
            return True
        sig = tuple((A.data_ptr(), B.data_ptr(), tuple(A.shape), tuple(B.shape), float(s),
                     a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                     0 if t is None else t.data_ptr(), 0 if t is None else t.stride(0))
                    for A, B, s, a, b, t, _ in jobs)
        if sig != self._sig:
            if torch.cuda.is_current_stream_capturing():
                return False
            rows = []
            for A, B, s, a, b, t, _ in jobs:
                self._check(A, B, a, b, t)
                r, K = A.shape
                N = B.shape[0]
                rows.append([A.data_ptr(), B.data_ptr(), a.data_ptr(), a.stride(0), b.data_ptr(),
                             b.stride(0), 0 if t is None else t.data_ptr(),
                             0 if t is None else t.stride(0), r, K, N,
                             struct.unpack("<i", struct.pack("<f", float(s)))[0]])
            self._table = torch.tensor(rows, dtype=torch.int64, device=jobs[0][0].device)
            self._max = max(A.shape[0] * A.shape[1] + 2 * B.numel() for A, B, *_ in jobs)
            self._sig = sig
        _ext.ext().lora_pack_many(self._table, int(self._max))
        for *_, done in jobs:
            done()
        return True


def nf4_linear(x, packed, absmax, out_features: int, in_features: int, bias=None,
               lora_A=None, lora_B=None, scaling: float = 1.0, blocksize: int = 64,
               quant_type: str = "nf4", backend: str = "auto", lora_ops=None, peer=None,
               act_out=None, pre=None, rope=None, pre_u=None, gate=None):
    if backend == "auto":
        backend = "fused" if x.is_cuda else "torch"
    return NF4LinearFunction.apply(x, packed, absmax, lora_A, lora_B, bias, out_features,
                                   in_features, blocksize, quant_type, scaling, backend, lora_ops,
                                   peer, act_out, pre, rope, pre_u, gate)


class Linear4bit(nn.Module):
    """Frozen NF4 weight + optional bias + optional LoRA adapter.

    The module can hold its NF4 data permanently (4-bit compute, "gather once")
    or receive it from the coordinator before each use (gather/release with
    ``compute_in_4bit``) through :meth:`set_nf4` / :meth:`clear_nf4`.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 blocksize: int = 64, quant_type: str = "nf4", lora_r: int = 0,
                 lora_alpha: float = 16.0, device=None, dtype=torch.bfloat16,
                 backend: str = "auto"):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.blocksize = blocksize
        self.quant_type = quant_type
        self.compute_dtype = dtype
        self.backend = backend
        self.weight = nn.Parameter(torch.empty(0, device=device, dtype=dtype), requires_grad=False)
        self.register_buffer("weight_packed", None)
        self.register_buffer("weight_absmax", None)
        self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) \
            if bias else None
        self.lora_r = lora_r
        if lora_r > 0:
            self.scaling = lora_alpha / lora_r
            self.lora_A = nn.Parameter(torch.empty(lora_r, in_features, device=device,
                                                   dtype=torch.float32))
            self.lora_B = nn.Parameter(torch.zeros(out_features, lora_r, device=device,
                                                   dtype=torch.float32))
            nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        else:
            self.scaling = 0.0
            self.lora_A = None
            self.lora_B = None
        self._lora_ops = None
        self._lora_key = None
        self._peer = None
        self._master = None

    # -- weight management ---------------------------------------------------
    @classmethod
    def from_linear(cls, lin: nn.Linear, blocksize: int = 64, quant_type: str = "nf4",
                    lora_r: int = 0, lora_alpha: float = 16.0, dtype=torch.bfloat16,
                    quantize: bool = True):
        m = cls(lin.in_features, lin.out_features, bias=lin.bias is not None,
                blocksize=blocksize, quant_type=quant_type, lora_r=lora_r,
                lora_alpha=lora_alpha, device=lin.weight.device, dtype=dtype)
        if lin.bias is not None:
            m.bias.data.copy_(lin.bias.data)
        if quantize and lin.weight.numel():
            m.quantize_from(lin.weight.data)
        return m

    def quantize_from(self, w: torch.Tensor):
        """Quantise a full-precision ``[out, in]`` weight into resident NF4 storage.

        The weight is cast to fp16 first, as the reference does before calling
        bitsandbytes (``src/coordinator.py:166-168``)."""
        if tuple(w.shape) != (self.out_features, self.in_features):
            raise ValueError(f"weight shape {tuple(w.shape)} != "
                             f"{(self.out_features, self.in_features)}")
        packed, st = quantize_4bit(w.detach().to(torch.float16), self.blocksize, self.quant_type)
        self.set_nf4(packed, st.absmax)

    def set_nf4(self, packed: torch.Tensor, absmax: torch.Tensor, meta: Optional[dict] = None):
        self.weight_packed = packed.reshape(-1)
        self.weight_absmax = absmax.reshape(-1).float()
        self._peer = None

    def set_peer_source(self, pool, zq):
        """Use the NF4 shards of ``zq`` where they live (every rank's piece in
        ``pool``'s peer memory) instead of an assembled copy: the forward GEMM
        gathers and dequantises them itself (one kernel)."""
        self.weight_packed = None
        self.weight_absmax = None
        self._peer = (pool, zq)

    def clear_nf4(self):
        self.weight_packed = None
        self.weight_absmax = None
        self._peer = None

    def set_master_source(self, pool, zq):
        """Train-from-scratch: read the weight from every rank's fp32 master shard
        inside the forward GEMM (:class:`MasterGatherLinearFunction`) instead of an
        all-gathered full-precision copy."""
        self._master = (pool, zq)

    def clear_master_source(self):
        self._master = None

    @property
    def has_nf4(self) -> bool:
        return self.weight_packed is not None or getattr(self, "_peer", None) is not None

    def dequantized_weight(self, dtype=torch.float32) -> torch.Tensor:
        if getattr(self, "_peer", None) is not None:
            packed, absmax = self._peer[0].gather(self._peer[1]).wait()
            return _dequant_weight(packed, absmax, self.out_features, self.in_features,
                                   self.blocksize, self.quant_type, dtype)
        return _dequant_weight(self.weight_packed, self.weight_absmax, self.out_features,
                               self.in_features, self.blocksize, self.quant_type, dtype)

    # -- LoRA operand cache ------------------------------------------------------
    def refresh_lora_cache(self):
        """Drop the cached padded LoRA operands (after writes through ``.data``)."""
        self._lora_key = None

    def _lora_state_key(self):
        """What the cached LoRA operands were packed from (versions change on every
        in-place update, e.g. an optimizer step)."""
        A, B = self.lora_A, self.lora_B
        return (A._version, B._version, A.data_ptr(), B.data_ptr(), float(self.scaling),
                tuple(A.shape), tuple(B.shape))

    def _lora_operands(self):
        A, B = self.lora_A, self.lora_B
        if A is None or B is None or not A.is_cuda or A.shape[0] > 64:
            return None
        key = self._lora_state_key()
        if self._lora_key != key:
            reuse = self._lora_ops
            if reuse is not None and (reuse[0].shape != (64, A.shape[1])
                                      or reuse[1].shape != (B.shape[0], 64)
                                      or reuse[2].shape != (lora_k.round16(A.shape[0]),
                                                            B.shape[0])
                                      or reuse[0].device != A.device):
                reuse = None
            with torch.no_grad():
                self._lora_ops = _pack_lora(A.detach(), B.detach(), self.scaling, reuse)
            self._lora_key = key
        return self._lora_ops

    # -- forward -------------------------------------------------------------
    def forward(self, x: torch.Tensor, act_out: Optional[str] = None,
                pre=None, rope=None, gate: Optional[torch.Tensor] = None):
        """``act_out="gelu"``: return ``(y, gelu(y))`` with ``gelu(y)`` carrying no
        gradient of its own; ``pre=h``: ``x`` is ``gelu(h)`` and the gradient goes to
        ``h`` (the two halves of a GELU MLP; see :class:`NF4LinearFunction`).
        ``act_out="swiglu", gate=g``: return ``(y, silu(g)·y)``, the second carrying
        no gradient; ``pre=(g, u)``: ``x`` is ``silu(g)·u`` and the gradients go to
        ``g`` and ``u`` (the SwiGLU MLP).
        ``rope``: a cos/sin table or a :class:`~zeroq_b200.ops.rope.RopeSpec` - return
        the output rotary-embedded."""
        pre_u = None
        if isinstance(pre, tuple):
            pre, pre_u = pre
        master = getattr(self, "_master", None)
        if master is not None:
            pool, zq = master
            if (act_out is None and pre is None and rope is None and not self.lora_r
                    and _master_fused_ok(x, self.out_features, self.in_features)):
                return MasterGatherLinearFunction.apply(x, zq.master_shard, self.bias, pool, zq)
            # off the fused path: the regular fp32 all-gather into self.weight
            self._master = None
            zq._start_gather_fp32(zq.process_group, async_op=False)
        peer = getattr(self, "_peer", None)
        if peer is not None:
            ops = self._lora_operands() if (self.lora_r and x.is_cuda) else None
            return nf4_linear(x, None, None, self.out_features, self.in_features, self.bias,
                              self.lora_A, self.lora_B, self.scaling, self.blocksize,
                              self.quant_type, self.backend, ops, peer, act_out, pre, rope,
                              pre_u, gate)
        if self.weight_packed is None:
            if self.weight.numel() == 0:
                raise RuntimeError("Linear4bit has no weight: neither NF4 data nor a "
                                   "gathered full-precision weight is present")
            if pre is not None:  # same gradient path as the fused form: through h (g, u)
                from .activations import gelu, swiglu

                x = swiglu(pre, pre_u) if pre_u is not None else gelu(pre)
            y = torch.nn.functional.linear(x, self.weight.to(x.dtype),
                                           None if self.bias is None else self.bias.to(x.dtype))
            if self.lora_r:
                y = y + (x @ self.lora_A.t().to(x.dtype)) @ self.lora_B.t().to(x.dtype) * self.scaling
            if rope is not None:
                from .rope import rope_rows_autograd

                y = rope_rows_autograd(y.reshape(-1, y.shape[-1]), rope).view(y.shape)
            if act_out == "gelu":
                return y, _gelu_kernel(y.detach())
            if act_out == "swiglu":
                return y, _swiglu_kernel(gate.detach(), y.detach())
            return y
        ops = self._lora_operands() if (self.lora_r and x.is_cuda) else None
        return nf4_linear(x, self.weight_packed, self.weight_absmax, self.out_features,
                          self.in_features, self.bias, self.lora_A, self.lora_B,
                          self.scaling, self.blocksize, self.quant_type, self.backend, ops,
                          None, act_out, pre, rope, pre_u, gate)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"quant={self.quant_type}/{self.blocksize}, lora_r={self.lora_r}")

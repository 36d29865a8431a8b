"""Causal (GQA-capable) flash attention, forward and backward.

Tensors keep the projection layout ``[B, S, H, D]`` so no transposes surround
the kernels.  Forward and backward run on the 5th-generation tensor cores
(``csrc/attention_sm100.cu``): the forward with TMA-fed Q/K/V tiles, S and O
accumulated in tensor memory and softmax in registers, writing ``O`` and the
row log-sum-exp ``L``; the backward as a ``delta = rowsum(dO * O)`` pass, a dQ
kernel per query tile and a dK/dV kernel per key tile, both recomputing P from
``L`` with S, dP, P and dS in tensor memory, no atomics.  The kernels are built
for 128-wide heads; narrower heads (``D`` = 64 and other multiples of 16) are
zero-padded to 128 - padded columns change no score and come out zero - so
every head size up to 128 runs on the same kernels (at 128-wide cost).

CPU tensors, ``S`` not a multiple of 128 and heads wider than 128 use PyTorch's
SDPA (the oracle).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _ext


def attention_reference(q, k, v, causal: bool = True, scale=None):
    B, S, Hq, D = q.shape
    Hk = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qt = q.transpose(1, 2).float()
    kt = k.transpose(1, 2).float()
    vt = v.transpose(1, 2).float()
    if Hk != Hq:
        rep = Hq // Hk
        kt = kt.repeat_interleave(rep, dim=1)
        vt = vt.repeat_interleave(rep, dim=1)
    o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, scale=scale)
    return o.transpose(1, 2).to(q.dtype)


def _tma_ok(t: torch.Tensor) -> bool:
    return (t.stride(-1) == 1 and all(st % 8 == 0 for st in t.stride()[:-1])
            and t.data_ptr() % 16 == 0)


def _pad128(t: torch.Tensor) -> torch.Tensor:
    """``[B, S, H, D]`` (D < 128) zero-padded to ``[B, S, H, 128]``."""
    out = t.new_zeros(*t.shape[:-1], 128)
    out[..., : t.shape[-1]] = t
    return out


def _tc_ok(q: torch.Tensor) -> bool:
    D = q.shape[-1]
    return q.shape[1] % 128 == 0 and q.shape[1] > 0 and D <= 128 and D % 16 == 0


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, rope=None):
        D = q.shape[-1]
        ctx.d = D
        if D < 128:   # narrower heads run zero-padded on the 128-wide kernels
            q, k, v = _pad128(q), _pad128(k), _pad128(v)
        # the tcgen05 kernels read q/k/v through TMA maps and take strided views
        # (column slices of a fused q/k/v projection) as they are
        q, k, v = (t if _tma_ok(t) else t.contiguous() for t in (q, k, v))
        B, S, Hq, _ = q.shape
        o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        lse = torch.empty(B, Hq, S, dtype=torch.float32, device=q.device)
        _ext.ext().attn_fwd_tc(q, k, v, o, lse, bool(causal), float(scale))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        ctx.rope = rope if (rope is not None and hasattr(rope, "grads_unrotated")) else None
        return o if D == 128 else o[..., :D]

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        D = ctx.d
        do = do.contiguous() if D == 128 else _pad128(do)
        dq, dk = (torch.empty(t.shape, dtype=t.dtype, device=t.device) for t in (q, k))
        dv = _like_token_pitched(v) if D == 128 else None
        if dv is None:
            dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
        rope = ctx.rope
        cs = rope.cs if (rope is not None and D == 128 and rope.cs.shape[0] == q.shape[1]) else None
        _ext.ext().attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, bool(ctx.causal), float(ctx.scale),
                               None, cs)
        if cs is not None:
            rope.grads_unrotated = True  # dQ/dK are gradients of the pre-rotation q/k
        if D < 128:
            dq, dk, dv = dq[..., :D], dk[..., :D], dv[..., :D]
        return dq, dk, dv, None, None, None


def _like_token_pitched(v: torch.Tensor):
    """For ``v`` a column slice of a token-pitched 2-D buffer (the fused q/k/v
    projection's output ``[B*S, Nq+Nk+Nv]``), a gradient with the same layout in a
    fresh buffer of that width: the backward writes dV straight into the slice
    the fused projection's backward reads, so no copy assembles its gradient."""
    B, S, H, D = v.shape
    P = v.stride(1)
    if (v.stride(3) != 1 or v.stride(2) != D or P <= H * D or v.stride(0) != S * P
            or P % 8 or v.storage_offset() + H * D > P):
        return None
    buf = torch.empty(B * S * P, dtype=v.dtype, device=v.device)
    return buf.as_strided(v.shape, v.stride(), v.storage_offset())


def flash_attention(q, k, v, causal: bool = True, scale=None, rope=None):
    """``rope``: the :class:`~zeroq_b200.ops.rope.RopeSpec` with which q and k were
    rotated by their projections; the backward then writes dQ/dK rotated back
    (tcgen05 path) and marks the spec so the projections do not rotate again."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if q.is_cuda and q.dtype == torch.bfloat16 and _tc_ok(q):
        return _FlashAttn.apply(q, k, v, causal, scale, rope)
    return attention_reference(q, k, v, causal, scale)

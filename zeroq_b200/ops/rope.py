"""Rotary position embedding (rotate-half convention: pairs ``(i, i + D/2)``).

``apply_rope(q, k, theta)`` rotates ``q [B,S,Hq,D]`` and ``k [B,S,Hk,D]`` by
position-dependent angles ``pos * theta^(-2i/D)``; the backward is the rotation
by the negated angle.  CUDA tensors run ``csrc/elementwise.cu``'s kernel, which
computes the angles in fp32 per element (no cos/sin table in HBM).
"""

from __future__ import annotations

import torch

from . import _ext


def rope_reference(x: torch.Tensor, theta: float, sign: float = 1.0) -> torch.Tensor:
    B, S, H, D = x.shape
    half = D // 2
    inv = theta ** (-torch.arange(0, half, dtype=torch.float64, device=x.device) * 2.0 / D)
    pos = torch.arange(S, dtype=torch.float64, device=x.device)
    ang = (pos[:, None] * inv[None, :]).float()
    cos = torch.cos(ang)[None, :, None, :]
    sin = torch.sin(ang)[None, :, None, :] * sign
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


_TABLES = {}


def rope_table(S: int, D: int, theta: float, device) -> torch.Tensor:
    """fp32 ``[S, D/2, 2]`` (cos, sin) of the angles ``pos * theta^(-2i/D)``; the
    angle is formed in fp64 and rounded to fp32 before cos/sin, as in
    :func:`rope_reference`.  Cached per (S, D, theta, device)."""
    key = (S, D, float(theta), str(device))
    t = _TABLES.get(key)
    if t is None:
        half = D // 2
        inv = theta ** (-torch.arange(0, half, dtype=torch.float64, device=device) * 2.0 / D)
        pos = torch.arange(S, dtype=torch.float64, device=device)
        ang = (pos[:, None] * inv[None, :]).float()
        t = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).contiguous()
        _TABLES[key] = t
    return t


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, theta):
        cs = rope_table(q.shape[1], q.shape[3], theta, q.device)
        qo = torch.empty_like(q)
        ko = torch.empty_like(k)
        _ext.ext().rope(q.contiguous(), qo, cs, 1.0)
        _ext.ext().rope(k.contiguous(), ko, cs, 1.0)
        ctx.cs = cs
        return qo, ko

    @staticmethod
    def backward(ctx, gq, gk):
        dq = torch.empty_like(gq)
        dk = torch.empty_like(gk)
        _ext.ext().rope(gq.contiguous(), dq, ctx.cs, -1.0)
        _ext.ext().rope(gk.contiguous(), dk, ctx.cs, -1.0)
        return dq, dk, None


def apply_rope(q: torch.Tensor, k: torch.Tensor, theta: float = 10000.0):
    if q.is_cuda and q.dtype == torch.bfloat16:
        return _Rope.apply(q, k, theta)
    return rope_reference(q, theta), rope_reference(k, theta)


def rope_rows(x: torch.Tensor, cs: torch.Tensor, sign: float = 1.0) -> torch.Tensor:
    """Rotate the rows of ``x [M, H*D]`` (row m at position m % S, heads of
    ``D = 2 * cs.shape[1]``) by the table ``cs [S, D/2, 2]`` (``sign=-1``: the
    inverse rotation, i.e. the backward).  No autograd."""
    S, half = cs.shape[0], cs.shape[1]
    D = 2 * half
    M, N = x.shape
    x4 = x.reshape(M // S, S, N // D, D)
    if x.is_cuda and x.dtype == torch.bfloat16:
        out = torch.empty_like(x4)
        _ext.ext().rope(x4.contiguous(), out, cs, float(sign))
        return out.view(M, N)
    xf = x4.float()
    c = cs[..., 0][None, :, None, :].float()
    s_ = cs[..., 1][None, :, None, :].float() * sign
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], dim=-1).to(x.dtype).view(M, N)


class RopeSpec:
    """The rotary table ``cs`` of one layer's q/k projections, shared with the
    attention that consumes their outputs.  A projection given a spec returns its
    output rotated (in the GEMM epilogue where it can); when the attention backward
    writes dQ/dK already rotated back it sets ``grads_unrotated``, and the
    projections then skip their own inverse rotation."""

    def __init__(self, cs: torch.Tensor):
        self.cs = cs
        self.grads_unrotated = False


def rope_table_of(rope) -> torch.Tensor:
    return rope.cs if isinstance(rope, RopeSpec) else rope


def rope_grad_done(rope) -> bool:
    return isinstance(rope, RopeSpec) and rope.grads_unrotated


class _RopeRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, rope):
        ctx.rope = rope
        return rope_rows(x, rope_table_of(rope), 1.0)

    @staticmethod
    def backward(ctx, g):
        if rope_grad_done(ctx.rope):
            return g, None
        return rope_rows(g.contiguous(), rope_table_of(ctx.rope), -1.0), None


def rope_rows_autograd(x: torch.Tensor, rope) -> torch.Tensor:
    return _RopeRows.apply(x, rope)

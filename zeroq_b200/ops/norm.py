"""RMSNorm with an optional fused residual add.

``add_rmsnorm(h, delta, w)`` returns ``(h + delta, rmsnorm(h + delta) * w)`` in
one kernel (``csrc/elementwise.cu``); its backward adds the incoming residual
gradient to the norm's input gradient in the same kernel and writes one row of
per-CTA weight-gradient partial sums, reduced here.  On CPU the PyTorch
expressions below are used; they are also the numerics oracle.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _ext


def rmsnorm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * r * w.float()).to(x.dtype)


class _AddRMSNorm(torch.autograd.Function):
    """``(h + delta, rmsnorm(h + delta))`` in one kernel."""

    @staticmethod
    def forward(ctx, h, delta, w, eps):
        D = h.shape[-1]
        h2 = h.reshape(-1, D).contiguous()
        d2 = delta.reshape(-1, D).contiguous()
        M = h2.shape[0]
        hout = torch.empty_like(h2)
        y = torch.empty_like(h2)
        rstd = torch.empty(M, dtype=torch.float32, device=h.device)
        _ext.ext().add_rmsnorm_fwd(h2, d2, w, hout, y, rstd, float(eps))
        ctx.save_for_backward(hout, w, rstd)
        ctx.shape = h.shape
        return hout.view(h.shape), y.view(h.shape)

    @staticmethod
    def backward(ctx, g_h, g_y):
        hout, w, rstd = ctx.saved_tensors
        dx, dw = _norm_bwd(g_y, g_h, hout, w, rstd, ctx.needs_input_grad[2])
        dx = dx.view(ctx.shape)
        return dx, dx, None if dw is None else dw.to(w.dtype), None


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        _ext.ext().add_rmsnorm_fwd(x2, None, w, x2, y, rstd, float(eps))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, g_y):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = _norm_bwd(g_y, None, x2, w, rstd, ctx.needs_input_grad[1])
        return dx.view(ctx.shape), None if dw is None else dw.to(w.dtype), None


def _norm_bwd(g_y, g_h, x2, w, rstd, want_dw: bool = True):
    """``(dx, dw)``; ``dw`` is None when not wanted or when it was added straight
    into ``w``'s bound fp32 gradient (a parameter bound by ``FlatParams``)."""
    D = x2.shape[-1]
    gy2 = g_y.reshape(-1, D).contiguous() if g_y is not None else torch.zeros_like(x2)
    gh2 = g_h.reshape(-1, D).contiguous() if g_h is not None else None
    dx = torch.empty_like(x2)
    grid = min(x2.shape[0], _num_sms(x2.device) * 2)
    dw_part = torch.empty(grid, D, dtype=torch.float32, device=x2.device)
    E = _ext.ext()
    E.rmsnorm_bwd(gy2, x2, w, rstd, gh2, dx, dw_part)
    if not want_dw:
        return dx, None
    # the per-CTA partial rows fold into the gradient in one column-sum kernel
    direct = (getattr(w, "_zq_flat_grad", False) and w.grad is not None
              and w.grad.dtype == torch.float32 and w.grad.is_contiguous() and D % 4 == 0
              and w.grad.data_ptr() % 16 == 0)
    if direct:
        E.colsum_accum(dw_part, w.grad)
        return dx, None
    dw = torch.zeros(D, dtype=torch.float32, device=x2.device)
    if D % 4 == 0:
        E.colsum_accum(dw_part, dw)
    else:
        dw = dw_part.sum(0)
    return dx, dw


_SMS = {}


def _num_sms(device) -> int:
    i = device.index if device.index is not None else torch.cuda.current_device()
    if i not in _SMS:
        _SMS[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SMS[i]


def add_rmsnorm(h: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor,
                eps: float = 1e-6):
    """Returns ``(h_new, y)`` with ``h_new = h + delta`` (or ``h``) and
    ``y = h_new / rms(h_new) * w``."""
    if h.is_cuda and h.dtype == torch.bfloat16:
        if delta is None:
            return h, _RMSNorm.apply(h, w, eps)
        return _AddRMSNorm.apply(h, delta, w, eps)
    hn = h + delta if delta is not None else h
    return hn, rmsnorm_reference(hn, w, eps)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return add_rmsnorm(x, None, w, eps)[1]

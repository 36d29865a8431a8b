"""GELU (erf form) and SwiGLU, forward and backward (``csrc/elementwise.cu``).

``swiglu(gate, up) = silu(gate) * up``.  Both kernels read bf16 and compute in
fp32; the erf and exp calls are CUDA's own functions.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = torch.empty_like(x)
        _ext.ext().gelu_fwd(x.contiguous(), y)
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        _ext.ext().gelu_bwd(g.contiguous(), x.contiguous(), dx)
        return dx


def gelu(x: torch.Tensor) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.bfloat16:
        return _Gelu.apply(x)
    return F.gelu(x.float()).to(x.dtype)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        y = torch.empty_like(gate)
        _ext.ext().swiglu_fwd(gate.contiguous(), up.contiguous(), y)
        ctx.save_for_backward(gate, up)
        return y

    @staticmethod
    def backward(ctx, g):
        gate, up = ctx.saved_tensors
        dg = torch.empty_like(gate)
        du = torch.empty_like(up)
        _ext.ext().swiglu_bwd(g.contiguous(), gate.contiguous(), up.contiguous(), dg, du)
        return dg, du


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    if gate.is_cuda and gate.dtype == torch.bfloat16:
        return _SwiGLU.apply(gate, up)
    return (F.silu(gate.float()) * up.float()).to(gate.dtype)

"""Optimizer update kernels on flat buffers.

* :func:`adamw_step` - decoupled-weight-decay Adam on a flat fp32 master with
  fp32 moments; optionally writes a bf16 copy of the updated parameters.  The
  grad may be scaled by ``grad_scale`` (1/W after a reduce-scatter, and gradient
  clipping) inside the kernel.
* :func:`lion_step` - Lion (Chen et al. 2023, "Symbolic Discovery of
  Optimization Algorithms") on an fp32 or fp16 master shard.  For fp16 masters
  the new value is rounded stochastically: ``x + u * |x| * eps_fp16`` with
  ``u ~ U(-0.5, 0.5)`` drawn from a counter-based Philox4x32-10 stream (Salmon
  et al., SC'11) keyed by ``seed`` and the element index, as the reference does
  with ``torch.uniform_`` (``src/coordinator.py:1031-1035``).

CPU tensors take the PyTorch expressions (the oracle).
"""

from __future__ import annotations

import torch

from . import _ext


def adamw_step(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor,
               exp_avg_sq: torch.Tensor, *, lr: float, beta1: float = 0.9,
               beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.0,
               step: int = 1, grad_scale: float = 1.0, param_bf16: torch.Tensor = None,
               bc_dev: torch.Tensor = None, clip_sq: torch.Tensor = None, max_norm: float = 0.0):
    """In-place AdamW on flat fp32 tensors (``grad`` may be fp32 or bf16).
    ``bc_dev``: fp32 [2] bias corrections on the device (device-side optimizer
    clock), used instead of ``step``.  ``clip_sq``: fp32 [1] squared global
    gradient norm on the device; the gradient is then also scaled by
    ``min(1, max_norm / sqrt(clip_sq))`` inside the kernel."""
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    if param.is_cuda and (bc_dev is not None or clip_sq is not None):
        _ext.ext().adamw_step_dev(param, grad, exp_avg, exp_avg_sq, param_bf16, float(lr),
                                  float(beta1), float(beta2), float(eps), float(weight_decay),
                                  float(bc1), float(bc2), float(grad_scale), bc_dev, clip_sq,
                                  float(max_norm))
        return
    if param.is_cuda:
        _ext.ext().adamw_step(param, grad, exp_avg, exp_avg_sq, param_bf16, float(lr),
                              float(beta1), float(beta2), float(eps), float(weight_decay),
                              float(bc1), float(bc2), float(grad_scale))
        return
    if clip_sq is not None:
        grad_scale = grad_scale * min(1.0, max_norm / (float(clip_sq.reshape(-1)[0]) ** 0.5 + 1e-6))
    g = grad.float() * grad_scale
    param.mul_(1.0 - lr * weight_decay)
    exp_avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    denom = (exp_avg_sq / bc2).sqrt_().add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)
    if param_bf16 is not None:
        param_bf16.copy_(param)


def lion_step(master: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, *, lr: float,
              beta1: float = 0.9, beta2: float = 0.99, wd: float = 0.0, seed: int = 0):
    """In-place Lion on a flat master shard (fp32 or fp16) with fp32 momentum ``m``."""
    if master.is_cuda:
        _ext.ext().lion_step(master.view(-1), grad.reshape(-1), m.view(-1), float(lr),
                             float(beta1), float(beta2), float(wd), int(seed) & 0xFFFFFFFFFFFF)
        return
    g = grad.reshape(-1).float()
    upd = torch.sign(m * beta1 + g * (1.0 - beta1))
    x = master.view(-1).float()
    x = x - lr * (upd + wd * x)
    m.mul_(beta2).add_(g, alpha=1.0 - beta2)
    if master.dtype == torch.float16:
        gen = torch.Generator(device="cpu").manual_seed(int(seed))
        noise = torch.rand(x.shape, generator=gen) - 0.5
        eps = (x.abs() * torch.finfo(torch.float16).eps).clamp(min=torch.finfo(torch.float16).tiny)
        master.view(-1).copy_((x + noise * eps).half())
    else:
        master.view(-1).copy_(x.to(master.dtype))

"""Cross-entropy over (vocab-padded) logits, fused softmax + loss + gradient.

The logits buffer is ``[M, V_pad]`` with ``V_pad`` a multiple of 64 (so rows stay
16-byte aligned for TMA); only the first ``vocab`` columns are real.  Forward
(``csrc/elementwise.cu``) makes one pass per row with an online max/sum and
returns per-row loss and log-sum-exp; backward writes
``(softmax - onehot) * g / n_valid`` in place of the logits (the logits are dead
after the loss), so the gradient costs one read and one write.
Targets equal to ``ignore_index`` contribute nothing.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext


class _FusedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, vocab, ignore_index):
        M = logits.shape[0]
        loss_rows = torch.empty(M, dtype=torch.float32, device=logits.device)
        lse = torch.empty(M, dtype=torch.float32, device=logits.device)
        count = torch.zeros(1, dtype=torch.float32, device=logits.device)
        _ext.ext().ce_fwd(logits, targets, loss_rows, lse, count, int(vocab), int(ignore_index))
        loss = loss_rows.sum() / count.clamp_min(1.0)
        ctx.save_for_backward(logits, targets, lse, count)
        ctx.vocab, ctx.ignore_index = vocab, ignore_index
        return loss

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse, count = ctx.saved_tensors
        scale = (g.float() / count.clamp_min(1.0)).reshape(1)
        _ext.ext().ce_bwd(logits, targets, lse, scale, int(ctx.vocab), int(ctx.ignore_index))
        return logits, None, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, vocab: int = None,
                  ignore_index: int = -100) -> torch.Tensor:
    """Mean next-token loss over non-ignored rows. ``logits [M, V_pad]``, ``targets [M]``."""
    vocab = logits.shape[-1] if vocab is None else vocab
    if logits.is_cuda and logits.dtype == torch.bfloat16:
        return _FusedCE.apply(logits.contiguous(), targets.contiguous().to(torch.int64), vocab,
                              ignore_index)
    return F.cross_entropy(logits[:, :vocab].float(), targets.long(), ignore_index=ignore_index)

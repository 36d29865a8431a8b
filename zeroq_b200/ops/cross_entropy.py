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
        _ext.ext().ce_fwd(logits, targets, loss_rows, lse, count, int(vocab), int(ignore_index), 0,
                          int(vocab))
        loss = loss_rows.sum() / count.clamp_min(1.0)
        ctx.save_for_backward(logits, targets, lse, count)
        ctx.vocab, ctx.ignore_index = vocab, ignore_index
        return loss

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse, count = ctx.saved_tensors
        scale = (g.float() / count.clamp_min(1.0)).reshape(1)
        _ext.ext().ce_bwd(logits, targets, lse, scale, int(ctx.vocab), int(ctx.ignore_index), 0,
                          int(ctx.vocab))
        return logits, None, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, vocab: int = None,
                  ignore_index: int = -100) -> torch.Tensor:
    """Mean next-token loss over non-ignored rows. ``logits [M, V_pad]``, ``targets [M]``."""
    vocab = logits.shape[-1] if vocab is None else vocab
    if logits.is_cuda and logits.dtype == torch.bfloat16:
        return _FusedCE.apply(logits.contiguous(), targets.contiguous().to(torch.int64), vocab,
                              ignore_index)
    return F.cross_entropy(logits[:, :vocab].float(), targets.long(), ignore_index=ignore_index)


class _ChunkedHeadCE(torch.autograd.Function):
    """``loss = CE(h · Wᵀ, targets)`` with the vocabulary processed in column chunks,
    so the ``[M, V]`` logits never exist at once (only one ``[M, chunk]`` block).

    Forward, per chunk: head GEMM into the block, then the chunk's row
    log-sum-exp and (for rows whose target lies in it) the target logit; the
    chunks' log-sum-exps combine into the row's.  Backward, per chunk: the head
    GEMM again, ``(softmax - onehot) · g / n`` in place, and ``dh += block · W_c``
    (fp32 accumulation).  Costs one extra head GEMM against the unchunked path
    and saves ``M × V`` bf16 logits (2.5 GB at 8192 tokens and V = 152064).
    ``W`` is frozen here (a trainable head takes the unchunked path).
    """

    @staticmethod
    def forward(ctx, h, W, targets, vocab, ignore_index, chunk):
        from .gemm import gemm_bt

        E = _ext.ext()
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        M = h2.shape[0]
        tg = targets.reshape(-1).contiguous().to(torch.int64)
        starts = list(range(0, vocab, chunk))
        lses = torch.empty(len(starts), M, dtype=torch.float32, device=h2.device)
        tlog = torch.zeros(M, dtype=torch.float32, device=h2.device)
        count = torch.zeros(1, dtype=torch.float32, device=h2.device)
        loss_c = torch.empty(M, dtype=torch.float32, device=h2.device)
        for i, c0 in enumerate(starts):
            n = min(chunk, vocab - c0)
            npad = (n + 127) // 128 * 128      # whole GEMM tiles; padded columns unused
            block = gemm_bt(h2, W[c0:c0 + npad])
            E.ce_fwd(block, tg, loss_c, lses[i], count, n, int(ignore_index), c0, vocab)
            # rows whose target is in this chunk: logit[target] = lse_c - loss_c
            inside = (tg >= c0) & (tg < c0 + n)
            tlog = torch.where(inside, lses[i] - loss_c, tlog)
            del block
        lse = torch.logsumexp(lses, dim=0)
        valid = (tg != ignore_index) & (tg >= 0) & (tg < vocab)
        loss = torch.where(valid, lse - tlog, torch.zeros_like(lse)).sum() / count.clamp_min(1.0)
        ctx.save_for_backward(h2, W, tg, lse, count)
        ctx.meta = (h.shape, vocab, ignore_index, chunk)
        return loss

    @staticmethod
    def backward(ctx, g):
        from .gemm import gemm_bt, gemm_nn

        h2, W, tg, lse, count = ctx.saved_tensors
        hshape, vocab, ignore_index, chunk = ctx.meta
        E = _ext.ext()
        scale = (g.float() / count.clamp_min(1.0)).reshape(1)
        dh = torch.zeros(h2.shape, dtype=torch.float32, device=h2.device)
        Wd = W.detach()
        for c0 in range(0, vocab, chunk):
            n = min(chunk, vocab - c0)
            npad = (n + 127) // 128 * 128
            block = gemm_bt(h2, Wd[c0:c0 + npad])
            E.ce_bwd(block, tg, lse, scale, n, int(ignore_index), c0, vocab)
            dh.add_(gemm_nn(block, Wd[c0:c0 + npad]))
            del block
        return dh.to(h2.dtype).view(hshape), None, None, None, None, None


def lm_head_cross_entropy(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor, vocab: int,
                          ignore_index: int = -100, chunk: int = 16384) -> torch.Tensor:
    """Mean next-token loss of ``h · Wᵀ`` (``W [V_pad, d]``, rows past ``vocab``
    unused) without materialising the logits: the vocabulary is processed in
    chunks of ``chunk`` columns (a multiple of 128).  CUDA bf16 with a frozen
    ``W``; otherwise the logits are formed and :func:`cross_entropy` is used."""
    if (h.is_cuda and h.dtype == torch.bfloat16 and W.dtype == torch.bfloat16
            and not W.requires_grad and chunk % 128 == 0 and h.shape[-1] % 64 == 0
            and W.shape[0] >= (vocab + 127) // 128 * 128 and W.is_contiguous()):
        return _ChunkedHeadCE.apply(h, W, targets, int(vocab), int(ignore_index), int(chunk))
    from .gemm import LMHeadFunction

    logits = LMHeadFunction.apply(h, W)
    return cross_entropy(logits, targets.reshape(-1), vocab=vocab, ignore_index=ignore_index)

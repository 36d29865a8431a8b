"""Uneven-shard collectives (reference ``src/hetero/varlen_collectives.py:18-94``).

:func:`all_gather_varlen_1d` keeps the reference's contract (lengths are
discovered with a small all-gather, then a padded ``all_gather_into_tensor``).
:func:`all_gather_by_plan` is the form the engine uses: every rank already knows
the plan, so the length exchange is skipped, and the result is assembled into a
caller-provided output with one copy per rank.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .shard_plan import ShardPlan


def _all_gather_int(value: int, *, group=None, device=None) -> List[int]:
    t = torch.tensor([int(value)], dtype=torch.int64, device=device)
    ws = dist.get_world_size(group)
    out = t.new_empty(ws)
    dist.all_gather_into_tensor(out, t, group=group)
    return [int(x) for x in out.tolist()]


def all_gather_varlen_1d(local: torch.Tensor, *, group: Optional[dist.ProcessGroup] = None
                         ) -> Tuple[List[int], torch.Tensor]:
    """All-gather 1-D tensors whose lengths differ per rank.

    Returns ``(lengths, concatenated)``.
    """
    if not dist.is_initialized():
        return [int(local.numel())], local.contiguous()
    if local.dim() != 1:
        raise ValueError("all_gather_varlen_1d requires a 1D tensor")
    local = local.contiguous()
    lengths = _all_gather_int(local.numel(), group=group, device=local.device)
    max_len = max(lengths) if lengths else 0
    if max_len == 0:
        return lengths, local.new_empty((0,))
    send = local
    if local.numel() != max_len:
        send = local.new_zeros((max_len,))
        send[: local.numel()].copy_(local)
    ws = dist.get_world_size(group)
    gathered = local.new_empty((ws * max_len,))
    dist.all_gather_into_tensor(gathered, send, group=group)
    chunks = [gathered[i * max_len: i * max_len + n] for i, n in enumerate(lengths) if n > 0]
    if not chunks:
        return lengths, local.new_empty((0,))
    return lengths, torch.cat(chunks, dim=0)


def all_gather_by_plan(local: torch.Tensor, plan: ShardPlan, *, group=None,
                       out: Optional[torch.Tensor] = None, async_op: bool = False):
    """Gather shards laid out by ``plan`` into ``out`` (``[plan.total]``).

    With ``async_op=True`` returns ``(out, finish)`` where ``finish()`` waits and
    assembles; otherwise returns ``out``.
    """
    total = plan.total
    if out is None:
        out = local.new_empty((total,))
    if not dist.is_initialized() or plan.world_size == 1:
        out.copy_(local.reshape(-1)[:total])
        return (out, lambda: out) if async_op else out
    stride = plan.max_length
    ws = plan.world_size
    rank = dist.get_rank(group)
    if local.numel() != plan.lengths[rank]:
        raise ValueError(f"rank {rank}: local shard has {local.numel()} elements, "
                         f"plan says {plan.lengths[rank]}")
    if all(n == stride for n in plan.lengths):
        work = dist.all_gather_into_tensor(out, local.contiguous(), group=group,
                                           async_op=async_op)
        if async_op:
            def finish_direct():
                work.wait()
                return out
            return out, finish_direct
        return out
    send = local.new_zeros((stride,))
    send[: local.numel()].copy_(local.reshape(-1))
    staging = local.new_empty((ws * stride,))
    work = dist.all_gather_into_tensor(staging, send, group=group, async_op=async_op)

    def finish():
        if async_op:
            work.wait()
        for r in range(ws):
            o, n = plan.offsets[r], plan.lengths[r]
            if n:
                out[o:o + n].copy_(staging[r * stride: r * stride + n])
        return out

    if async_op:
        return out, finish
    return finish()

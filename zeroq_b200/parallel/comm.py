"""Gather paths for sharded parameters.

Two implementations sit behind one handle type:

* ``nccl`` (baseline): one ``all_gather_into_tensor`` per buffer (packed bytes,
  absmax), padded to the plan's largest shard and assembled with one copy per
  rank - ``zeroq_b200.parallel.varlen.all_gather_by_plan``.
* ``fused`` (CUDA, world size > 1, shards registered in the peer pool): the
  sm_100a peer-gather kernel (``csrc/p2p.cu``) reads every rank's shard over
  NVLink straight into the assembled buffer; uneven plans cost nothing extra.

Single-process runs skip communication entirely.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..utils.metrics import count, nvtx_range
from .varlen import all_gather_by_plan


class GatherHandle:
    """Result of an asynchronous gather; ``wait()`` returns the assembled tensors."""

    def __init__(self, finishers):
        self._finishers = finishers
        self._result = None

    def wait(self):
        if self._result is None:
            outs = tuple(f() for f in self._finishers)
            self._result = outs if len(outs) > 1 else outs[0]
            self._finishers = None
        return self._result


def alloc_shard(numel: int, dtype: torch.dtype, device: torch.device, owner=None) -> torch.Tensor:
    """Storage for a parameter's local shard.

    Shards start as ordinary allocations; ``zeroq_b200.parallel.peer.PeerPool``
    later moves every shard of a coordinator into one peer-mapped buffer so the
    fused gather can read it from other GPUs.
    """
    return torch.empty(int(numel), dtype=dtype, device=device)


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def _backend(zq) -> str:
    b = getattr(zq.config, "backend", "auto")
    if b == "auto":
        b = "fused" if zq.local_packed is not None and zq.local_packed.is_cuda else "torch"
    return b


def remote_nf4_bytes(zq) -> int:
    """Bytes of ``zq``'s packed NF4 data and absmax held by the other ranks."""
    p0, p1 = zq.packed_plan.range_of(zq.rank)
    a0, a1 = zq.absmax_plan.range_of(zq.rank)
    return (zq.packed_plan.total - (p1 - p0)) + 4 * (zq.absmax_plan.total - (a1 - a0))


def gather_nf4(zq, group=None, async_op: bool = True) -> GatherHandle:
    """Gather the packed bytes and absmax of ``zq`` according to its plans."""
    if _world(group) == 1 or zq.world_size == 1:
        p, a = zq.local_packed, zq.local_absmax
        return GatherHandle([lambda: p, lambda: a])
    pool = getattr(zq, "_peer_pool", None)
    if _backend(zq) == "fused" and pool is not None:
        with nvtx_range("gather_nf4_peer"):
            return pool.gather(zq)   # (counts its own bytes)
    count("gather_bytes", remote_nf4_bytes(zq))
    with nvtx_range("gather_nf4_nccl"):
        _, fin_p = all_gather_by_plan(zq.local_packed, zq.packed_plan, group=group, async_op=True)
        _, fin_a = all_gather_by_plan(zq.local_absmax, zq.absmax_plan, group=group, async_op=True)
    h = GatherHandle([fin_p, fin_a])
    if not async_op:
        h.wait()
    return h


def gather_master(zq, group=None, async_op: bool = True) -> GatherHandle:
    """Gather the fp32 master shards (ceil split, zero-padded tail)."""
    shard = zq.master_shard.data
    if _world(group) == 1 or zq.world_size == 1:
        return GatherHandle([lambda: shard])
    out = shard.new_empty(shard.numel() * zq.world_size)
    work = dist.all_gather_into_tensor(out, shard.contiguous(), group=group, async_op=True)

    def fin():
        work.wait()
        return out

    h = GatherHandle([fin])
    if not async_op:
        h.wait()
    return h

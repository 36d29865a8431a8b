"""Weighted (heterogeneous) sharding (reference ``src/hetero/zeroq_hetero.py``).

A rank with twice the capacity weight holds twice the packed bytes.  The packed
bytes and the absmax values are split by two independent weighted plans, as in
the reference (:258-270), so a block's bytes and its absmax may live on
different ranks; the gather paths (NCCL baseline and the peer-memory kernel)
address each buffer by its own plan.

* :func:`discover_rank_weights` - env ``ZEROQ_HETERO_RANK_WEIGHTS``, else each
  rank's ``total_memory`` (MB) minus ``activation_reserve_mb`` (floor 1.0),
  else uniform (reference :59-126).
* :class:`HeteroZeroQCoordinator` - adds :meth:`verify_registration_consistency`
  (SHA-256 of the registration list, all-gathered, mismatch raises; :629-669) and
  :meth:`debug_collective_seq` (:713-740).
* :class:`HeteroZeroQModuleWrapper` - registers modules and parameters sorted by
  name so every rank issues collectives in the same order (:765-767).
"""

from __future__ import annotations

import hashlib
import os
from typing import List, Optional

import torch
import torch.distributed as dist

from .coordinator import (ZeroQCoordinator, ZeroQModuleWrapper, ZeroQParameter,
                          ZeroQParamStatus)
from .shard_plan import make_plan

HeteroZeroQParamStatus = ZeroQParamStatus


def _coll_device(group=None) -> torch.device:
    if dist.is_initialized() and dist.get_backend(group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _parse_rank_weights_env(world_size: int) -> Optional[List[float]]:
    raw = os.environ.get("ZEROQ_HETERO_RANK_WEIGHTS")
    if not raw:
        return None
    parts = [p.strip() for p in raw.split(",") if p.strip()]
    if len(parts) != world_size:
        raise ValueError(f"ZEROQ_HETERO_RANK_WEIGHTS expects {world_size} comma-separated "
                         f"values; got {len(parts)}")
    return [float(x) for x in parts]


def discover_rank_weights(*, group: Optional[dist.ProcessGroup] = None,
                          activation_reserve_mb: float = 0.0) -> List[float]:
    """Per-rank capacity weights (larger = more shard)."""
    if not dist.is_initialized():
        return [1.0]
    ws = dist.get_world_size(group)
    env = _parse_rank_weights_env(ws)
    if env is not None:
        return env
    w = 1.0
    if torch.cuda.is_available():
        try:
            props = torch.cuda.get_device_properties(torch.cuda.current_device())
            w = float(props.total_memory) / (1024 ** 2)
        except Exception:
            w = 1.0
    t = torch.tensor([w], dtype=torch.float64, device=_coll_device(group))
    out = t.new_empty(ws)
    dist.all_gather_into_tensor(out, t, group=group)
    raw = [float(x) for x in out.tolist()]
    if not any(v > 0 for v in raw):
        return [1.0] * ws
    if activation_reserve_mb > 0:
        return [max(v - activation_reserve_mb, 1.0) for v in raw]
    return raw


class HeteroZeroQParameter(ZeroQParameter):
    """A :class:`ZeroQParameter` whose shards follow weighted plans."""

    def __init__(self, *, param, rank, world_size, config, param_id, rank_weights=None,
                 module=None, param_name=None, process_group=None):
        super().__init__(param=param, rank=rank, world_size=world_size, config=config,
                         param_id=param_id, module=module, param_name=param_name,
                         process_group=process_group)
        self.rank_weights = list(rank_weights) if rank_weights is not None else [1.0] * world_size

    def _make_plans(self, packed_total: int, absmax_total: int):
        return make_plan(packed_total, self.rank_weights), make_plan(absmax_total, self.rank_weights)


class HeteroZeroQCoordinator(ZeroQCoordinator):
    param_cls = HeteroZeroQParameter

    def __init__(self, config, process_group: Optional[dist.ProcessGroup] = None,
                 rank_weights: Optional[List[float]] = None):
        super().__init__(config, process_group)
        if rank_weights is None:
            rank_weights = discover_rank_weights(
                group=process_group,
                activation_reserve_mb=float(getattr(config, "activation_reserve_mb", 0.0)))
        if len(rank_weights) != self.world_size:
            raise ValueError(f"{len(rank_weights)} rank weights for world size {self.world_size}")
        self.rank_weights = list(rank_weights)

    def _new_param(self, param, module, param_name, param_id):
        return HeteroZeroQParameter(param=param, rank=self.rank, world_size=self.world_size,
                                    config=self.config, param_id=param_id,
                                    rank_weights=self.rank_weights, module=module,
                                    param_name=param_name, process_group=self.process_group)

    def registration_fingerprint(self) -> int:
        entries = [f"{pid}:{tuple(self._params[pid].original_shape)}:"
                   f"{self._params[pid].original_numel}" for pid in sorted(self._params)]
        return int(hashlib.sha256("|".join(entries).encode()).hexdigest()[:15], 16)

    def verify_registration_consistency(self):
        """Raise if any rank registered a different parameter list (which would
        otherwise deadlock the first mismatched collective)."""
        if self.world_size <= 1:
            return
        h = self.registration_fingerprint()
        t = torch.tensor([h], dtype=torch.int64, device=_coll_device(self.process_group))
        out = t.new_empty(self.world_size)
        dist.all_gather_into_tensor(out, t, group=self.process_group)
        hashes = [int(x) for x in out.tolist()]
        if len(set(hashes)) != 1:
            bad = [r for r, v in enumerate(hashes) if v != hashes[0]]
            raise RuntimeError(
                "ZeRO-Q FATAL: Registration order mismatch across ranks!\n"
                f"  Rank 0 hash: {hashes[0]}\n"
                f"  Mismatched ranks: {bad} (hashes: {[hashes[r] for r in bad]})\n"
                f"  Rank {self.rank} registered {len(self._params)} params.\n"
                "  Check that all ranks load the same model with the same LoRA config.")

    def get_memory_stats(self):
        st = super().get_memory_stats()
        st["num_params"] = float(st["num_params"])
        st["rank_weight"] = float(self.rank_weights[self.rank])
        return st

    def collective_seqs(self) -> List[int]:
        if self.world_size <= 1:
            return [self._collective_seq]
        t = torch.tensor([self._collective_seq], dtype=torch.int64,
                         device=_coll_device(self.process_group))
        out = t.new_empty(self.world_size)
        dist.all_gather_into_tensor(out, t, group=self.process_group)
        return [int(x) for x in out.tolist()]

    def debug_collective_seq(self) -> str:
        """All ranks must call together; reports which rank fell behind."""
        seqs = self.collective_seqs()
        if len(seqs) == 1:
            return f"[ZeRO-Q] Single rank, seq={seqs[0]}"
        if len(set(seqs)) == 1:
            return f"[ZeRO-Q] All {len(seqs)} ranks at collective_seq={seqs[0]}"
        lines = ["[ZeRO-Q] COLLECTIVE SEQUENCE MISMATCH - potential deadlock source:"]
        top = max(seqs)
        for r, s in enumerate(seqs):
            lines.append(f"  Rank {r}: seq={s}{' <- BEHIND' if s < top else ''}")
        return "\n".join(lines)


class HeteroZeroQModuleWrapper(ZeroQModuleWrapper):
    sort_registration = True


__all__ = ["HeteroZeroQParameter", "HeteroZeroQCoordinator", "HeteroZeroQModuleWrapper",
           "HeteroZeroQParamStatus", "discover_rank_weights"]

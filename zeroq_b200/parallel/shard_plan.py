"""Shard plans: which rank owns which contiguous range of a flat tensor.

Three split rules are used by the engine:

* :func:`make_plan` - weighted split proportional to per-rank capacity (reference
  ``src/hetero/shard_plan.py:15-93``): floor of the proportional share, then the
  leftover items go one each to the ranks with the largest fractional parts
  (ties to the lower rank).  The rule must stay identical to the reference so a
  hetero checkpoint written by either places the same bytes on the same rank.
* :func:`uniform_remainder_plan` - the uniform coordinator's rule
  (reference ``src/coordinator.py:191-212``): ``total // W`` per rank with the
  remainder on the last rank.
* :func:`ceil_plan` - the fp32 master rule (reference ``src/partition.py:454-482``):
  ``ceil(total / W)`` per rank, the tail rank shorter.

Every plan can be turned into a small int64 table (``plan.table()``) that the
peer-memory gather kernels take as an argument to map a global index to
``(owner rank, local offset)``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch


@dataclass(frozen=True)
class ShardPlan:
    """Per-rank lengths and exclusive-prefix offsets of a contiguous split."""

    lengths: List[int]
    offsets: List[int]

    @property
    def world_size(self) -> int:
        return len(self.lengths)

    @property
    def total(self) -> int:
        return sum(self.lengths)

    @property
    def max_length(self) -> int:
        return max(self.lengths) if self.lengths else 0

    def range_of(self, rank: int) -> Tuple[int, int]:
        o = self.offsets[rank]
        return o, o + self.lengths[rank]

    def owner_of(self, index: int) -> Tuple[int, int]:
        """``(rank, local_offset)`` of global element ``index``."""
        if index < 0 or index >= self.total:
            raise IndexError(index)
        for r in range(self.world_size):
            o, e = self.range_of(r)
            if o <= index < e:
                return r, index - o
        raise IndexError(index)  # pragma: no cover

    def table(self, device=None) -> torch.Tensor:
        """int64 ``[W+1]`` boundaries: rank r owns ``[t[r], t[r+1])``."""
        t = list(self.offsets) + [self.total]
        return torch.tensor(t, dtype=torch.int64, device=device)


def prefix_sums(lengths: List[int]) -> List[int]:
    out, acc = [], 0
    for n in lengths:
        out.append(acc)
        acc += int(n)
    return out if out else [0]


def compute_weighted_shard_lengths(total: int, weights: List[float]) -> List[int]:
    """Split ``total`` items proportionally to ``weights`` (largest-remainder rounding)."""
    total = int(total)
    if total < 0:
        raise ValueError("total must be >= 0")
    if not weights:
        raise ValueError("weights must be non-empty")
    ws = [float(w) for w in weights]
    if any(w < 0 for w in ws):
        raise ValueError("weights must be >= 0")
    s = sum(ws)
    if s <= 0:
        ws = [1.0] * len(ws)
        s = float(len(ws))
    shares = [total * (w / s) for w in ws]
    lengths = [int(x) for x in shares]
    left = total - sum(lengths)
    # rank order: larger fractional part first; equal fractions -> lower rank first
    order = sorted(range(len(ws)), key=lambda i: (-(shares[i] - lengths[i]), i))
    for k in range(left):
        lengths[order[k]] += 1
    return lengths


def make_plan(total: int, weights: List[float]) -> ShardPlan:
    lengths = compute_weighted_shard_lengths(total, weights)
    plan = ShardPlan(lengths=lengths, offsets=prefix_sums(lengths))
    if sum(plan.lengths) != int(total):
        raise AssertionError("lengths do not sum to total")
    return plan


def uniform_remainder_plan(total: int, world_size: int) -> ShardPlan:
    per = total // world_size
    rem = total % world_size
    lengths = [per] * world_size
    lengths[-1] += rem
    return ShardPlan(lengths=lengths, offsets=prefix_sums(lengths))


def ceil_plan(total: int, world_size: int) -> ShardPlan:
    chunk = (total + world_size - 1) // world_size
    lengths = []
    for r in range(world_size):
        s = min(r * chunk, total)
        e = min(s + chunk, total)
        lengths.append(e - s)
    return ShardPlan(lengths=lengths, offsets=prefix_sums(lengths))

"""Step metrics and tracing: NVTX ranges, byte counters, a per-step JSONL writer.

The reference's production trainer prints tokens/s, loss and diagnostics per
step (``examples/train_32b_maxwell.py:744-746,806-947``).  Here:

* :func:`nvtx_range` marks layers, gathers and gradient syncs for a profiler
  timeline (NVTX ranges; off unless ``ZEROQ_NVTX=1`` or :func:`set_nvtx`, so the
  hot path pays nothing by default);
* :data:`counters` accumulate bytes moved by the gather paths (``gather_bytes``:
  bytes read from other ranks' shards) and the gradient syncs
  (``sync_bytes``), so a step can report what it moved;
* :class:`StepLogger` writes one JSON line per training step on rank 0: step,
  loss, device-timed step milliseconds and tokens/s (CUDA events, the max over
  ranks), bytes gathered and synced, and the model-FLOP fraction of a peak.
  Events are read back in batches (``flush_every`` steps), so logging adds no
  per-step host synchronisation.
"""

from __future__ import annotations

import contextlib
import json
import os
from collections import defaultdict
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

_NVTX = os.environ.get("ZEROQ_NVTX", "0") == "1"

counters: Dict[str, int] = defaultdict(int)


def set_nvtx(enabled: bool) -> None:
    global _NVTX
    _NVTX = bool(enabled)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def nvtx_range(name: str):
    """An NVTX range around the block when tracing is on (no-op otherwise)."""
    if not _NVTX or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def count(name: str, n: int) -> None:
    counters[name] += int(n)


def reset_counters() -> None:
    counters.clear()


def snapshot() -> Dict[str, int]:
    return dict(counters)


class StepLogger:
    """Per-step JSONL metrics (rank 0 writes; every rank takes part in the max).

    ``begin()`` / ``end(loss, tokens)`` bracket one step on the current stream;
    every ``flush_every`` steps the recorded events are resolved, the step times
    are max-reduced over ranks in one collective, and one line per step is
    appended to ``path``.  ``tokens`` is this rank's token count for the step;
    tokens/s is computed over all ranks.
    """

    def __init__(self, path: Optional[str], flush_every: int = 10,
                 flops_per_token: Optional[float] = None, peak_tflops: Optional[float] = None,
                 process_group=None):
        self.path = path
        self.flush_every = max(1, int(flush_every))
        self.fpt = flops_per_token
        self.peak = peak_tflops
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self._pending: List[tuple] = []
        self._step = 0
        self._start = None
        self._mark = {}
        self.records: List[dict] = []

    def begin(self) -> None:
        self._start = torch.cuda.Event(enable_timing=True)
        self._start.record()
        self._mark = snapshot()

    def end(self, loss: torch.Tensor, tokens: int) -> None:
        if self._start is None:
            raise RuntimeError("StepLogger.end() without begin()")
        stop = torch.cuda.Event(enable_timing=True)
        stop.record()
        now = snapshot()
        moved = {k: now.get(k, 0) - self._mark.get(k, 0) for k in ("gather_bytes", "sync_bytes")}
        self._pending.append((self._step, self._start, stop, loss.detach().float().reshape(1),
                              int(tokens), moved))
        self._step += 1
        self._start = None
        if len(self._pending) >= self.flush_every:
            self.flush()

    def flush(self) -> List[dict]:
        if not self._pending:
            return []
        dev = self._pending[0][3].device
        torch.cuda.synchronize(dev)
        vals = torch.tensor([[p[1].elapsed_time(p[2]) for p in self._pending]],
                            dtype=torch.float64, device=dev)
        if self.world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX, group=self.pg)
        losses = torch.cat([p[3] for p in self._pending]).cpu().tolist()
        out = []
        for (step, _, _, _, tok, moved), ms, loss in zip(self._pending, vals[0].tolist(), losses):
            tps = tok * self.world / (ms / 1e3) if ms > 0 else 0.0
            rec = {"step": step, "loss": loss, "ms": round(ms, 3), "tokens_per_s": round(tps, 1),
                   "gather_bytes": moved["gather_bytes"], "sync_bytes": moved["sync_bytes"]}
            if self.fpt is not None and self.peak:
                rec["model_tflops_per_gpu"] = round(self.fpt * tps / self.world / 1e12, 3)
                # (6 decimals: small models sit far below a B200's peak)
                rec["frac_of_peak"] = round(self.fpt * tps / self.world / 1e12 / self.peak, 6)
            out.append(rec)
        self._pending = []
        self.records.extend(out)
        if self.rank == 0 and self.path:
            with open(self.path, "a") as f:
                for rec in out:
                    f.write(json.dumps(rec) + "\n")
        return out

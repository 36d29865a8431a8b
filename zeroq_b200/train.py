"""Training loop pieces: the step API, synthetic data, device timing, clock sampling.

:class:`Trainer` is the public step call of this framework:
``loss = trainer.step(input_ids, targets)`` copies the batch host -> device
(pinned, non-blocking), runs forward (fused cross-entropy), backward, the
optimizer (reduce-scatter + AdamW across ranks), and returns the loss as a
Python float (one device -> host read).  ``step_device`` is the same step with
device-resident inputs and the loss left on the device.

``Trainer(..., logger=StepLogger(path))`` (``zeroq_b200.utils.metrics``) writes one
JSON line per step on rank 0: loss, device-timed milliseconds and tokens/s (max
over ranks), bytes gathered and synced, model-FLOP fraction of a peak.

The reference's production trainer adds all-ranks-agree checks before each
collective so a non-finite loss on one rank cannot desynchronise the others
(``examples/train_32b_maxwell.py:522-547``); :meth:`Trainer.all_ranks_finite`
provides that check.
"""

from __future__ import annotations

import json
import os
import subprocess
import threading
import time
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


class Trainer:
    def __init__(self, model: torch.nn.Module, optimizer, device: torch.device,
                 process_group=None, logger=None):
        self.model = model
        self.logger = logger
        self.opt = optimizer
        self.device = device
        self.pg = process_group
        self._in = None
        self._tg = None
        self._graph_on = False
        self._graph = None
        self._graph_bytes = {}
        self.graph_launches = 0   # this framework's kernels in one captured step

    def enable_cuda_graph(self):
        """Run every later step as one CUDA graph replay (the whole forward,
        backward and optimizer step: no per-kernel launch gaps).  The first step
        after this call runs eagerly on the capture stream (allocating per-stream
        state) and then captures the step; it counts as one training step.  Needs
        fixed input shapes and an optimizer with a device-side clock
        (:meth:`~zeroq_b200.parallel.optimizer.ShardedAdamW.use_device_clock`)."""
        if not hasattr(self.opt, "use_device_clock"):
            raise RuntimeError("CUDA-graph steps need ShardedAdamW (device-side optimizer clock)")
        self.opt.use_device_clock()
        self._graph_on = True

    def _eager(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        loss = self.model(input_ids, targets)
        if hasattr(self.opt, "arm_overlap"):   # one backward per step: sync buckets may start
            self.opt.arm_overlap()
        loss.backward()
        self.opt.step()
        pack = getattr(self.model, "pack_lora_operands", None)
        if pack is not None:   # every adapter's bf16 operands in one launch
            pack()
        self.opt.zero_grad()
        return loss.detach()

    def _capture(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        from .ops._ext import LaunchCounter

        self._gin = input_ids.clone()
        self._gtg = targets.clone()
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            loss = self._eager(self._gin, self._gtg)   # this call's step
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        from .utils.metrics import snapshot

        graph = torch.cuda.CUDAGraph()
        before = snapshot()
        with LaunchCounter() as lc:
            with torch.cuda.graph(graph, stream=stream):
                self._gloss = self._eager(self._gin, self._gtg)
        after = snapshot()
        self._graph_bytes = {k: after[k] - before.get(k, 0) for k in after
                             if after[k] != before.get(k, 0)}
        self.graph_launches = lc.count
        self._graph = graph
        return loss

    def _buffers(self, shape):
        if self._in is None or self._in.shape != shape:
            self._in = torch.empty(shape, dtype=torch.int64, device=self.device)
            self._tg = torch.empty(shape, dtype=torch.int64, device=self.device)
        return self._in, self._tg

    def step_device(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        if self.logger is None:
            return self._step_device(input_ids, targets)
        self.logger.begin()
        loss = self._step_device(input_ids, targets)
        self.logger.end(loss, input_ids.numel())
        return loss

    def _step_device(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        from .utils.metrics import nvtx_range

        if not self._graph_on:
            with nvtx_range("train_step"):
                return self._eager(input_ids, targets)
        if self._graph is None:
            return self._capture(input_ids, targets)
        if input_ids.data_ptr() != self._gin.data_ptr():
            self._gin.copy_(input_ids, non_blocking=True)
            self._gtg.copy_(targets, non_blocking=True)
        self._graph.replay()
        if self._graph_bytes:   # a replay moves what the captured step moved
            from .utils.metrics import count

            for k, v in self._graph_bytes.items():
                count(k, v)
        return self._gloss

    def step(self, input_ids_host: torch.Tensor, targets_host: torch.Tensor) -> float:
        if self._graph is not None:  # straight into the graph's static inputs
            self._gin.copy_(input_ids_host, non_blocking=True)
            self._gtg.copy_(targets_host, non_blocking=True)
            return float(self.step_device(self._gin, self._gtg).item())
        dev_in, dev_tg = self._buffers(input_ids_host.shape)
        dev_in.copy_(input_ids_host, non_blocking=True)
        dev_tg.copy_(targets_host, non_blocking=True)
        loss = self.step_device(dev_in, dev_tg)
        return float(loss.item())

    def all_ranks_finite(self, value: torch.Tensor) -> bool:
        ok = torch.isfinite(value).all().to(torch.int32).reshape(1)
        if dist.is_initialized() and dist.get_world_size(self.pg) > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.pg)
        return bool(ok.item())


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, pinned: bool = True
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Uniform random token ids; targets are the next token (last position wraps)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=g, dtype=torch.int64)
    x, y = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
    if pinned and torch.cuda.is_available():
        x, y = x.pin_memory(), y.pin_memory()
    return x, y


class ClockSampler:
    """Samples ``nvidia-smi`` SM clocks and throttle reasons while active."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 200, log_path: Optional[str] = None):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.log_path = log_path
        self.proc = None
        self.lines: List[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()
            self._t.join(timeout=2)
        if self.log_path:
            with open(self.log_path, "a") as f:
                f.write("\n".join(self.lines) + "\n")
        return False

    def summary(self) -> dict:
        mhz, max_mhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        mhz.sort()
        loaded = [m for m in mhz if max_mhz is None or m > 0.3 * max_mhz] or mhz
        return {"sm_mhz": loaded[len(loaded) // 2], "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz)}


def device_time_ms(fn, steps: int, sync_group=None) -> float:
    """Run ``fn`` ``steps`` times between CUDA events; barrier + synchronize on both sides.
    Returns the max over ranks of the elapsed milliseconds."""
    if dist.is_initialized():
        dist.barrier(group=sync_group)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier(group=sync_group)
    ms = torch.tensor([start.elapsed_time(end)], dtype=torch.float64,
                      device=torch.device("cuda", torch.cuda.current_device()))
    if dist.is_initialized():
        dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=sync_group)
    return float(ms.item())

"""Flat-buffer optimizers for the trainable surface (LoRA adapters, norms).

:class:`FlatParams` moves a list of fp32 parameters into one contiguous fp32
buffer (each parameter becomes a view of it) and pre-assigns every ``.grad`` as
a view of one contiguous gradient buffer; autograd accumulates into those views
in place.  One kernel launch then updates every parameter, and one collective
moves every gradient.

:class:`ShardedAdamW` is the data-parallel AdamW of the reference's training
loops (``examples/train_32b_maxwell.py:472-475`` all-reduces each LoRA grad,
then steps torch's AdamW), restructured ZeRO-style:

* world size 1: one fused AdamW kernel over the flat buffer;
* world size W, backend ``nccl``: one ``reduce_scatter_tensor`` of the flat
  gradient, AdamW on this rank's 1/W shard (moments are sharded too, with the
  1/W averaging folded into the kernel's ``grad_scale``), one
  ``all_gather_into_tensor`` of the updated shard;
* backend ``fused``: the same three steps with the reduce-scatter done by the
  peer-memory kernel of ``zeroq_b200.parallel.peer`` (it sums the peers' slices
  over NVLink and applies AdamW in the same pass).

Optional global-norm gradient clipping (``max_grad_norm``, as
``torch.nn.utils.clip_grad_norm_`` in the reference's trainer) is computed on
the device: the squared norm of the averaged gradient is summed (over NVLink for
the fused backend, then one scalar all-reduce) and the update kernels read it
and scale by ``min(1, max_norm / norm)`` themselves - no host synchronisation,
so clipped steps also run as CUDA graph replays.
"""

from __future__ import annotations

import math
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist

from ..ops.optim import adamw_step
from ..utils.metrics import count, nvtx_range


class FlatParams:
    """``alloc(numel, dtype, role)`` (role ``"data"`` then ``"grad"``) may place the
    buffers elsewhere, e.g. in peer memory for the fused optimizer.

    ``groups`` (lists of parameters, together exactly ``params``): lay the
    parameters out group by group, each group padded to a multiple of ``pad_to``;
    ``group_ranges[k]`` is group k's ``[start, end)`` in the buffer."""

    def __init__(self, params: Iterable[torch.nn.Parameter], pad_to: int = 1, device=None,
                 alloc=None, groups: Optional[List[List[torch.nn.Parameter]]] = None):
        self.params: List[torch.nn.Parameter] = [p for p in params]
        if not self.params:
            raise ValueError("FlatParams needs at least one parameter")
        for p in self.params:
            if p.dtype != torch.float32:
                raise TypeError(f"FlatParams holds fp32 parameters; got {p.dtype}")
        device = device or self.params[0].device
        self.numel = sum(p.numel() for p in self.params)
        if groups is None:
            groups = [self.params]
        if sorted(id(p) for g in groups for p in g) != sorted(id(p) for p in self.params):
            raise ValueError("FlatParams groups must hold every parameter exactly once")
        self.params = [p for g in groups for p in g]
        starts, off = [], 0
        self.group_ranges = []
        for g in groups:
            n = sum(p.numel() for p in g)
            end = off + (n + pad_to - 1) // pad_to * pad_to
            self.group_ranges.append((off, end))
            starts += [off + sum(q.numel() for q in g[:i]) for i in range(len(g))]
            off = end
        self.padded = off
        if alloc is None:
            self.data = torch.zeros(self.padded, dtype=torch.float32, device=device)
            self.grad = torch.zeros(self.padded, dtype=torch.float32, device=device)
        else:
            self.data = alloc(self.padded, torch.float32, "data")
            self.grad = alloc(self.padded, torch.float32, "grad")
        self.offsets = []
        with torch.no_grad():
            for p, off in zip(self.params, starts):
                n = p.numel()
                self.data[off:off + n].copy_(p.data.reshape(-1))
                p.data = self.data[off:off + n].view(p.shape)
                p.grad = self.grad[off:off + n].view(p.shape)
                # layers may accumulate this parameter's gradient in place into
                # the bound fp32 .grad instead of returning it to autograd
                p._zq_flat_grad = True
                self.offsets.append(off)

    def zero_grad(self):
        self.grad.zero_()
        # autograd may have replaced a .grad (e.g. after a set_to_none elsewhere): rebind
        for p, off in zip(self.params, self.offsets):
            if p.grad is None or p.grad.data_ptr() != self.grad[off:].data_ptr():
                p.grad = self.grad[off:off + p.numel()].view(p.shape)

    def mark_updated(self):
        """Bump every parameter's version counter after the buffers were written by
        kernels (caches keyed on ``_version`` then see the update)."""
        torch.autograd.graph.increment_version(self.params)

    def grads_bound(self) -> bool:
        return all(p.grad is not None and p.grad.data_ptr() == self.grad[off:].data_ptr()
                   for p, off in zip(self.params, self.offsets))


class ShardedAdamW:
    """AdamW over a :class:`FlatParams`, data-parallel across the process group."""

    def __init__(self, params, lr: float = 1e-4, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, process_group: Optional[dist.ProcessGroup] = None,
                 backend: str = "auto", max_grad_norm: Optional[float] = None,
                 broadcast_initial: bool = True,
                 overlap_buckets: Optional[List[List[torch.nn.Parameter]]] = None,
                 overlap_ctas: int = 32):
        """``broadcast_initial``: start every rank from rank 0's parameters (one
        broadcast of the flat buffer), as data-parallel training requires - layers
        initialise adapters from each process's own random state (LoRA ``A``), and
        the sharded update only keeps replicas equal if they start equal.

        ``overlap_buckets`` (fused backend, several ranks, no clipping): groups of
        parameters whose gradients are final together, e.g. one decoder layer's.
        Each group becomes a contiguous bucket of the flat buffer; after
        :meth:`arm_overlap`, :meth:`bucket_ready` (called from a backward hook once a
        group's gradients are written) launches that bucket's reduce-scatter + AdamW
        + all-gather kernel on a side stream, ``overlap_ctas`` CTAs wide, while the
        backward continues; :meth:`step` launches the rest and joins the streams.
        Every bucket kernel of a rank runs on that one stream in the same order on
        every rank: each kernel's closing barrier is what lets the next one reuse
        the cross-rank flags.  (Clipping needs the global norm before any update,
        so it keeps the single step-end launch.)"""
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        params = list(params)
        on_cuda = bool(params) and params[0].is_cuda
        if backend == "auto":
            backend = "fused" if on_cuda and self.world > 1 else "nccl"
        alloc = None
        self._peer_error = None
        if backend == "fused" and self.world > 1:
            try:
                from .peer import peer_flat_allocator

                alloc = peer_flat_allocator(process_group)
            except Exception as e:  # no IPC / extension: NCCL path
                self._peer_error = repr(e)
                backend = "nccl"
        groups = None
        self._bucket_of = {}
        if (overlap_buckets is not None and alloc is not None and self.world > 1
                and max_grad_norm is None):
            ids = {id(p) for p in params}
            seen = set()
            groups = []
            for i, g in enumerate(overlap_buckets):
                g2 = [p for p in g if id(p) in ids and id(p) not in seen]
                if g2:
                    seen.update(id(p) for p in g2)
                    self._bucket_of[i] = len(groups)
                    groups.append(g2)
            rest = [p for p in params if id(p) not in seen]
            if rest:
                groups.append(rest)
        # pad so that every rank's shard (of every bucket) is a whole number of
        # 16-byte vectors
        self.flat = FlatParams(params, pad_to=self.world * 4, alloc=alloc, groups=groups)
        if broadcast_initial and self.world > 1:
            src = dist.get_global_rank(process_group, 0) if process_group is not None else 0
            dist.broadcast(self.flat.data, src=src, group=process_group)
            self.flat.mark_updated()
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.shard = self.flat.padded // self.world
        dev = self.flat.data.device
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.grad_shard = torch.zeros(self.shard, dtype=torch.float32, device=dev) \
            if self.world > 1 else None
        self.step_count = 0
        self.backend = backend
        self._peer = getattr(self.flat.grad, "_zq_peer", None) if backend == "fused" else None
        if backend == "fused" and self._peer is None:
            self.backend = "nccl"
        self.last_grad_norm: Optional[torch.Tensor] = None
        self._sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.device_clock = None   # (clk int64 [step, epoch], bc fp32 [2]) once enabled
        # bucket k: this rank's part [lo, lo + n) of the flat buffer and its offset
        # in the moment tensors (one bucket = the whole buffer without overlap)
        self._parts = []
        moff = 0
        for start, end in self.flat.group_ranges:
            n = (end - start) // self.world
            self._parts.append((start + self.rank * n, n, moff))
            moff += n
        self.overlap = (groups is not None and len(self._parts) > 1 and self.backend == "fused"
                        and self._peer is not None)
        if len(self._parts) > 1 and not self.overlap:   # (the other paths take one shard)
            raise RuntimeError("bucketed flat layout without the fused overlap path")
        self.overlap_ctas = int(overlap_ctas)
        self._comm = torch.cuda.Stream(device=dev) if self.overlap else None
        self._armed = False
        self._launched: List[int] = []
        self._begun = False

    def use_device_clock(self):
        """Keep the step count, the bias corrections and (fused backend) the
        cross-rank barrier epoch on the device, advanced by a kernel at the start of
        every step, so a CUDA graph that captured a step replays it correctly."""
        if self.device_clock is not None:
            return
        dev = self.flat.data.device
        epoch = self._peer.flags.epoch if self._peer is not None else 0
        clk = torch.tensor([self.step_count, epoch], dtype=torch.int64, device=dev)
        bc = torch.ones(2, dtype=torch.float32, device=dev)
        self.device_clock = (clk, bc)

    def _tick(self):
        from ..ops import _ext

        b1, b2 = self.betas
        clk, bc = self.device_clock
        _ext.ext().opt_tick(clk, bc, float(b1), float(b2), self._peer is not None)

    @property
    def params(self):
        return self.flat.params

    # -- gradient sync overlapped with the backward (fused backend) ------------------
    def arm_overlap(self):
        """Let :meth:`bucket_ready` launch buckets during the coming backward (call
        once per step, before the step's only backward)."""
        if self.overlap:
            self._armed = True

    def bucket_ready(self, i: int):
        """Group ``i`` of ``overlap_buckets`` has its final gradients (on the current
        stream): launch its bucket on the side stream."""
        if not (self.overlap and self._armed):
            return
        k = self._bucket_of.get(i)
        if k is not None and k not in self._launched:
            self._launch([k])

    def _launch(self, ks):
        cur = torch.cuda.current_stream(self.flat.data.device)
        self._comm.wait_stream(cur)
        with torch.cuda.stream(self._comm):
            if not self._begun:
                self._begin_step()
            b1, b2 = self.betas
            nb = len(self._parts)
            for k in ks:
                lo, n, moff = self._parts[k]
                # epochs: one per launch, in launch order (device clock: clk * nb + i)
                epoch = (nb, len(self._launched)) if self.device_clock is not None else None
                with nvtx_range(f"grad_sync_bucket{k}"):
                    self._peer.run(lo, n, self.exp_avg[moff:moff + n], self.exp_avg_sq[moff:moff + n],
                                   lr=self.lr, beta1=b1, beta2=b2, eps=self.eps,
                                   weight_decay=self.wd, step=self.step_count,
                                   grad_scale=1.0 / self.world, push=True,
                                   clock=self.device_clock, epoch=epoch, max_ctas=self.overlap_ctas)
                self._launched.append(k)

    def _begin_step(self):
        self.step_count += 1
        if self.device_clock is not None:
            self._tick()
        self._begun = True

    def _step_overlap(self):
        self._armed = False
        count("sync_bytes", 4 * self.flat.padded)
        rest = [k for k in range(len(self._parts)) if k not in self._launched]
        self._launch(rest)
        torch.cuda.current_stream(self.flat.data.device).wait_stream(self._comm)
        self._launched = []
        self._begun = False

    def zero_grad(self, set_to_none: bool = False):
        self.flat.zero_grad()

    def _clip_sq(self, g: Optional[torch.Tensor] = None, scale: float = 1.0) -> Optional[torch.Tensor]:
        """Squared global norm of the averaged gradient on the device (None without
        clipping): the kernels scale by ``min(1, max_norm / norm)`` themselves, so
        clipping costs no host synchronisation (and runs inside CUDA graphs).
        ``g``: this rank's part of the averaged gradient times ``1/scale``."""
        if self.max_grad_norm is None:
            return None
        if g is not None:
            sq = (g.float() * scale).pow(2).sum().reshape(1)
            if self.world > 1:
                dist.all_reduce(sq, group=self.pg)
        else:  # fused backend: the shard is summed over NVLink by rs_sumsq
            sq = self._sq
            sq.zero_()
            lo = self.rank * self.shard
            self._peer.sumsq(self, lo, sq)
            dist.all_reduce(sq, group=self.pg)
        self.last_grad_norm = sq  # squared; see grad_norm()
        return sq

    def grad_norm(self) -> Optional[float]:
        """Global L2 norm of the last clipped gradient (host read; call outside the
        hot loop)."""
        if self.last_grad_norm is None:
            return None
        return float(self.last_grad_norm.sqrt().item())

    @torch.no_grad()
    def step(self):
        self._step()
        self.flat.mark_updated()

    def _step(self):
        if self.overlap:
            self._step_overlap()
            return
        self.step_count += 1
        b1, b2 = self.betas
        bc_dev = None
        if self.device_clock is not None:
            self._tick()
            bc_dev = self.device_clock[1]
        if self.world == 1:
            sq = self._clip_sq(self.flat.grad)
            adamw_step(self.flat.data, self.flat.grad, self.exp_avg, self.exp_avg_sq, lr=self.lr,
                       beta1=b1, beta2=b2, eps=self.eps, weight_decay=self.wd,
                       step=self.step_count, bc_dev=bc_dev, clip_sq=sq,
                       max_norm=self.max_grad_norm or 0.0)
            return
        lo = self.rank * self.shard
        mine = self.flat.data[lo:lo + self.shard]
        count("sync_bytes", 4 * self.flat.padded)
        if self.backend == "fused":
            with nvtx_range("grad_sync_fused"):
                # one kernel: peers' gradient slices summed over NVLink, AdamW, and the
                # updated shard written into every peer's parameter buffer (with
                # clipping, a sum-of-squares pass over the same slices comes first)
                sq = self._clip_sq()
                self._peer.reduce_scatter_adamw(self, mine, clip_sq=sq)
            return
        dist.reduce_scatter_tensor(self.grad_shard, self.flat.grad, op=dist.ReduceOp.SUM,
                                   group=self.pg)
        sq = self._clip_sq(self.grad_shard, 1.0 / self.world)
        adamw_step(mine, self.grad_shard, self.exp_avg, self.exp_avg_sq, lr=self.lr,
                   beta1=b1, beta2=b2, eps=self.eps, weight_decay=self.wd,
                   step=self.step_count, grad_scale=1.0 / self.world, bc_dev=bc_dev, clip_sq=sq,
                   max_norm=self.max_grad_norm or 0.0)
        # NCCL gathers in place when the input is this rank's slice of the output;
        # other backends get a private copy of the shard.
        src = mine if self.flat.data.is_cuda else mine.clone()
        dist.all_gather_into_tensor(self.flat.data, src, group=self.pg)

    def state_dict(self) -> dict:
        if self.device_clock is not None:   # replays advance only the device clock
            self.step_count = int(self.device_clock[0][0])
        return {"step": self.step_count, "exp_avg": self.exp_avg.detach().cpu(),
                "exp_avg_sq": self.exp_avg_sq.detach().cpu(), "lr": self.lr,
                "betas": self.betas, "eps": self.eps, "weight_decay": self.wd,
                "world": self.world, "rank": self.rank, "shard": self.shard,
                "buckets": [list(r) for r in self.flat.group_ranges]}

    def load_state_dict(self, st: dict):
        if st["shard"] != self.shard:
            raise ValueError("optimizer shard size differs (different world size or params)")
        if "buckets" in st and [tuple(r) for r in st["buckets"]] != list(self.flat.group_ranges):
            raise ValueError("optimizer bucket layout differs (overlap_buckets changed)")
        self.step_count = int(st["step"])
        if self.device_clock is not None:
            self.device_clock[0][0] = self.step_count
        self.exp_avg.copy_(st["exp_avg"])
        self.exp_avg_sq.copy_(st["exp_avg_sq"])

"""Peer memory over NVLink / NVSwitch: IPC-shared buffers and the kernels that use them.

:class:`PeerBuffer` is one ``cudaMalloc`` allocation per rank, opened on every
other rank of the node through CUDA IPC handles that are exchanged once over
the process group.  The kernels in ``csrc/p2p.cu`` then read and write peers'
buffers with ordinary loads and stores.

* :class:`PeerReduceScatterAdamW` - the optimizer path of
  :class:`~zeroq_b200.parallel.optimizer.ShardedAdamW` with ``backend="fused"``:
  one kernel per rank sums every peer's gradient slice of its shard, scales by
  1/W, applies AdamW, and writes the updated shard into every peer's parameter
  buffer (reduce-scatter + update + all-gather in one pass).  It replaces the
  reference's per-tensor NCCL all-reduce + torch AdamW
  (``examples/train_32b_maxwell.py:472-475``, ``src/gradient_sync.py:489-532``).
* :class:`PeerShardPool` - holds every NF4 shard of a coordinator in one peer
  buffer per rank; ``gather(zq)`` assembles a parameter's packed bytes and absmax
  straight from the owners' buffers by their shard plans (uniform or weighted),
  with no padding, staging or unpad copies (reference
  ``src/coordinator.py:385-533``, ``src/hetero/zeroq_hetero.py:312-452``), and
  ``gather_dequant(zq)`` additionally expands to the bf16 GEMM operand in the
  same kernel, and ``ag_gemm(zq, x)`` runs gather, dequantise and the tcgen05
  GEMM ``x Wᵀ`` as ONE kernel (:func:`ag_gemm_pieces`).
* :class:`PeerMasterPool` - the fp32 master shards of a train-from-scratch
  coordinator in one peer buffer per rank (the optimizer updates them in place);
  ``ag_gemm(zq, x)`` gathers the masters, casts them to bf16 and multiplies in
  one kernel, replacing the reference's fp32 all-gather before the layer
  (``src/coordinator.py:606-611``).

Cross-rank synchronisation is by epoch flags with bounded waits; a timeout
leaves an error code that :meth:`PeerFlags.check` raises on the host.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..ops import _ext


def _group_info(group):
    return dist.get_rank(group), dist.get_world_size(group)


class PeerBuffer:
    """A device buffer of ``nbytes`` on every rank, mapped into every rank."""

    def __init__(self, nbytes: int, group=None):
        E = _ext.ext()
        self.group = group
        self.rank, self.world = _group_info(group)
        self.nbytes = max(16, (int(nbytes) + 255) // 256 * 256)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.local_ptr = int(E.peer_alloc(self.nbytes)[0])
        handle = bytes(E.peer_handle(self.local_ptr).numpy().tobytes())
        handles: List[bytes] = [b""] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs: List[int] = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.ptrs.append(self.local_ptr)
            else:
                t = torch.frombuffer(bytearray(h), dtype=torch.uint8)
                self.ptrs.append(int(E.peer_open(t)))
        self._closed = False

    def tensor(self, numel: int, dtype: torch.dtype, byte_offset: int = 0) -> torch.Tensor:
        esz = torch.empty(0, dtype=dtype).element_size()
        if byte_offset % esz or byte_offset + numel * esz > self.nbytes:
            raise ValueError("view outside the peer buffer")
        return _ext.ext().tensor_from_ptr(self.local_ptr + byte_offset, numel, dtype,
                                          self.device.index)

    def close(self):
        if self._closed:
            return
        E = _ext.ext()
        torch.cuda.synchronize()
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                E.peer_close(p)
        E.peer_free(self.local_ptr)
        self._closed = True


class PeerFlags(PeerBuffer):
    """Flag words for the cross-rank barriers of the peer kernels."""

    def __init__(self, group=None):
        super().__init__(4 * int(_ext.ext().peer_flag_words()), group)
        self.epoch = 0

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def check(self):
        code, detail = _ext.ext().peer_status_read(self.local_ptr)
        if code:
            raise RuntimeError(f"peer collective on rank {self.rank} failed: code {code} "
                               f"(detail {detail}); a peer did not arrive within the wait limit")


class PeerReduceScatterAdamW:
    """Fused reduce-scatter + AdamW + all-gather over peer memory."""

    def __init__(self, grad_buf: PeerBuffer, param_buf: PeerBuffer, flags: PeerFlags,
                 grad_is_bf16: bool = False):
        self.grad_buf, self.param_buf, self.flags = grad_buf, param_buf, flags
        self.grad_is_bf16 = grad_is_bf16

    @classmethod
    def create(cls, flat_grad: torch.Tensor, group):
        owner = getattr(flat_grad, "_zq_peer", None)
        if owner is None:
            raise RuntimeError("flat gradient is not in peer memory")
        return owner

    def run(self, lo: int, n: int, m: torch.Tensor, v: torch.Tensor, *, lr, beta1, beta2, eps,
            weight_decay, step, grad_scale, push: bool = True, timeout_ms: int = 0,
            clock=None, clip_sq: Optional[torch.Tensor] = None, max_norm: float = 0.0,
            epoch: Optional[tuple] = None, max_ctas: int = 0):
        """``clock = (clk, bc)``: take the barrier epoch and the bias corrections from
        the device-side optimizer clock (see :meth:`ShardedAdamW.use_device_clock`)
        instead of launch arguments.  ``clip_sq``: squared global gradient norm on
        the device (:meth:`sumsq` + all-reduce); the kernel clips to ``max_norm``.
        A clipped step runs two peer kernels, on epochs ``2e`` and ``2e + 1`` of the
        device clock; ``epoch = (mul, add)`` sets that pair for other schedules
        (``k`` launches per step: ``(k, i)`` for the i-th).  ``max_ctas`` caps the
        grid (a launch beside compute kernels)."""
        bc1 = 1.0 - beta1 ** step
        bc2 = 1.0 - beta2 ** step
        mul, add = (2, 1) if clip_sq is not None else (1, 0)
        if epoch is not None:
            mul, add = epoch
        if clock is not None:
            _ext.ext().rs_adamw_dev(self.grad_buf.ptrs, self.param_buf.ptrs, self.flags.ptrs,
                                    self.flags.rank, 0, int(lo), int(n), m, v,
                                    1 if self.grad_is_bf16 else 0, float(lr), float(beta1),
                                    float(beta2), float(eps), float(weight_decay), 1.0, 1.0,
                                    float(grad_scale), bool(push), int(timeout_ms), clock[0], clock[1],
                                    clip_sq, float(max_norm), mul, add, int(max_ctas))
            return
        _ext.ext().rs_adamw_dev(self.grad_buf.ptrs, self.param_buf.ptrs, self.flags.ptrs,
                                self.flags.rank, self.flags.next_epoch(), int(lo), int(n), m, v,
                                1 if self.grad_is_bf16 else 0, float(lr), float(beta1), float(beta2),
                                float(eps), float(weight_decay), float(bc1), float(bc2),
                                float(grad_scale), bool(push), int(timeout_ms), None, None,
                                clip_sq, float(max_norm), 1, 0, int(max_ctas))

    def sumsq(self, opt, lo: int, sq: torch.Tensor, timeout_ms: int = 0):
        """``sq += ‖shard of the averaged gradient‖²`` for this rank's shard, read from
        every rank's gradient over NVLink (the first of a clipped step's two kernels)."""
        clock = opt.device_clock
        if clock is not None:
            _ext.ext().rs_sumsq(self.grad_buf.ptrs, self.flags.ptrs, self.flags.rank, 0, int(lo),
                                int(opt.shard), sq, 1 if self.grad_is_bf16 else 0, 1.0 / opt.world,
                                int(timeout_ms), clock[0], 2, 0)
            return
        _ext.ext().rs_sumsq(self.grad_buf.ptrs, self.flags.ptrs, self.flags.rank,
                            self.flags.next_epoch(), int(lo), int(opt.shard), sq,
                            1 if self.grad_is_bf16 else 0, 1.0 / opt.world, int(timeout_ms))

    def reduce_scatter_adamw(self, opt, mine: torch.Tensor, clip_sq: Optional[torch.Tensor] = None):
        b1, b2 = opt.betas
        lo = opt.rank * opt.shard
        self.run(lo, opt.shard, opt.exp_avg, opt.exp_avg_sq, lr=opt.lr, beta1=b1, beta2=b2,
                 eps=opt.eps, weight_decay=opt.wd, step=opt.step_count,
                 grad_scale=1.0 / opt.world, push=True, clock=opt.device_clock,
                 clip_sq=clip_sq, max_norm=opt.max_grad_norm or 0.0)


def peer_flat_allocator(group):
    """Allocator for :class:`FlatParams`: data and grad in peer memory, plus the fused
    optimizer object attached to the grad tensor."""
    state: Dict[str, PeerBuffer] = {}

    def alloc(numel: int, dtype: torch.dtype, role: str) -> torch.Tensor:
        buf = PeerBuffer(numel * torch.empty(0, dtype=dtype).element_size(), group)
        state[role] = buf
        t = buf.tensor(numel, dtype)
        t.zero_()
        t._zq_peer_buffer = buf
        if role == "grad" and "data" in state:
            t._zq_peer = PeerReduceScatterAdamW(buf, state["data"], PeerFlags(group))
        return t

    return alloc


def ag_gemm_ok(M: int, N: int, K: int, blocksize: int) -> bool:
    """Shapes the fused gather + dequantise + GEMM kernel takes."""
    return M >= 256 and K % 128 == 0 and N % 8 == 0 and blocksize % 32 == 0


def ag_gemm_pieces(x: torch.Tensor, packed_ptrs: List[int], packed_starts: List[int],
                   absmax_ptrs: List[int], absmax_starts: List[int], N: int, K: int,
                   blocksize: int, quant_type: str = "nf4", rank: int = 0,
                   out: Optional[torch.Tensor] = None, wbuf: Optional[torch.Tensor] = None,
                   extra: Optional[tuple] = None, swiglu: Optional[tuple] = None):
    """``y [M, N] = x [M, K] · Wᵀ`` for a 4-bit ``W [N, K]`` whose flat packed
    bytes and absmax are split into per-rank pieces (piece ``q`` starts at flat
    index ``*_starts[q]`` and lives at device address ``*_ptrs[q]``: local memory
    or a peer's through CUDA IPC).

    One kernel (``csrc/gemm_sm100.cu``, gather mode of the pair GEMM): warps of
    every CTA pull 8 x 1024 pieces of ``W`` over NVLink, dequantise them into
    ``wbuf`` (bf16 ``[N, K]``) and publish a per-N-tile counter; the TMA producer
    loads an N tile's B once its counter is full, and each rank starts on the N
    tiles of its own rows.  ``extra = (x2 [M, 64], w2 [N, 64])`` adds the 64-wide
    K slab of the LoRA up-projection.  ``swiglu = (g [M, N], act [M, N])``: the
    epilogue also writes ``act = silu(g)·y`` (the up-projection of a SwiGLU MLP).
    Returns ``(y, wbuf)``; ``wbuf`` holds the assembled bf16 weight afterwards.
    Needs :func:`ag_gemm_ok`.
    """
    from ..ops.nf4 import QUANT_TYPE_ID

    M = x.shape[0]
    if not ag_gemm_ok(M, N, K, blocksize):
        raise ValueError(f"ag_gemm: unsupported shape M={M} N={N} K={K} blocksize={blocksize}")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if wbuf is None:
        wbuf = torch.empty(N, K, dtype=torch.bfloat16, device=x.device)
    a2, b2 = extra if extra is not None else (None, None)
    sg, sa = swiglu if swiglu is not None else (None, None)
    _ext.ext().ag_gemm_nf4(x, [int(p) for p in packed_ptrs], [int(v) for v in packed_starts],
                           [int(p) for p in absmax_ptrs], [int(v) for v in absmax_starts],
                           N * K // 2, -(-N * K // blocksize), int(rank), int(N), int(K),
                           int(blocksize), QUANT_TYPE_ID[quant_type], wbuf, out, a2, b2, sg, sa)
    return out, wbuf


def ag_gemm_f32_pieces(x: torch.Tensor, ptrs: List[int], starts: List[int], total: int, N: int,
                       K: int, rank: int = 0, out: Optional[torch.Tensor] = None,
                       wbuf: Optional[torch.Tensor] = None, extra: Optional[tuple] = None):
    """``y = x · bf16(W)ᵀ`` for an fp32 ``W [N, K]`` split into per-rank pieces
    (flat elements ``[starts[q], starts[q+1])`` at ``ptrs[q]``; ``total`` >= N*K
    counts a zero-padded tail): gather, cast and GEMM in one kernel, like
    :func:`ag_gemm_pieces`.  Returns ``(y, wbuf)`` with ``wbuf`` = bf16 ``W``."""
    M = x.shape[0]
    if not ag_gemm_ok(M, N, K, 32):
        raise ValueError(f"ag_gemm_f32: unsupported shape M={M} N={N} K={K}")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if wbuf is None:
        wbuf = torch.empty(N, K, dtype=torch.bfloat16, device=x.device)
    a2, b2 = extra if extra is not None else (None, None)
    _ext.ext().ag_gemm_f32(x, [int(p) for p in ptrs], [int(v) for v in starts], int(total),
                           int(rank), int(N), int(K), wbuf, out, a2, b2)
    return out, wbuf


class PeerShardPool:
    """Every NF4 shard of a coordinator, in one peer buffer per rank.

    Shard byte offsets are computed identically on every rank from the shard
    plans (which every rank knows), so rank ``q``'s piece of parameter ``p``
    lives at ``ptrs[q] + offset_q(p)`` with no per-parameter exchange.
    """

    ALIGN = 16

    def __init__(self, coordinator, group=None):
        self.group = group if group is not None else coordinator.process_group
        self.rank, self.world = _group_info(self.group)
        params = [p for p in coordinator._params.values() if p.local_packed is not None]
        self.offsets: Dict[int, List[List[int]]] = {}   # pid -> [rank] -> [packed_off, absmax_off]
        ends = [0] * self.world
        for zq in params:
            entry = []
            for q in range(self.world):
                po = ends[q]
                ends[q] = (po + zq.packed_plan.lengths[q] + self.ALIGN - 1) // self.ALIGN * self.ALIGN
                ao = ends[q]
                ends[q] = (ao + 4 * zq.absmax_plan.lengths[q] + self.ALIGN - 1) // self.ALIGN * self.ALIGN
                entry.append([po, ao])
            self.offsets[zq.param_id] = entry
        self.buf = PeerBuffer(max(ends + [16]), self.group)
        self.flags = PeerFlags(self.group)
        for zq in params:
            po, ao = self.offsets[zq.param_id][self.rank]
            pk = self.buf.tensor(zq.local_packed.numel(), torch.uint8, po)
            am = self.buf.tensor(zq.local_absmax.numel(), torch.float32, ao)
            pk.copy_(zq.local_packed)
            am.copy_(zq.local_absmax)
            zq.local_packed, zq.local_absmax = pk, am
            zq._peer_pool = self
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def _segments(self, zq, which: int):
        plan = zq.packed_plan if which == 0 else zq.absmax_plan
        esz = 1 if which == 0 else 4
        src = [self.buf.ptrs[q] + self.offsets[zq.param_id][q][which] for q in range(self.world)]
        offs = [o * esz for o in plan.offsets]
        lens = [n * esz for n in plan.lengths]
        return src, offs, lens

    def gather(self, zq):
        """Assembled ``(packed, absmax)`` of ``zq`` (shards are static between
        re-quantisations, so no barrier is needed)."""
        from .comm import GatherHandle

        E = _ext.ext()
        from ..utils.metrics import count
        from .comm import remote_nf4_bytes

        count("gather_bytes", remote_nf4_bytes(zq))
        packed = torch.empty(zq.packed_plan.total, dtype=torch.uint8, device=zq.local_packed.device)
        absmax = torch.empty(zq.absmax_plan.total, dtype=torch.float32, device=zq.local_packed.device)
        for which, out in ((0, packed), (1, absmax)):
            src, offs, lens = self._segments(zq, which)
            E.plan_gather(src, self.flags.ptrs, self.rank, 0, offs, lens, out, 0)
        return GatherHandle([lambda: packed, lambda: absmax])

    def gather_dequant(self, zq, rows: int, cols: int, transpose: bool = False,
                       out: Optional[torch.Tensor] = None, row0: int = 0) -> torch.Tensor:
        """bf16 operand: rows ``[row0, row0+rows)`` of ``W [*, cols]`` (or their
        transpose) read straight from the owners' NF4 shards over NVLink: the
        gather and the dequantisation are one kernel."""
        from ..ops.nf4 import QUANT_TYPE_ID

        from ..utils.metrics import count
        from .comm import remote_nf4_bytes

        count("gather_bytes", remote_nf4_bytes(zq) * rows // max(1, zq.original_shape[0]))
        psrc, _, _ = self._segments(zq, 0)
        asrc, _, _ = self._segments(zq, 1)
        if out is None:
            out = torch.empty(rows * cols, dtype=torch.bfloat16, device=zq.local_packed.device)
        m = zq._quant_meta
        _ext.ext().plan_gather_dequant(psrc, list(zq.packed_plan.offsets), asrc,
                                       list(zq.absmax_plan.offsets), rows, cols, int(row0),
                                       int(m["blocksize"]), QUANT_TYPE_ID[m["quant_type"]],
                                       bool(transpose), out)
        return out.view(cols, rows) if transpose else out.view(rows, cols)

    def ag_gemm(self, zq, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                wbuf: Optional[torch.Tensor] = None, extra: Optional[tuple] = None,
                swiglu: Optional[tuple] = None):
        """``x Wᵀ`` with ``W`` read from the owners' NF4 shards inside the GEMM
        kernel (:func:`ag_gemm_pieces`, SwiGLU epilogue with ``swiglu``); returns
        ``(y, wbuf)``."""
        from ..utils.metrics import count
        from .comm import remote_nf4_bytes

        count("gather_bytes", remote_nf4_bytes(zq))
        psrc, _, _ = self._segments(zq, 0)
        asrc, _, _ = self._segments(zq, 1)
        N, K = zq.original_shape
        m = zq._quant_meta
        return ag_gemm_pieces(x, psrc, list(zq.packed_plan.offsets), asrc,
                              list(zq.absmax_plan.offsets), N, K, int(m["blocksize"]),
                              m["quant_type"], self.rank, out, wbuf, extra, swiglu)

    def sync_after_update(self):
        """Barrier after shards were re-quantised in place (training mode)."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def close(self):
        self.buf.close()
        self.flags.close()


class PeerMasterPool:
    """The fp32 master shards of every training-mode parameter of a coordinator,
    moved into one peer buffer per rank.

    Each parameter's shard is ``ceil(n / W)`` elements on every rank (zero-padded
    on the last), so its offset in the buffer is the same everywhere.  The
    shards' ``master_shard`` parameters keep their identity (the optimizer's
    state stays valid); only their storage moves.  After an optimizer step every
    rank must call :meth:`sync_after_update` before the next forward reads a
    peer's masters.
    """

    ALIGN = 16

    def __init__(self, coordinator, group=None):
        self.group = group if group is not None else coordinator.process_group
        self.rank, self.world = _group_info(self.group)
        params = [p for p in coordinator._params.values()
                  if getattr(p, "master_shard", None) is not None
                  and p.master_shard.dtype == torch.float32 and p.master_shard.is_cuda]
        self.offsets: Dict[int, int] = {}
        end = 0
        for zq in params:
            self.offsets[zq.param_id] = end
            end = (end + 4 * zq.master_shard.numel() + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        self.buf = PeerBuffer(max(end, 16), self.group)
        for zq in params:
            view = self.buf.tensor(zq.master_shard.numel(), torch.float32, self.offsets[zq.param_id])
            view.copy_(zq.master_shard.data)
            zq.master_shard.data = view
            zq._peer_master_pool = self
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def ag_gemm(self, zq, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                wbuf: Optional[torch.Tensor] = None, extra: Optional[tuple] = None):
        """``x · bf16(W)ᵀ`` with ``W`` gathered from every rank's master shard inside
        the GEMM kernel; returns ``(y, wbuf)``."""
        chunk = zq.master_shard.numel()
        off = self.offsets[zq.param_id]
        ptrs = [self.buf.ptrs[q] + off for q in range(self.world)]
        starts = [q * chunk for q in range(self.world)]
        N, K = zq.original_shape
        return ag_gemm_f32_pieces(x, ptrs, starts, chunk * self.world, N, K, self.rank, out,
                                  wbuf, extra)

    def sync_after_update(self):
        """Barrier after the masters were updated in place."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def close(self):
        self.buf.close()

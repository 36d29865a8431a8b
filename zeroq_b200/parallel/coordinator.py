"""Sharded 4-bit parameter engine: parameter state machine, coordinator, hooks.

Public classes keep the reference's names and behaviour
(``src/coordinator.py``):

* :class:`ZeroQParameter` - NOT_AVAILABLE / INFLIGHT / AVAILABLE state machine
  over one parameter's local shard (reference :37-712).  Uniform split rule:
  ``total // W`` packed bytes (and absmax values, split independently) per rank,
  remainder on the last rank (reference :191-212).
* :class:`ZeroQCoordinator` - registry, fetch/wait/release, memory stats,
  master params, full state dict (reference :715-884).
* :class:`ZeroQModuleWrapper` - forward/backward hooks that gather before a
  module runs and release after (reference :887-1045).

What differs from the reference, by design:

* Quantisation runs on this framework's sm_100a kernel (``csrc/nf4.cu``) and
  gathers go through :mod:`zeroq_b200.parallel.comm` - either one NCCL
  ``all_gather_into_tensor`` per buffer with in-place assembly (backend
  ``"nccl"``), or the peer-memory gather kernel over NVLink that writes the
  assembled buffer directly (backend ``"fused"``).  There are no Python unpad
  loops over ranks and no ``empty_cache`` on the hot path.
* In 4-bit compute mode, a module that is a :class:`zeroq_b200.ops.qlinear.Linear4bit`
  receives the gathered packed bytes and absmax and runs the fused NF4-dequant
  tcgen05 GEMM; no full-precision copy of the weight is made (reference
  ``src/hetero/zeroq_hetero.py:477-500`` does this with bitsandbytes' Params4bit).
* The training-mode gradient hook accumulates into ``master_shard.grad`` instead
  of overwriting it, so gradient accumulation over micro-batches is correct.
"""

from __future__ import annotations

from enum import Enum
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..config import ZeroQConfig
from ..ops.nf4 import QuantState, code_table, dequantize_4bit, quantize_4bit
from . import comm
from .gradient_sync import reduce_scatter_grads, reduce_scatter_grads_async
from .shard_plan import ShardPlan, ceil_plan, uniform_remainder_plan


class ZeroQParamStatus(Enum):
    NOT_AVAILABLE = 0
    AVAILABLE = 1
    INFLIGHT = 2


def _cfg(cfg: Any, name: str, default: Any) -> Any:
    return getattr(cfg, name, default)


def _target_device(param: torch.Tensor) -> torch.device:
    if param.device.type == "cuda":
        return param.device
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


class ZeroQParameter:
    """One parameter's shard and its gather/release lifecycle."""

    def __init__(self, param: torch.nn.Parameter, rank: int, world_size: int,
                 config: ZeroQConfig, param_id: int, module: Optional[torch.nn.Module] = None,
                 param_name: Optional[str] = None,
                 process_group: Optional[dist.ProcessGroup] = None):
        self.param = param
        self.rank = int(rank)
        self.world_size = int(world_size)
        self.config = config
        self.param_id = int(param_id)
        self.module = module
        self.param_name = param_name
        self.process_group = process_group

        self.original_shape = param.data.shape
        self.original_numel = param.data.numel()
        self.original_dtype = param.data.dtype
        self.compute_in_4bit = bool(_cfg(config, "compute_in_4bit", False))

        self.status = ZeroQParamStatus.NOT_AVAILABLE
        self.local_packed: Optional[torch.Tensor] = None
        self.local_absmax: Optional[torch.Tensor] = None
        self._quant_meta: Optional[Dict[str, Any]] = None
        self.packed_plan: Optional[ShardPlan] = None
        self.absmax_plan: Optional[ShardPlan] = None
        self._packed_total = 0
        self._absmax_total = 0

        self._pending = None  # in-flight gather (comm.GatherHandle)
        self._assembled_packed: Optional[torch.Tensor] = None
        self._assembled_absmax: Optional[torch.Tensor] = None

        # training-from-scratch state
        self.master_shard: Optional[torch.nn.Parameter] = None
        self._fp32_chunk_size = 0
        self.master_plan: Optional[ShardPlan] = None

    # -- plans ---------------------------------------------------------------
    def _make_plans(self, packed_total: int, absmax_total: int):
        return (uniform_remainder_plan(packed_total, self.world_size),
                uniform_remainder_plan(absmax_total, self.world_size))

    # compatibility accessors used by the reference's callers and tests
    @property
    def packed_per_rank(self) -> int:
        return self._packed_total // self.world_size if self.packed_plan else 0

    @property
    def absmax_per_rank(self) -> int:
        return self._absmax_total // self.world_size if self.absmax_plan else 0

    @property
    def _packed_remainder(self) -> int:
        return self._packed_total % self.world_size

    @property
    def _absmax_remainder(self) -> int:
        return self._absmax_total % self.world_size

    # -- partition -----------------------------------------------------------
    def partition(self):
        if self.status != ZeroQParamStatus.NOT_AVAILABLE:
            return
        if self.local_packed is not None or self.master_shard is not None:
            return
        self.partition_from_full_precision(self.param.data)

    def _replace_placeholder(self, device: torch.device, dtype: torch.dtype,
                             requires_grad: Optional[bool] = None):
        rg = self.param.requires_grad if requires_grad is None else requires_grad
        if self.param.device.type == "meta" or self.param.device != device:
            if self.module is None or self.param_name is None:
                raise RuntimeError(
                    "ZeroQParameter needs module+param_name to replace meta/cpu parameters "
                    "safely. Register parameters via ZeroQModuleWrapper.")
            new_param = torch.nn.Parameter(torch.empty(0, device=device, dtype=dtype),
                                           requires_grad=rg)
            setattr(self.module, self.param_name, new_param)
            self.param = new_param

    def _quantize_and_keep_shard(self, weight: torch.Tensor, device: torch.device):
        """Quantise only the 64-value blocks that cover this rank's bytes.

        The plans depend only on the tensor's size, so this rank's packed-byte and
        absmax ranges are known before quantising; NF4 blocks are independent, so
        quantising the covering blocks gives exactly the bytes a full quantisation
        would.  The reference quantises the whole tensor on every rank and slices
        (``src/coordinator.py:166-212``); here no rank materialises more than its
        own range (plus one block at each end) in fp16 or NF4."""
        bs = int(self.config.blocksize)
        flat = weight.detach().reshape(-1)
        n = flat.numel()
        self._packed_total = (n + 1) // 2
        self._absmax_total = (n + bs - 1) // bs
        self.packed_plan, self.absmax_plan = self._make_plans(self._packed_total,
                                                              self._absmax_total)
        p0, p1 = self.packed_plan.range_of(self.rank)
        a0, a1 = self.absmax_plan.range_of(self.rank)
        # blocks [b0, b1) cover elements [2 p0, 2 p1) and absmax entries [a0, a1)
        b0 = min((2 * p0) // bs, a0) if p1 > p0 or a1 > a0 else 0
        b1 = max((2 * p1 + bs - 1) // bs, a1)
        e0, e1 = b0 * bs, min(n, b1 * bs)
        # The reference quantises fp16-cast weights (src/coordinator.py:166-168);
        # casting first keeps the stored bytes identical.
        w = flat[e0:e1].to(device=device, dtype=torch.float16)
        if e1 > e0:
            packed, state = quantize_4bit(w, blocksize=bs, quant_type=self.config.quant_type)
            packed, absmax = packed.view(-1), state.absmax.view(-1)
        else:
            packed = torch.empty(0, dtype=torch.uint8, device=device)
            absmax = torch.empty(0, dtype=torch.float32, device=device)
        self.local_packed = comm.alloc_shard(p1 - p0, torch.uint8, device, self)
        self.local_packed.copy_(packed[p0 - e0 // 2:p1 - e0 // 2])
        self.local_absmax = comm.alloc_shard(a1 - a0, torch.float32, device, self)
        self.local_absmax.copy_(absmax[a0 - b0:a1 - b0])
        self._quant_meta = {
            "shape": tuple(weight.shape), "dtype": torch.float16,
            "blocksize": bs, "quant_type": self.config.quant_type,
        }

    def partition_from_full_precision(self, weight: torch.Tensor):
        """Quantise ``weight`` and keep this rank's shard (streamed loading entry)."""
        if self.status != ZeroQParamStatus.NOT_AVAILABLE:
            return
        if self.local_packed is not None or self.master_shard is not None:
            return
        if _cfg(self.config, "training_mode", False):
            self._partition_fp32_training(weight)
            return
        if weight.numel() != self.original_numel:
            raise ValueError(f"Weight numel mismatch for param_id={self.param_id}: "
                             f"expected {self.original_numel}, got {weight.numel()}")
        device = _target_device(self.param)
        self._replace_placeholder(device, self.original_dtype)
        self._quantize_and_keep_shard(weight, device)
        self.param.data = torch.empty(0, device=device, dtype=self.original_dtype)
        self.status = ZeroQParamStatus.NOT_AVAILABLE

    def _partition_fp32_training(self, weight: torch.Tensor):
        if _cfg(self.config, "cpu_offload", False) or _cfg(self.config, "fused_shard_step", False):
            self._partition_cpu_offload(weight)
            return
        device = _target_device(self.param)
        self._replace_placeholder(device, torch.float32, requires_grad=True)
        flat = weight.detach().contiguous().view(-1).to(dtype=torch.float32, device=device)
        self.master_plan = ceil_plan(flat.numel(), self.world_size)
        chunk = (flat.numel() + self.world_size - 1) // self.world_size
        s, e = self.master_plan.range_of(self.rank)
        shard = flat[s:e].clone()
        if shard.numel() < chunk:
            shard = F.pad(shard, (0, chunk - shard.numel()))
        self.master_shard = torch.nn.Parameter(shard, requires_grad=True)
        self._fp32_chunk_size = chunk
        self.param.data = torch.empty(0, device=device, dtype=torch.float32)
        self.status = ZeroQParamStatus.NOT_AVAILABLE

    def _partition_cpu_offload(self, weight: torch.Tensor):
        """NF4 shard on the GPU (forward cache) + master shard (CPU when
        ``cpu_offload``, else GPU) - reference ``src/coordinator.py:265-347``."""
        device = _target_device(self.param)
        self._replace_placeholder(device, self.original_dtype, requires_grad=True)
        self._quantize_and_keep_shard(weight, device)
        mdtype = _cfg(self.config, "master_dtype", torch.float32)
        flat = weight.detach().contiguous().view(-1).to(mdtype)
        chunk = (flat.numel() + self.world_size - 1) // self.world_size
        self.master_plan = ceil_plan(flat.numel(), self.world_size)
        s, e = self.master_plan.range_of(self.rank)
        shard = flat[s:e].clone()
        shard = shard.cpu() if _cfg(self.config, "cpu_offload", False) else shard.to(device)
        if _cfg(self.config, "cpu_offload", False) and torch.cuda.is_available():
            shard = shard.pin_memory()
        if shard.numel() < chunk:
            shard = F.pad(shard, (0, chunk - shard.numel()))
        self.master_shard = torch.nn.Parameter(shard, requires_grad=True)
        self._fp32_chunk_size = chunk
        self.param.data = torch.empty(0, device=device, dtype=self.original_dtype)
        self.status = ZeroQParamStatus.NOT_AVAILABLE

    def _make_trainable_with_cpu_grad(self):
        """Mark the gathered weight frozen for autograd: its gradient is computed
        by the post-backward hook (reference ``src/coordinator.py:349-359``)."""
        self.param.requires_grad_(False)
        if self.param.data.dtype != torch.float32:
            self.param.data = self.param.data.float()

    # -- gather --------------------------------------------------------------
    def _is_fp32_mode(self) -> bool:
        return bool(_cfg(self.config, "training_mode", False)) and not bool(
            _cfg(self.config, "cpu_offload", False)) and not bool(
            _cfg(self.config, "fused_shard_step", False))

    def start_gather(self, group: Optional[dist.ProcessGroup] = None, async_op: bool = True,
                     force_local: bool = False):
        """Start gathering this parameter.

        ``force_local=True`` always assembles the whole NF4 weight on this rank
        (through the peer plan-gather kernel when a peer pool is registered, NCCL
        otherwise) instead of attaching the module to its owners' shards."""
        if self.status == ZeroQParamStatus.AVAILABLE:
            return None
        if self.status == ZeroQParamStatus.INFLIGHT:
            if not async_op:
                self.wait_gather()
                return None
            return self._pending
        group = group if group is not None else self.process_group
        if self._is_fp32_mode():
            if self._use_master_source():
                # the module's GEMM gathers and casts the fp32 masters itself
                self.module.set_master_source(self._peer_master_pool, self)
                self.status = ZeroQParamStatus.AVAILABLE
                return None
            return self._start_gather_fp32(group, async_op)
        if self.local_packed is None:
            raise RuntimeError(f"param_id={self.param_id} is not partitioned")
        if not force_local and self._use_peer_source():
            # fused backend, 4-bit compute: nothing is gathered here; the module's
            # GEMM reads every owner's shard itself (gather + dequant + GEMM kernel)
            self.module.set_peer_source(self._peer_pool, self)
            self.status = ZeroQParamStatus.AVAILABLE
            return None
        self._pending = comm.gather_nf4(self, group=group, async_op=async_op)
        self.status = ZeroQParamStatus.INFLIGHT
        if not async_op:
            self.wait_gather()
            return None
        return self._pending

    def _use_master_source(self) -> bool:
        if (getattr(self, "_peer_master_pool", None) is None or self.param_name != "weight"
                or self.world_size == 1):
            return False
        from ..ops.qlinear import Linear4bit

        return isinstance(self.module, Linear4bit)

    def _use_peer_source(self) -> bool:
        if (getattr(self, "_peer_pool", None) is None or not self.compute_in_4bit
                or self.param_name != "weight" or self.world_size == 1
                or comm._backend(self) != "fused"):
            return False
        from ..ops.qlinear import Linear4bit

        return isinstance(self.module, Linear4bit)

    def wait_gather(self):
        if self.status != ZeroQParamStatus.INFLIGHT:
            return
        if self._is_fp32_mode():
            self._complete_gather_fp32()
            return
        packed, absmax = self._pending.wait()
        self._pending = None
        self._assembled_packed, self._assembled_absmax = packed, absmax
        self._complete_gather()
        if _cfg(self.config, "training_mode", False) and (
                _cfg(self.config, "cpu_offload", False) or _cfg(self.config, "fused_shard_step", False)):
            self._make_trainable_with_cpu_grad()

    def quant_state(self, absmax: torch.Tensor) -> QuantState:
        m = self._quant_meta
        return QuantState(absmax=absmax, shape=torch.Size(m["shape"]), dtype=m["dtype"],
                          blocksize=m["blocksize"],
                          code=code_table(m["quant_type"], device=absmax.device),
                          quant_type=m["quant_type"])

    def _complete_gather(self):
        if self._quant_meta is None:
            raise RuntimeError(f"Missing quant metadata for param_id={self.param_id}")
        from ..ops.qlinear import Linear4bit  # local import: ops depend on torch only

        if (self.compute_in_4bit and isinstance(self.module, Linear4bit)
                and self.param_name == "weight"):
            # 4-bit compute: hand the module the gathered NF4 data, no dequant.
            self.module.set_nf4(self._assembled_packed, self._assembled_absmax,
                                self._quant_meta)
            self.status = ZeroQParamStatus.AVAILABLE
            return
        state = self.quant_state(self._assembled_absmax)
        restored = dequantize_4bit(self._assembled_packed, state, out_dtype=self.original_dtype)
        restored = restored.view(self.original_shape)
        if self.module is not None and self.param_name is not None:
            # Install a new Parameter instead of mutating .data, so tensors that
            # activation checkpointing saved stay valid (reference :573-583).
            new_param = torch.nn.Parameter(restored, requires_grad=self.param.requires_grad)
            setattr(self.module, self.param_name, new_param)
            self.param = new_param
        else:
            self.param.data = restored
        self._assembled_packed = None
        self._assembled_absmax = None
        self.status = ZeroQParamStatus.AVAILABLE

    def _start_gather_fp32(self, group, async_op):
        self._pending = comm.gather_master(self, group=group, async_op=async_op)
        self.status = ZeroQParamStatus.INFLIGHT
        if not async_op:
            self._complete_gather_fp32()
            return None
        return self._pending

    def _complete_gather_fp32(self):
        full = self._pending.wait() if self._pending is not None else \
            self.master_shard.data[: self.original_numel]
        self._pending = None
        full = full[: self.original_numel].view(self.original_shape)
        new_param = torch.nn.Parameter(full, requires_grad=True)
        zq = self

        def _grad_hook(grad):
            # the reduce-scatter starts now and overlaps the rest of the backward;
            # it is finished (and added into the master shard's .grad) by a
            # callback at the end of this backward pass, so .grad is complete when
            # backward() returns, as with the synchronous form
            coord = getattr(zq, "coordinator", None)
            if coord is None:   # a parameter used outside a coordinator: synchronous
                local = reduce_scatter_grads(grad, zq.world_size, zq.rank, group=zq.process_group)
                local = local[: zq.master_shard.numel()].to(zq.master_shard.dtype)
                if zq.master_shard.grad is None:
                    zq.master_shard.grad = local
                else:
                    zq.master_shard.grad.add_(local)
                return grad
            coord._pending_grad_sync(zq, reduce_scatter_grads_async(
                grad, zq.world_size, zq.rank, group=zq.process_group))
            return grad

        new_param.register_hook(_grad_hook)
        if self.module is not None and self.param_name is not None:
            setattr(self.module, self.param_name, new_param)
        self.param = new_param
        self.status = ZeroQParamStatus.AVAILABLE

    # -- release -------------------------------------------------------------
    def release(self):
        if self.status == ZeroQParamStatus.NOT_AVAILABLE:
            return
        if self.status == ZeroQParamStatus.INFLIGHT:
            self.wait_gather()
        from ..ops.qlinear import Linear4bit

        if self._is_fp32_mode():
            device = self.master_shard.device if self.master_shard.device.type != "cpu" \
                else self.param.device
            dtype, rg = torch.float32, True
        else:
            device, dtype, rg = self.param.device, self.original_dtype, self.param.requires_grad
        if isinstance(self.module, Linear4bit) and self.param_name == "weight":
            self.module.clear_master_source()
        if (self.compute_in_4bit and isinstance(self.module, Linear4bit)
                and self.param_name == "weight" and not self._is_fp32_mode()):
            self.module.clear_nf4()
        elif self.module is not None and self.param_name is not None:
            placeholder = torch.nn.Parameter(torch.empty(0, device=device, dtype=dtype),
                                             requires_grad=rg)
            setattr(self.module, self.param_name, placeholder)
            self.param = placeholder
        else:
            self.param.data = torch.empty(0, device=device, dtype=dtype)
        self._assembled_packed = None
        self._assembled_absmax = None
        self.status = ZeroQParamStatus.NOT_AVAILABLE

    # -- accounting ----------------------------------------------------------
    @property
    def local_memory_bytes(self) -> int:
        if self.master_shard is not None:
            return self.master_shard.numel() * self.master_shard.element_size()
        if self.local_packed is None:
            return 0
        return (self.local_packed.numel() * self.local_packed.element_size()
                + self.local_absmax.numel() * self.local_absmax.element_size())

    @property
    def full_memory_bytes(self) -> int:
        return self.original_numel * 2

    def shard_state(self) -> Dict[str, Any]:
        """Everything needed to restore this rank's shard (sharded checkpoint)."""
        out: Dict[str, Any] = {"param_id": self.param_id, "name": self.param_name,
                               "shape": list(self.original_shape),
                               "dtype": str(self.original_dtype)}
        if self.local_packed is not None:
            out.update(local_packed=self.local_packed.detach().cpu(),
                       local_absmax=self.local_absmax.detach().cpu(),
                       packed_plan=[self.packed_plan.lengths, self.packed_plan.offsets],
                       absmax_plan=[self.absmax_plan.lengths, self.absmax_plan.offsets],
                       quant_meta={k: (str(v) if isinstance(v, torch.dtype) else v)
                                   for k, v in self._quant_meta.items()})
        if self.master_shard is not None:
            out["master_shard"] = self.master_shard.detach().cpu()
        return out

    def load_shard_state(self, st: Dict[str, Any]):
        from ..config import _dtype_from

        device = _target_device(self.param)
        if "local_packed" in st:
            self._replace_placeholder(device, self.original_dtype)
            self.packed_plan = ShardPlan(*[list(x) for x in st["packed_plan"]])
            self.absmax_plan = ShardPlan(*[list(x) for x in st["absmax_plan"]])
            self._packed_total = self.packed_plan.total
            self._absmax_total = self.absmax_plan.total
            self.local_packed = comm.alloc_shard(st["local_packed"].numel(), torch.uint8,
                                                 device, self)
            self.local_packed.copy_(st["local_packed"])
            self.local_absmax = comm.alloc_shard(st["local_absmax"].numel(), torch.float32,
                                                 device, self)
            self.local_absmax.copy_(st["local_absmax"])
            qm = dict(st["quant_meta"])
            qm["dtype"] = _dtype_from(qm["dtype"])
            qm["shape"] = tuple(qm["shape"])
            self._quant_meta = qm
            self.param.data = torch.empty(0, device=device, dtype=self.original_dtype)
        if "master_shard" in st:
            ms = st["master_shard"]
            dev = ms.device if _cfg(self.config, "cpu_offload", False) else device
            if self.master_shard is None:
                self.master_shard = torch.nn.Parameter(ms.to(dev).clone(), requires_grad=True)
            else:
                self.master_shard.data.copy_(ms)
            self.master_plan = ceil_plan(self.original_numel, self.world_size)
            self._fp32_chunk_size = ms.numel()
        self.status = ZeroQParamStatus.NOT_AVAILABLE


class ZeroQCoordinator:
    """Registry of sharded parameters (reference ``src/coordinator.py:715-884``)."""

    param_cls = ZeroQParameter

    def __init__(self, config: ZeroQConfig, process_group: Optional[dist.ProcessGroup] = None):
        self.config = config
        self.process_group = process_group
        if dist.is_initialized():
            self.rank = dist.get_rank(process_group)
            self.world_size = dist.get_world_size(process_group)
        else:
            self.rank, self.world_size = 0, 1
        self._params: Dict[int, ZeroQParameter] = {}
        self._params_by_obj_id: Dict[int, ZeroQParameter] = {}
        self._param_to_module: Dict[int, torch.nn.Module] = {}
        self._next_param_id = 0
        self._collective_seq = 0
        self._grad_sync_pending = []     # (ZeroQParameter, finish) of this backward
        self._grad_sync_queued = False

    # -- train mode: reduce-scatters overlapped with the backward -----------------
    def _pending_grad_sync(self, zq, finish):
        """Called from a gradient hook: remember the started reduce-scatter and, once
        per backward pass, queue the callback that finishes them all when the
        autograd engine is done (how DDP overlaps its buckets with the backward)."""
        self._grad_sync_pending.append((zq, finish))
        if not self._grad_sync_queued:
            self._grad_sync_queued = True
            torch.autograd.Variable._execution_engine.queue_callback(self._finish_grad_sync)

    def _finish_grad_sync(self):
        pending, self._grad_sync_pending = self._grad_sync_pending, []
        self._grad_sync_queued = False
        for zq, finish in pending:
            local = finish()[: zq.master_shard.numel()].to(zq.master_shard.dtype)
            if zq.master_shard.grad is None:
                zq.master_shard.grad = local
            else:
                zq.master_shard.grad.add_(local)

    def _new_param(self, param, module, param_name, param_id):
        return self.param_cls(param=param, rank=self.rank, world_size=self.world_size,
                              config=self.config, param_id=param_id, module=module,
                              param_name=param_name, process_group=self.process_group)

    def register_parameter(self, param: Any, module: Optional[torch.nn.Module] = None,
                           param_name: Optional[str] = None) -> ZeroQParameter:
        if isinstance(param, str) and isinstance(module, torch.nn.Parameter):
            param_name, param, module = param, module, None
        pid = self._next_param_id
        self._next_param_id += 1
        zq = self._new_param(param, module, param_name, pid)
        zq.coordinator = self
        self._params[pid] = zq
        self._params_by_obj_id[id(param)] = zq
        if module is not None:
            self._param_to_module[pid] = module
        return zq

    def get_param_for_tensor(self, param: torch.nn.Parameter) -> Optional[ZeroQParameter]:
        return self._params_by_obj_id.get(id(param))

    def partition_all(self):
        for zq in self._params.values():
            zq.partition()

    @staticmethod
    def _is_partitioned(p: ZeroQParameter) -> bool:
        return p.local_packed is not None or p.master_shard is not None

    def fetch_params(self, param_ids: List[int], async_op: bool = True):
        for pid in param_ids:
            p = self._params.get(pid)
            if p is not None and self._is_partitioned(p):
                if p.status == ZeroQParamStatus.NOT_AVAILABLE:
                    self._collective_seq += 1
                p.start_gather(group=self.process_group, async_op=async_op)

    def wait_params(self, param_ids: List[int]):
        for pid in param_ids:
            p = self._params.get(pid)
            if p is not None:
                p.wait_gather()

    def release_params(self, param_ids: List[int]):
        for pid in param_ids:
            p = self._params.get(pid)
            if p is not None and self._is_partitioned(p):
                p.release()

    def get_memory_stats(self) -> Dict[str, float]:
        local = sum(p.local_memory_bytes for p in self._params.values())
        full = sum(p.full_memory_bytes for p in self._params.values())
        return {
            "local_memory_mb": local / 1024 ** 2,
            "full_fp16_memory_mb": full / 1024 ** 2,
            "compression_ratio": full / max(local, 1),
            "num_params": len(self._params),
            "collective_seq": float(self._collective_seq),
        }

    def trainable_master_params(self) -> List[torch.nn.Parameter]:
        return [p.master_shard for p in self._params.values() if p.master_shard is not None]

    def update_4bit_from_masters(self):
        """Re-quantise each master shard's full tensor into this rank's NF4 shard
        after an optimizer step (reference ``src/coordinator.py:830-864``).

        Every rank holds only its master slice, so the full weight is gathered
        first (the reference quantised the local master as if it were the whole
        tensor, which only works at world size 1)."""
        for zq in self._params.values():
            if zq.master_shard is None or zq.local_packed is None:
                continue
            dev = zq.local_packed.device
            shard = zq.master_shard.data.to(device=dev, dtype=torch.float32)
            if zq.world_size > 1 and dist.is_initialized():
                full = shard.new_empty(shard.numel() * zq.world_size)
                dist.all_gather_into_tensor(full, shard.contiguous(), group=zq.process_group)
            else:
                full = shard
            full = full[: zq.original_numel].to(torch.float16)
            packed, st = quantize_4bit(full, blocksize=zq.config.blocksize,
                                       quant_type=zq.config.quant_type)
            p0, p1 = zq.packed_plan.range_of(zq.rank)
            a0, a1 = zq.absmax_plan.range_of(zq.rank)
            zq.local_packed.copy_(packed.view(-1)[p0:p1])
            zq.local_absmax.copy_(st.absmax.view(-1)[a0:a1])

    def gather_full_state_dict(self, key_by_name: bool = True) -> Dict[str, torch.Tensor]:
        """Gather every master-sharded parameter; rank 0 gets the full tensors.

        Keys are ``<module path>.<param name>`` when the wrapper recorded module
        paths (portable), else the reference's ``f"{id(module)}.{name}"``."""
        state: Dict[str, torch.Tensor] = {}
        for zq in self._params.values():
            if zq.master_shard is None:
                continue
            zq.start_gather(group=self.process_group, async_op=False)
            if zq.status == ZeroQParamStatus.INFLIGHT:
                zq.wait_gather()
            if self.rank == 0:
                path = getattr(zq, "module_path", None)
                key = (f"{path}.{zq.param_name}" if (key_by_name and path is not None)
                       else f"{id(zq.module)}.{zq.param_name}")
                state[key] = zq.param.data.detach().clone()
            zq.release()
        return state

    def __len__(self):
        return len(self._params)


class ZeroQModuleWrapper:
    """Install gather/release hooks on every module that owns registered params."""

    sort_registration = False

    def __init__(self, module: torch.nn.Module, coordinator: ZeroQCoordinator,
                 trainable_only: bool = False):
        self.module = module
        self.coordinator = coordinator
        self.trainable_only = trainable_only
        self._module_param_ids: Dict[torch.nn.Module, List[int]] = {}
        self._hook_handles: list = []
        self._register_parameters(module)
        self._install_hooks(module)
        self._prefetcher = None
        cfg = coordinator.config
        if (_cfg(cfg, "async_gather", False) and int(_cfg(cfg, "prefetch_count", 0)) > 0
                and coordinator.world_size > 1):
            from .prefetch import AutoPrefetcher

            self._prefetcher = AutoPrefetcher(coordinator, self._module_param_ids,
                                              int(_cfg(cfg, "prefetch_count", 1)))

    def _named_modules(self, module):
        items = list(module.named_modules())
        return sorted(items, key=lambda t: t[0]) if self.sort_registration else items

    def _register_parameters(self, module: torch.nn.Module):
        cfg = self.coordinator.config
        excluded = set(_cfg(cfg, "exclude_modules", []) or [])
        targets = _cfg(cfg, "target_modules", None)
        for name, child in self._named_modules(module):
            if any(ex in name for ex in excluded):
                continue
            if targets is not None and name and not any(t in name for t in targets):
                continue
            params = list(child.named_parameters(recurse=False))
            if self.sort_registration:
                params.sort(key=lambda t: t[0])
            pids = []
            for pname, p in params:
                if self.trainable_only and not p.requires_grad:
                    continue
                if p.requires_grad and not _cfg(cfg, "partition_trainable", False):
                    continue
                if _cfg(cfg, "frozen_only", True) and p.requires_grad:
                    continue
                existing = self.coordinator.get_param_for_tensor(p)
                if existing is not None:
                    pids.append(existing.param_id)
                else:
                    zq = self.coordinator.register_parameter(p, child, param_name=pname)
                    zq.module_path = name
                    pids.append(zq.param_id)
            if pids:
                self._module_param_ids[child] = pids

    def _install_hooks(self, module: torch.nn.Module):
        for child in module.modules():
            if child in self._module_param_ids:
                h = self._hook_handles
                h.append(child.register_forward_pre_hook(self._pre_forward_hook))
                h.append(child.register_forward_hook(self._post_forward_hook))
                h.append(child.register_full_backward_pre_hook(self._pre_backward_hook))
                h.append(child.register_full_backward_hook(self._post_backward_hook))

    def remove_hooks(self):
        for h in self._hook_handles:
            h.remove()
        self._hook_handles = []

    def _pre_forward_hook(self, module, inputs):
        pids = self._module_param_ids.get(module)
        if pids is None:
            return
        self.coordinator.fetch_params(pids, async_op=False)
        if self._prefetcher is not None:
            self._prefetcher.on_forward(module)
        cfg = self.coordinator.config
        if _cfg(cfg, "cpu_offload", False) or _cfg(cfg, "fused_shard_step", False):
            module._zq_saved_input = inputs[0].detach()

    def _post_forward_hook(self, module, inputs, outputs):
        pids = self._module_param_ids.get(module)
        if pids is not None:
            self.coordinator.release_params(pids)

    def _pre_backward_hook(self, module, grad_output):
        pids = self._module_param_ids.get(module)
        if pids is not None:
            self.coordinator.fetch_params(pids, async_op=False)
            if self._prefetcher is not None:
                self._prefetcher.on_backward(module)

    def _post_backward_hook(self, module, grad_input, grad_output):
        pids = self._module_param_ids.get(module)
        if pids is None:
            return
        cfg = self.coordinator.config
        if ((_cfg(cfg, "cpu_offload", False) or _cfg(cfg, "fused_shard_step", False))
                and hasattr(module, "_zq_saved_input") and grad_output[0] is not None):
            self._manual_weight_grad(module, grad_output[0])
            del module._zq_saved_input
        self.coordinator.release_params(pids)

    def _manual_weight_grad(self, module, grad_output):
        """Weight/bias gradient of a Linear from the saved input, reduce-scattered
        into the master shard (reference ``src/coordinator.py:990-1014``)."""
        x = module._zq_saved_input
        go = grad_output.reshape(-1, grad_output.shape[-1])
        x = x.reshape(-1, x.shape[-1])
        fused = _cfg(self.coordinator.config, "fused_shard_step", False)
        for pid in self._module_param_ids[module]:
            zq = self.coordinator._params[pid]
            if zq.master_shard is None:
                continue
            if zq.param_name == "weight":
                flat = (go.t().float() @ x.float()).contiguous().view(-1)
            elif zq.param_name == "bias":
                flat = go.float().sum(0).contiguous().view(-1)
            else:
                continue
            if zq.world_size > 1 and dist.is_initialized():
                local = reduce_scatter_grads(flat, zq.world_size, zq.rank,
                                             group=zq.process_group)
            else:
                local = flat
            local = local[: zq.master_shard.numel()]
            if local.numel() < zq.master_shard.numel():
                local = F.pad(local, (0, zq.master_shard.numel() - local.numel()))
            if fused:
                self._fused_lion_step(zq, local)
            else:
                g = local.to(device=zq.master_shard.device, dtype=zq.master_shard.dtype)
                if zq.master_shard.grad is None:
                    zq.master_shard.grad = g
                else:
                    zq.master_shard.grad.add_(g)

    def _fused_lion_step(self, zq: ZeroQParameter, grad_shard: torch.Tensor):
        """Lion update of the master shard right after its gradient arrives,
        with stochastic rounding for fp16 masters (reference :1016-1037)."""
        from ..ops.optim import lion_step

        cfg = self.coordinator.config
        if not hasattr(zq, "_lion_m"):
            zq._lion_m = torch.zeros(zq.master_shard.numel(), device=zq.master_shard.device,
                                     dtype=torch.float32)
        zq._lion_step_count = getattr(zq, "_lion_step_count", 0) + 1
        lion_step(zq.master_shard.data, grad_shard.to(zq.master_shard.device), zq._lion_m,
                  lr=cfg.lion_lr, beta1=cfg.lion_beta1, beta2=cfg.lion_beta2, wd=cfg.lion_wd,
                  seed=zq.param_id * 1000003 + zq._lion_step_count)

    def partition(self):
        self.coordinator.partition_all()

    def get_memory_stats(self) -> Dict[str, float]:
        return self.coordinator.get_memory_stats()

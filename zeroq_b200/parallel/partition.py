"""Functional quantise-and-shard API (reference ``src/partition.py``).

* :func:`compute_aligned_partition_sizes` - block-aligned split math
  (reference ``src/partition.py:78-129``).
* :func:`partition_quantized_tensor` - flatten, pad, quantise, keep this rank's
  slice (reference ``:132-238``).  Because the aligned split puts every block
  wholly on one rank, each rank quantises only its own element range; no rank
  materialises the full packed tensor.  The bytes are identical to quantising the
  whole tensor and slicing.
* :func:`gather_and_dequantize` - all-gather the packed bytes and absmax and
  dequantise (reference ``:241-354``).  On CUDA the two collectives are one
  NCCL ``all_gather_into_tensor`` each into a contiguous buffer (no list + cat).
* :func:`repartition_tensor`, :func:`estimate_memory_savings`,
  :func:`partition_fp32`, :func:`gather_fp32` - reference ``:357-513``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops.nf4 import QuantState, code_table, dequantize_4bit, quantize_4bit

# The reference gates its quantisation on bitsandbytes; this framework's
# quantiser is built in, so the functional API is always available.
BNB_AVAILABLE = True


@dataclass
class PartitionInfo:
    """Metadata to rebuild a tensor from block-aligned quantised shards."""

    rank: int
    world_size: int
    original_shape: torch.Size
    original_numel: int
    original_dtype: torch.dtype
    packed_partition_size: int
    absmax_partition_size: int
    blocksize: int
    elements_per_rank: int
    padded_numel: int

    @property
    def needs_padding(self) -> bool:
        return self.padded_numel > self.original_numel

    @property
    def padding_elements(self) -> int:
        return self.padded_numel - self.original_numel


def compute_aligned_partition_sizes(
    numel: int, world_size: int, blocksize: int = 64
) -> Tuple[int, int, int, int]:
    """Split ``numel`` into ``world_size`` equal, block-aligned parts.

    Returns ``(elements_per_rank, packed_bytes_per_rank, absmax_per_rank,
    padded_numel)``; ``padded_numel`` is the number of blocks rounded up to a
    multiple of ``world_size``, times ``blocksize``.
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    num_blocks = (numel + blocksize - 1) // blocksize
    aligned_blocks = ((num_blocks + world_size - 1) // world_size) * world_size
    aligned_blocks = max(aligned_blocks, world_size)
    blocks_per_rank = aligned_blocks // world_size
    elements_per_rank = blocks_per_rank * blocksize
    padded_numel = aligned_blocks * blocksize
    return elements_per_rank, elements_per_rank // 2, blocks_per_rank, padded_numel


def partition_quantized_tensor(
    weight: torch.Tensor,
    rank: int,
    world_size: int,
    blocksize: int = 64,
    quant_type: str = "nf4",
    compute_dtype: torch.dtype = torch.float32,
) -> Tuple[torch.Tensor, torch.Tensor, QuantState, PartitionInfo]:
    """Quantise ``weight`` and return this rank's ``(packed, absmax, state, info)``.

    ``state.absmax`` is this rank's absmax slice; ``state.shape`` is the padded
    flat shape of the whole tensor.
    """
    if rank >= world_size or rank < 0:
        raise ValueError(f"rank ({rank}) must be < world_size ({world_size})")
    original_shape = weight.shape
    numel = weight.numel()
    elements, packed_n, absmax_n, padded = compute_aligned_partition_sizes(
        numel, world_size, blocksize)
    flat = weight.detach().contiguous().view(-1)
    start = rank * elements
    end = start + elements
    local = flat[start:min(end, numel)]
    if local.numel() < elements:
        local = F.pad(local, (0, elements - local.numel()))
    local = local.to(compute_dtype)
    packed, state = quantize_4bit(local, blocksize=blocksize, quant_type=quant_type)
    info = PartitionInfo(
        rank=rank, world_size=world_size, original_shape=original_shape,
        original_numel=numel, original_dtype=weight.dtype,
        packed_partition_size=packed_n, absmax_partition_size=absmax_n,
        blocksize=blocksize, elements_per_rank=elements, padded_numel=padded,
    )
    qs = QuantState(absmax=state.absmax, shape=torch.Size([padded]), dtype=compute_dtype,
                    blocksize=blocksize, code=state.code, quant_type=quant_type)
    return packed, state.absmax, qs, info


def _all_gather_flat(local: torch.Tensor, world_size: int, group=None,
                     async_op: bool = False):
    out = local.new_empty(local.numel() * world_size)
    work = dist.all_gather_into_tensor(out, local.contiguous(), group=group, async_op=async_op)
    return out, work


def gather_and_dequantize(
    local_packed: torch.Tensor,
    local_absmax: torch.Tensor,
    quant_state: QuantState,
    partition_info: PartitionInfo,
    group: Optional[dist.ProcessGroup] = None,
    async_op: bool = False,
) -> torch.Tensor:
    """All-gather aligned shards from every rank and dequantise to the original shape."""
    ws = partition_info.world_size
    if not dist.is_initialized() or ws == 1:
        full_packed, full_absmax = local_packed, local_absmax
        n_flat = partition_info.elements_per_rank
    else:
        full_packed, w1 = _all_gather_flat(local_packed, ws, group, async_op=True)
        full_absmax, w2 = _all_gather_flat(local_absmax, ws, group, async_op=True)
        w1.wait()
        w2.wait()
        n_flat = partition_info.padded_numel
    state = QuantState(
        absmax=full_absmax, shape=torch.Size([n_flat]), dtype=quant_state.dtype,
        blocksize=quant_state.blocksize,
        code=quant_state.code, quant_type=quant_state.quant_type,
    )
    full = dequantize_4bit(full_packed, state)
    full = full.reshape(-1)[: partition_info.original_numel]
    return full.view(partition_info.original_shape)


def repartition_tensor(
    full_weight: torch.Tensor,
    partition_info: PartitionInfo,
    quant_type: str = "nf4",
) -> Tuple[torch.Tensor, torch.Tensor, QuantState]:
    """Re-quantise an updated full tensor and return this rank's new shard."""
    packed, absmax, state, _ = partition_quantized_tensor(
        full_weight, partition_info.rank, partition_info.world_size,
        partition_info.blocksize, quant_type, compute_dtype=full_weight.dtype
        if full_weight.dtype in (torch.float32, torch.float16, torch.bfloat16) else torch.float32)
    return packed, absmax, state


def estimate_memory_savings(numel: int, world_size: int,
                            original_dtype: torch.dtype = torch.float16) -> dict:
    """ZeRO-3 (fp16 shards) vs 4-bit shards, bytes per GPU (absmax counted as fp16,
    as the reference does at ``src/partition.py:436-438``)."""
    dtype_bytes = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}
    original_bytes = numel * dtype_bytes.get(original_dtype, 4)
    zero3_per_gpu = (numel * 2) // world_size
    packed_per_gpu = (numel // 2) // world_size
    absmax_per_gpu = (numel // 64) // world_size * 2
    zeroq_per_gpu = packed_per_gpu + absmax_per_gpu
    return {
        "original_total_bytes": original_bytes,
        "zero3_per_gpu_bytes": zero3_per_gpu,
        "zeroq_per_gpu_bytes": zeroq_per_gpu,
        "memory_reduction": zero3_per_gpu / zeroq_per_gpu if zeroq_per_gpu > 0 else 0,
        "communication_reduction": 2.0 / 0.53,
    }


def partition_fp32(tensor: torch.Tensor, world_size: int, rank: int
                   ) -> Tuple[torch.Tensor, torch.Size]:
    """Even ceil-split of a tensor as fp32; the last shard is zero-padded."""
    flat = tensor.detach().contiguous().view(-1).to(torch.float32)
    chunk = (flat.numel() + world_size - 1) // world_size
    start = rank * chunk
    end = min(start + chunk, flat.numel())
    shard = flat[start:end].clone() if start < flat.numel() else flat.new_zeros(0)
    if shard.numel() < chunk:
        shard = F.pad(shard, (0, chunk - shard.numel()))
    return shard, tensor.shape


def gather_fp32(local_shard: torch.Tensor, original_shape: torch.Size, world_size: int,
                group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    numel = 1
    for s in original_shape:
        numel *= int(s)
    if not dist.is_initialized() or world_size == 1:
        return local_shard[:numel].view(original_shape)
    full, _ = _all_gather_flat(local_shard, world_size, group)
    return full[:numel].view(original_shape)


def full_quant_state(meta: dict, absmax: torch.Tensor, device=None) -> QuantState:
    """Build a :class:`QuantState` from stored metadata and a gathered absmax."""
    return QuantState(absmax=absmax, shape=torch.Size(meta["shape"]), dtype=meta["dtype"],
                      blocksize=meta["blocksize"],
                      code=code_table(meta["quant_type"], device=device),
                      quant_type=meta["quant_type"])

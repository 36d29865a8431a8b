"""Blockwise 4-bit (NF4 / FP4) quantisation.

Storage format (kept byte-compatible with bitsandbytes' ``quantize_4bit`` so shards
and checkpoints interoperate with the reference, which calls it at
``src/partition.py:209`` and ``src/coordinator.py:174``):

* the tensor is flattened (row-major) and split into blocks of ``blocksize``
  consecutive values; the last block is zero-padded;
* ``absmax[b] = max |x|`` over block ``b`` (fp32);
* each value ``x`` maps to the index of the nearest code value of ``x / absmax``
  (ties resolve to the lower code);
* two 4-bit indices per byte, the even-indexed element in the HIGH nibble;
  ``packed`` has ``ceil(numel / 2)`` bytes.

The NF4 code values are the 16 normal-quantile levels of the QLoRA paper
(Dettmers et al. 2023, "QLoRA", appendix E); ``nf4_code_from_normal_quantiles``
rebuilds them from that construction and the tests check the two agree.  The FP4
table is bitsandbytes' sign/2-bit-exponent/1-bit-mantissa layout with the largest
magnitude normalised to 1.

CPU tensors go through the PyTorch implementation below (the oracle).  CUDA
tensors go through the sm_100a kernels in ``csrc/nf4.cu``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _ext

NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)

# index -> value for bitsandbytes' FP4 (bit 3 = sign; bits 2..0 = exponent/mantissa)
FP4_CODE = (
    0.0, 0.005208333333, 0.66666667, 1.0, 0.33333333, 0.5, 0.16666667, 0.25,
    -0.0, -0.005208333333, -0.66666667, -1.0, -0.33333333, -0.5, -0.16666667, -0.25,
)

QUANT_TYPE_ID = {"nf4": 0, "fp4": 1}


def nf4_code_from_normal_quantiles(offset: float = 0.9677083) -> list:
    """Rebuild the NF4 levels from the QLoRA construction (8 positive quantiles of
    N(0,1) between 0.5 and ``offset``, 7 negative ones, plus an exact zero, then
    normalised to [-1, 1])."""
    from scipy.stats import norm  # optional dependency, only used by tests

    import numpy as np

    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1]).tolist()
    neg = (-norm.ppf(np.linspace(offset, 0.5, 8)[:-1])).tolist()
    v = sorted(pos + [0.0] + neg)
    m = max(abs(x) for x in v)
    return [x / m for x in v]


def code_table(quant_type: str, device=None) -> torch.Tensor:
    if quant_type == "nf4":
        vals = NF4_CODE
    elif quant_type == "fp4":
        vals = FP4_CODE
    else:
        raise ValueError(f"unknown quant_type {quant_type!r}")
    return torch.tensor(vals, dtype=torch.float32, device=device)


@dataclass
class QuantState:
    """Metadata needed to dequantise a packed tensor.

    Field names follow bitsandbytes' ``QuantState`` (absmax, shape, dtype,
    blocksize, code, quant_type) because the reference rebuilds one from
    gathered shards (``src/coordinator.py:548-555``).
    """

    absmax: torch.Tensor
    shape: torch.Size
    dtype: torch.dtype
    blocksize: int = 64
    code: Optional[torch.Tensor] = None
    quant_type: str = "nf4"
    # double quantisation (8-bit absmax): when set, ``absmax`` holds uint8 codes
    nested_absmax: Optional[torch.Tensor] = None
    nested_offset: float = 0.0

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n

    def as_dict(self) -> dict:
        return {
            "shape": list(self.shape),
            "dtype": str(self.dtype),
            "blocksize": self.blocksize,
            "quant_type": self.quant_type,
        }


def _num_blocks(numel: int, blocksize: int) -> int:
    return (numel + blocksize - 1) // blocksize


# ----------------------------------------------------------------------------
# PyTorch reference implementation (the oracle; CPU path)
# ----------------------------------------------------------------------------

def _nearest_code_index(normed: torch.Tensor, quant_type: str) -> torch.Tensor:
    """Index of the nearest code value; ties go to the lower value (``x > mid``)."""
    if quant_type == "nf4":
        code = torch.tensor(NF4_CODE, dtype=torch.float32)
        mids = ((code[1:] + code[:-1]) * 0.5).to(normed.device)
        return torch.bucketize(normed, mids, right=False).to(torch.uint8)
    # fp4: sign bit + nearest magnitude among the 8 positive levels
    mag_vals = torch.tensor(FP4_CODE[:8], dtype=torch.float32)
    order = torch.argsort(mag_vals)
    sorted_vals = mag_vals[order]
    mids = ((sorted_vals[1:] + sorted_vals[:-1]) * 0.5).to(normed.device)
    pos = torch.bucketize(normed.abs(), mids, right=False)
    idx = order.to(normed.device)[pos]
    sign = (normed < 0).to(torch.int64) * 8
    return (idx + sign).to(torch.uint8)


def quantize_4bit_reference(
    x: torch.Tensor, blocksize: int = 64, quant_type: str = "nf4"
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns ``(packed uint8 [ceil(n/2)], absmax fp32 [ceil(n/blocksize)])``."""
    flat = x.detach().reshape(-1).to(torch.float32)
    n = flat.numel()
    nb = _num_blocks(n, blocksize)
    if nb * blocksize != n:
        flat = torch.nn.functional.pad(flat, (0, nb * blocksize - n))
    blocks = flat.view(nb, blocksize)
    absmax = blocks.abs().amax(dim=1)
    inv = torch.where(absmax > 0, 1.0 / absmax, torch.zeros_like(absmax))
    normed = blocks * inv[:, None]
    idx = _nearest_code_index(normed, quant_type).view(-1)
    if idx.numel() % 2:
        idx = torch.nn.functional.pad(idx, (0, 1))
    pairs = idx.view(-1, 2).to(torch.int32)
    packed = ((pairs[:, 0] << 4) | pairs[:, 1]).to(torch.uint8)
    return packed[: (n + 1) // 2].contiguous(), absmax.contiguous()


def dequantize_4bit_reference(
    packed: torch.Tensor,
    absmax: torch.Tensor,
    numel: int,
    blocksize: int = 64,
    quant_type: str = "nf4",
    out_dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    p = packed.reshape(-1).to(torch.int32)
    hi = (p >> 4) & 0xF
    lo = p & 0xF
    idx = torch.stack([hi, lo], dim=1).view(-1)[:numel]
    code = code_table(quant_type, device=packed.device)
    vals = code[idx.long()]
    nb = _num_blocks(numel, blocksize)
    scale = absmax.reshape(-1)[:nb].to(torch.float32).repeat_interleave(blocksize)[:numel]
    return (vals * scale).to(out_dtype)


# ----------------------------------------------------------------------------
# Public API (dispatches to the sm_100a kernels for CUDA tensors)
# ----------------------------------------------------------------------------

def quantize_4bit(
    x: torch.Tensor,
    blocksize: int = 64,
    quant_type: str = "nf4",
    out_packed: Optional[torch.Tensor] = None,
    out_absmax: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, QuantState]:
    """Quantise ``x`` (any float dtype, any shape) to packed 4-bit codes.

    Returns ``(packed, quant_state)`` like bitsandbytes' ``quantize_4bit``; the
    packed tensor is 1-D uint8.
    """
    if quant_type not in QUANT_TYPE_ID:
        raise ValueError(f"quant_type must be nf4 or fp4, got {quant_type!r}")
    if blocksize % 2 or blocksize < 2:
        raise ValueError("blocksize must be even")
    n = x.numel()
    if x.is_cuda:
        xc = x.detach().contiguous().view(-1)
        nb = _num_blocks(n, blocksize)
        packed = out_packed if out_packed is not None else torch.empty(
            (n + 1) // 2, dtype=torch.uint8, device=x.device)
        absmax = out_absmax if out_absmax is not None else torch.empty(
            nb, dtype=torch.float32, device=x.device)
        _ext.ext().nf4_quantize(xc, packed, absmax, blocksize, QUANT_TYPE_ID[quant_type])
    else:
        packed, absmax = quantize_4bit_reference(x, blocksize, quant_type)
        if out_packed is not None:
            out_packed.copy_(packed)
            packed = out_packed
        if out_absmax is not None:
            out_absmax.copy_(absmax)
            absmax = out_absmax
    state = QuantState(
        absmax=absmax, shape=x.shape, dtype=x.dtype, blocksize=blocksize,
        code=code_table(quant_type, device=x.device), quant_type=quant_type,
    )
    return packed, state


def dequantize_4bit(
    packed: torch.Tensor,
    quant_state: QuantState,
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Inverse of :func:`quantize_4bit`; returns a tensor of ``quant_state.shape``."""
    dtype = out_dtype or quant_state.dtype
    if dtype not in (torch.float32, torch.float16, torch.bfloat16):
        dtype = torch.float32
    absmax = quant_state.absmax
    if quant_state.nested_absmax is not None:
        absmax = dequantize_absmax(quant_state)
    n = quant_state.numel
    if packed.is_cuda:
        res = out if out is not None else torch.empty(n, dtype=dtype, device=packed.device)
        _ext.ext().nf4_dequantize(
            packed.contiguous().view(-1), absmax.contiguous().view(-1).float(), res.view(-1),
            n, quant_state.blocksize, QUANT_TYPE_ID[quant_state.quant_type])
        return res.view(quant_state.shape)
    res = dequantize_4bit_reference(packed, absmax, n, quant_state.blocksize,
                                    quant_state.quant_type, dtype)
    if out is not None:
        out.view(-1).copy_(res)
        res = out
    return res.view(quant_state.shape)


# ----------------------------------------------------------------------------
# Double quantisation: 8-bit blockwise absmax codec (``double_quant=True``)
# ----------------------------------------------------------------------------

def double_quantize_absmax(state: QuantState, blocksize: int = 256) -> QuantState:
    """Store ``absmax`` as uint8 with one fp32 scale per ``blocksize`` absmax values.

    The absmax values are positive; they are centred by their mean (``offset``)
    and linearly quantised to 255 levels per block.  This mirrors the purpose of
    bitsandbytes' ``compress_statistics`` (saving ~0.37 bits/param) with a plain
    linear codec.
    """
    a = state.absmax.float().reshape(-1)
    offset = float(a.mean()) if a.numel() else 0.0
    c = a - offset
    n = c.numel()
    nb = _num_blocks(n, blocksize)
    cp = torch.nn.functional.pad(c, (0, nb * blocksize - n)).view(nb, blocksize)
    scale = cp.abs().amax(dim=1).clamp_min(1e-12)
    q = torch.round(cp / scale[:, None] * 127.0).clamp(-127, 127).to(torch.int16) + 128
    return QuantState(
        absmax=q.to(torch.uint8).view(-1)[:n].contiguous(), shape=state.shape,
        dtype=state.dtype, blocksize=state.blocksize, code=state.code,
        quant_type=state.quant_type, nested_absmax=scale.contiguous(), nested_offset=offset,
    )


def dequantize_absmax(state: QuantState, blocksize: int = 256) -> torch.Tensor:
    q = state.absmax.to(torch.float32).reshape(-1) - 128.0
    n = q.numel()
    scale = state.nested_absmax.float().repeat_interleave(blocksize)[:n]
    return q / 127.0 * scale + state.nested_offset

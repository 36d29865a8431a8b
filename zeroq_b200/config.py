"""Configuration dataclasses for zeroq_b200.

Field names, defaults, validation and (de)serialisation follow the reference's
``src/config.py`` (``ZeroQConfig`` :12-143, presets :146-170, ``ZeroQTrainConfig``
:173-209, ``MultiNodeConfig`` :212-300) so a config written for the reference loads
here unchanged.

Additions that the reference declares but never reads, and which this framework
honours:

* ``async_gather`` / ``prefetch_count`` drive the layer prefetch pipeline of the
  gather/release mode (``zeroq_b200.parallel.prefetch``).
* ``double_quant`` selects an 8-bit absmax codec for stored shards
  (``zeroq_b200.ops.nf4.double_quantize_absmax``); it is off on the hot path
  because B200 has memory to spare and the fp32 absmax is what the fused GEMM
  reads.

New fields (not in the reference):

* ``backend``: ``"fused"`` runs this framework's sm_100a kernels (peer-memory
  gather fused with dequant + GEMM, reduce-scatter fused with AdamW),
  ``"nccl"`` runs the NCCL collectives + separate kernels (the baseline path),
  ``"torch"`` is the pure-PyTorch path (CPU, and the numerics oracle).
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields
from typing import List, Optional
import os
import socket

import torch

_VALID_QUANT_TYPES = ("nf4", "fp4")
_VALID_BLOCKSIZES = (64, 128, 256, 512, 1024, 2048, 4096)
_VALID_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_VALID_BACKENDS = ("auto", "fused", "nccl", "torch")

_DTYPE_FROM_STR = {
    "torch.float32": torch.float32,
    "torch.float16": torch.float16,
    "torch.bfloat16": torch.bfloat16,
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
}


def _dtype_from(value, default=torch.float32):
    if isinstance(value, torch.dtype):
        return value
    if isinstance(value, str):
        return _DTYPE_FROM_STR.get(value, default)
    return default


@dataclass
class ZeroQConfig:
    """Knobs for quantised, sharded training (reference ``src/config.py:12-96``).

    Attributes mirror the reference; see the module docstring for the fields
    this framework adds or actually wires up.
    """

    # Quantisation
    enabled: bool = True
    quant_type: str = "nf4"
    blocksize: int = 64
    double_quant: bool = True
    compute_dtype: torch.dtype = torch.float32

    # Partitioning
    partition_trainable: bool = False
    frozen_only: bool = True

    # Communication
    async_gather: bool = True
    prefetch_count: int = 1
    overlap_comm: bool = True

    # Memory
    pin_memory: bool = True
    contiguous_buffers: bool = True
    activation_reserve_mb: float = 0.0

    # 4-bit compute: frozen Linear weights stay NF4 and run through the fused
    # NF4-dequant GEMM instead of being dequantised to a full-precision copy.
    compute_in_4bit: bool = False
    # With compute_in_4bit: gather every weight once, keep it resident and drop
    # the gather/release hooks (True), or keep gathering per use (False, the
    # reference's hetero ``compute_in_4bit`` behaviour).
    gather_once: bool = False

    # Train-from-scratch: shard parameters as fp32 masters (no quantisation)
    training_mode: bool = False
    compress_between_steps: bool = False

    # Module targeting
    target_modules: Optional[List[str]] = None
    exclude_modules: List[str] = field(default_factory=lambda: ["lm_head"])

    # Kernel path selection (new in this framework)
    backend: str = "auto"

    def __post_init__(self):
        self._validate()

    def _validate(self):
        if self.quant_type not in _VALID_QUANT_TYPES:
            raise ValueError(
                f"quant_type must be one of {_VALID_QUANT_TYPES}, got {self.quant_type}"
            )
        if self.blocksize not in _VALID_BLOCKSIZES:
            raise ValueError(
                f"blocksize must be one of {_VALID_BLOCKSIZES}, got {self.blocksize}"
            )
        self.compute_dtype = _dtype_from(self.compute_dtype, self.compute_dtype)
        if self.compute_dtype not in _VALID_DTYPES:
            raise ValueError(
                f"compute_dtype must be one of {_VALID_DTYPES}, got {self.compute_dtype}"
            )
        if self.backend not in _VALID_BACKENDS:
            raise ValueError(f"backend must be one of {_VALID_BACKENDS}, got {self.backend}")

    def resolved_backend(self) -> str:
        """``auto`` -> ``fused`` when CUDA is present, else ``torch``."""
        if self.backend != "auto":
            return self.backend
        return "fused" if torch.cuda.is_available() else "torch"

    def to_dict(self) -> dict:
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            if isinstance(v, torch.dtype):
                v = str(v)
            elif isinstance(v, list):
                v = list(v)
            elif isinstance(v, dict):
                v = dict(v)
            out[f.name] = v
        return out

    @classmethod
    def from_dict(cls, d: dict) -> "ZeroQConfig":
        d = dict(d)
        known = {f.name for f in fields(cls)}
        for k in list(d):
            if k not in known:
                d.pop(k)
        for k in ("compute_dtype", "master_dtype"):
            if k in d and isinstance(d[k], str):
                d[k] = _dtype_from(d[k])
        return cls(**d)

    def __repr__(self) -> str:
        return (
            f"{type(self).__name__}(\n"
            f"  quant_type={self.quant_type!r},\n"
            f"  blocksize={self.blocksize},\n"
            f"  compute_dtype={self.compute_dtype},\n"
            f"  frozen_only={self.frozen_only},\n"
            f"  async_gather={self.async_gather},\n"
            f"  backend={self.backend!r},\n"
            f")"
        )


# Hardware presets (reference ``src/config.py:146-170``).  The B200 preset is new:
# bf16 compute, fused kernels, one layer of prefetch.
MAXWELL_CONFIG = ZeroQConfig(compute_dtype=torch.float32, double_quant=True, blocksize=64,
                             async_gather=True)
AMPERE_CONFIG = ZeroQConfig(compute_dtype=torch.bfloat16, double_quant=True, blocksize=64,
                            async_gather=True)
CONSUMER_CONFIG = ZeroQConfig(compute_dtype=torch.float16, double_quant=True, blocksize=64,
                              async_gather=True)
B200_CONFIG = ZeroQConfig(compute_dtype=torch.bfloat16, double_quant=False, blocksize=64,
                          async_gather=True, prefetch_count=1, backend="auto")


@dataclass
class ZeroQTrainConfig(ZeroQConfig):
    """Train-from-scratch config (reference ``src/config.py:173-201``).

    Validation runs only when ``compress_between_steps`` is set, as in the
    reference.
    """

    training_mode: bool = True
    frozen_only: bool = False
    partition_trainable: bool = True
    cpu_offload: bool = False
    master_dtype: torch.dtype = torch.float32
    fused_shard_step: bool = False
    lion_lr: float = 3e-4
    lion_beta1: float = 0.9
    lion_beta2: float = 0.99
    lion_wd: float = 0.01
    optimizer_cls: str = "AdamW"
    optimizer_kwargs: dict = field(default_factory=lambda: {"lr": 3e-4})

    def __post_init__(self):
        self.master_dtype = _dtype_from(self.master_dtype, self.master_dtype)
        if self.compress_between_steps:
            self._validate()


TRAIN_FROM_SCRATCH_CONFIG = ZeroQTrainConfig(
    compute_dtype=torch.float32,
    training_mode=True,
    frozen_only=False,
    partition_trainable=True,
)


@dataclass
class MultiNodeConfig:
    """Control-plane settings for the ZeroMQ transport (reference ``src/config.py:212-275``)."""

    enabled: bool = False
    coordinator_host: str = "localhost"
    coordinator_port: int = 5555
    node_id: str = ""
    local_hostname: str = "localhost"

    heartbeat_interval_sec: float = 5.0
    heartbeat_timeout_sec: float = 15.0

    use_hierarchical_sync: bool = True
    gradient_compression: bool = True
    compression_ratio: float = 0.01

    data_port_start: int = 5560
    tcp_buffer_size: int = 4 * 1024 * 1024

    def __post_init__(self):
        if not self.node_id:
            self.node_id = f"{socket.gethostname()}-{os.getpid()}"

    def to_dict(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)}

    @classmethod
    def from_dict(cls, d: dict) -> "MultiNodeConfig":
        return cls(**d)


PHOENIX_CLUSTER_CONFIG = MultiNodeConfig(
    enabled=True,
    coordinator_host="pe1",
    coordinator_port=5555,
    use_hierarchical_sync=True,
    gradient_compression=True,
    compression_ratio=0.01,
)

LOCAL_MULTINODE_CONFIG = MultiNodeConfig(
    enabled=True,
    coordinator_host="localhost",
    coordinator_port=5555,
    use_hierarchical_sync=False,
    gradient_compression=False,
)

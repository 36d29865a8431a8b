"""zeroq_b200 - quantised (NF4) ZeRO-style sharded training, built for B200 (sm_100a).

Public names follow the reference package ``zero_q`` (reference ``src/__init__.py``)
so code written against it switches by changing the import:

    >>> from zeroq_b200 import ZeroQConfig, initialize
    >>> model = initialize(model, ZeroQConfig(compute_in_4bit=True))

Everything the reference gates behind optional imports is always available
here (the quantiser is this package's own kernel, and pyzmq is in the image);
the ``HAS_*`` flags are kept for compatibility.
"""

from .config import (AMPERE_CONFIG, B200_CONFIG, CONSUMER_CONFIG, LOCAL_MULTINODE_CONFIG,
                     MAXWELL_CONFIG, PHOENIX_CLUSTER_CONFIG, TRAIN_FROM_SCRATCH_CONFIG,
                     MultiNodeConfig, ZeroQConfig, ZeroQTrainConfig)
from .parallel.partition import (PartitionInfo, compute_aligned_partition_sizes,
                                 estimate_memory_savings, gather_and_dequantize, gather_fp32,
                                 partition_fp32, partition_quantized_tensor, repartition_tensor)
from .parallel.coordinator import (ZeroQCoordinator, ZeroQModuleWrapper, ZeroQParameter,
                                   ZeroQParamStatus)
from .parallel.hetero import (HeteroZeroQCoordinator, HeteroZeroQModuleWrapper,
                              HeteroZeroQParameter, HeteroZeroQParamStatus, discover_rank_weights)
from .parallel.shard_plan import ShardPlan, compute_weighted_shard_lengths, make_plan
from .parallel.varlen import all_gather_varlen_1d
from .parallel.prefetch import LayerWiseZeroQ, PrefetchManager, create_prefetch_hooks
from .parallel.gradient_sync import (GradientAccumulator, GradSyncConfig, HierarchicalSync,
                                     RingAllReduce, SyncMode, TorchDistributedSync,
                                     create_gradient_sync, reduce_scatter_grads)
from .parallel.optimizer import FlatParams, ShardedAdamW
from .integration import (ZeroQTrainer, apply_lora_with_zeroq, convert_to_4bit_compute,
                          get_zeroq_memory_stats, initialize, inject_lora,
                          prepare_model_for_zeroq)
from .utils.checkpoint import (ZeroQCheckpointedModule, enable_gradient_checkpointing,
                               estimate_checkpoint_memory, load_adapters, load_sharded_checkpoint,
                               save_adapters, save_sharded_checkpoint)
from .ops.nf4 import QuantState, dequantize_4bit, quantize_4bit
from .ops.qlinear import Linear4bit

try:
    from .parallel.transport import (GradientCompressor, MessageType, NodeInfo, TransportConfig,
                                     TransportCoordinator, TransportWorker, create_transport,
                                     deserialize_tensor, serialize_tensor)
    HAS_TRANSPORT = True
except ImportError:  # pragma: no cover
    HAS_TRANSPORT = False

HAS_COORDINATOR = True
HAS_INTEGRATION = True
HAS_GRADIENT_SYNC = True

__version__ = "0.1.0"

__all__ = [
    "ZeroQConfig", "ZeroQTrainConfig", "MultiNodeConfig", "MAXWELL_CONFIG", "AMPERE_CONFIG",
    "CONSUMER_CONFIG", "B200_CONFIG", "TRAIN_FROM_SCRATCH_CONFIG", "PHOENIX_CLUSTER_CONFIG",
    "LOCAL_MULTINODE_CONFIG",
    "compute_aligned_partition_sizes", "partition_quantized_tensor", "gather_and_dequantize",
    "repartition_tensor", "estimate_memory_savings", "partition_fp32", "gather_fp32",
    "PartitionInfo",
    "ZeroQParamStatus", "ZeroQParameter", "ZeroQCoordinator", "ZeroQModuleWrapper",
    "HeteroZeroQParameter", "HeteroZeroQCoordinator", "HeteroZeroQModuleWrapper",
    "HeteroZeroQParamStatus", "discover_rank_weights", "ShardPlan", "make_plan",
    "compute_weighted_shard_lengths", "all_gather_varlen_1d",
    "PrefetchManager", "LayerWiseZeroQ", "create_prefetch_hooks",
    "SyncMode", "GradSyncConfig", "RingAllReduce", "TorchDistributedSync", "GradientAccumulator",
    "HierarchicalSync", "create_gradient_sync", "reduce_scatter_grads",
    "FlatParams", "ShardedAdamW",
    "initialize", "prepare_model_for_zeroq", "apply_lora_with_zeroq", "inject_lora",
    "convert_to_4bit_compute", "ZeroQTrainer", "get_zeroq_memory_stats",
    "enable_gradient_checkpointing", "ZeroQCheckpointedModule", "estimate_checkpoint_memory",
    "save_sharded_checkpoint", "load_sharded_checkpoint", "save_adapters", "load_adapters",
    "QuantState", "quantize_4bit", "dequantize_4bit", "Linear4bit",
    "TransportCoordinator", "TransportWorker", "TransportConfig", "MessageType", "NodeInfo",
    "GradientCompressor", "create_transport", "serialize_tensor", "deserialize_tensor",
    "HAS_COORDINATOR", "HAS_INTEGRATION", "HAS_TRANSPORT", "HAS_GRADIENT_SYNC",
]

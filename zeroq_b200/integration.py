"""User-facing setup API (reference ``src/integration.py``).

* :func:`prepare_model_for_zeroq` - freeze the base, unfreeze adapters, build a
  coordinator + hook wrapper, quantise and shard (reference :35-90).  With
  ``config.compute_in_4bit`` gathered Linear4bit weights stay NF4 per use; with
  ``gather_once`` as well it switches the model to resident 4-bit compute: every
  :class:`~zeroq_b200.ops.qlinear.Linear4bit` gathers its full NF4 weight ONCE and
  keeps it resident, other sharded params are gathered once and kept, and the
  gather/release hooks are removed - the mode the reference's README describes
  for its 4.7B decoder (``README.md:17,109``).
* :func:`apply_lora_with_zeroq` / :func:`inject_lora` - LoRA adapters with PEFT's
  names.  PEFT is used when importable; otherwise adapters are added to
  :class:`Linear4bit` modules directly (``lora_A``, ``lora_B``, ``alpha / r``).
* :func:`initialize`, :func:`get_zeroq_memory_stats`, :class:`ZeroQTrainer`.
"""

from __future__ import annotations

from typing import Dict, Iterable, Optional, Sequence

import torch
import torch.nn as nn
import torch.distributed as dist

from .config import B200_CONFIG, ZeroQConfig
from .ops.qlinear import Linear4bit
from .parallel.coordinator import ZeroQCoordinator, ZeroQModuleWrapper, ZeroQParamStatus
from .parallel.hetero import HeteroZeroQCoordinator, HeteroZeroQModuleWrapper

try:
    from transformers import Trainer as _HFTrainer

    HAS_TRANSFORMERS = True
except Exception:  # pragma: no cover
    _HFTrainer = object
    HAS_TRANSFORMERS = False

try:
    from peft import PeftModel, get_peft_model  # type: ignore

    HAS_PEFT = True
except Exception:
    PeftModel = None
    get_peft_model = None
    HAS_PEFT = False


def _lora_cfg_value(cfg, name, default=None):
    if isinstance(cfg, dict):
        return cfg.get(name, default)
    return getattr(cfg, name, default)


def inject_lora(model: nn.Module, r: int, lora_alpha: float,
                target_modules: Sequence[str]) -> nn.Module:
    """Add LoRA adapters to every projection whose name ends with a target.

    ``nn.Linear`` modules are replaced by :class:`Linear4bit` holding the same
    (still full-precision) weight, so the coordinator can shard and quantise it.
    """
    targets = tuple(target_modules)
    for name, mod in list(model.named_modules()):
        leaf = name.rsplit(".", 1)[-1]
        if not any(leaf == t or name.endswith(t) for t in targets):
            continue
        if isinstance(mod, Linear4bit):
            if mod.lora_r == 0:
                dev = mod.weight.device if mod.weight.numel() else (
                    mod.weight_packed.device if mod.has_nf4 else None)
                mod.lora_r = r
                mod.scaling = lora_alpha / r
                mod.lora_A = nn.Parameter(torch.empty(r, mod.in_features, device=dev))
                mod.lora_B = nn.Parameter(torch.zeros(mod.out_features, r, device=dev))
                nn.init.kaiming_uniform_(mod.lora_A, a=5 ** 0.5)
        elif isinstance(mod, nn.Linear):
            new = Linear4bit(mod.in_features, mod.out_features, bias=mod.bias is not None,
                             lora_r=r, lora_alpha=lora_alpha, device=mod.weight.device,
                             dtype=mod.weight.dtype)
            new.weight = nn.Parameter(mod.weight.data, requires_grad=False)
            if mod.bias is not None:
                new.bias.data.copy_(mod.bias.data)
            parent = model.get_submodule(name.rsplit(".", 1)[0]) if "." in name else model
            setattr(parent, leaf, new)
    return model


def _freeze_base(model: nn.Module, trainable_patterns: Iterable[str]):
    pats = tuple(trainable_patterns)
    for n, p in model.named_parameters():
        p.requires_grad = any(t in n.lower() for t in pats)


def convert_to_4bit_compute(model: nn.Module, coordinator: ZeroQCoordinator,
                            wrapper: Optional[ZeroQModuleWrapper] = None) -> int:
    """Gather every sharded weight once and keep it; remove the per-use hooks.

    Linear4bit weights stay NF4 (packed + absmax) and run through the fused
    GEMM; anything else is dequantised once.  Returns the number of converted
    parameters.
    """
    count = 0
    for zq in coordinator._params.values():
        if zq.local_packed is None:
            continue
        # Resident means a local copy: the gather assembles the whole NF4 weight
        # here once (with a peer pool registered, through the peer plan-gather
        # kernel).  A peer source would re-read every owner's shard over NVLink on
        # every use and rule out the fused q/k/v GEMM and its epilogues, so a
        # parameter that a forward hook already attached to its peer source is
        # released first.
        if zq.status == ZeroQParamStatus.AVAILABLE and getattr(zq.module, "_peer", None) is not None:
            zq.release()
        zq.start_gather(group=coordinator.process_group, async_op=False, force_local=True)
        if zq.status == ZeroQParamStatus.INFLIGHT:
            zq.wait_gather()
        if isinstance(zq.module, Linear4bit) and zq.param_name == "weight":
            if zq.module._peer is not None:
                raise RuntimeError(f"convert_to_4bit_compute: param_id={zq.param_id} is still "
                                   "attached to its peer shards after the local gather")
            if not zq.compute_in_4bit:
                # dequantised during the gather; quantised again for NF4 compute
                zq.module.quantize_from(zq.module.weight.data)
                zq.module.weight = nn.Parameter(torch.empty(0, device=zq.module.weight.device,
                                                            dtype=zq.original_dtype),
                                                requires_grad=False)
            # keep the gathered NF4 resident: the coordinator forgets it
        zq.status = ZeroQParamStatus.NOT_AVAILABLE
        zq._assembled_packed = zq._assembled_absmax = None
        count += 1
    if wrapper is not None:
        wrapper.remove_hooks()
    return count


def prepare_model_for_zeroq(model: nn.Module, config: Optional[ZeroQConfig] = None,
                            freeze_base: bool = True,
                            trainable_patterns: Iterable[str] = ("lora_",),
                            rank_weights: Optional[Sequence[float]] = None,
                            process_group=None, checkpoint: Optional[str] = None) -> nn.Module:
    """Freeze, register, quantise and shard; optionally switch to 4-bit compute.

    With ``checkpoint`` (a safetensors file or directory, Hugging Face
    Llama/Qwen2 names) the frozen weights are read tensor by tensor and sharded
    on arrival (:func:`zeroq_b200.utils.loading.stream_load`): register the model
    with meta-device projection weights (``DecoderLM.init_meta_``) and no rank
    ever holds the full model in full precision."""
    config = config or B200_CONFIG
    if freeze_base:
        _freeze_base(model, trainable_patterns)
    hetero = rank_weights is not None
    if hetero:
        coordinator = HeteroZeroQCoordinator(config, process_group, rank_weights=list(rank_weights))
        wrapper = HeteroZeroQModuleWrapper(model, coordinator, trainable_only=False)
    else:
        coordinator = ZeroQCoordinator(config, process_group)
        wrapper = ZeroQModuleWrapper(model, coordinator, trainable_only=False)
    if checkpoint is not None:
        from .utils.loading import stream_load

        model._zeroq_load_counts = stream_load(model, checkpoint, coordinator)
    else:
        wrapper.partition()
    if hetero:
        coordinator.verify_registration_consistency()
    if (config.resolved_backend() == "fused" and coordinator.world_size > 1
            and torch.cuda.is_available() and dist.is_initialized()
            and dist.get_backend(process_group) == "nccl"):
        from .parallel.peer import PeerShardPool

        coordinator.peer_pool = PeerShardPool(coordinator, process_group)
    if getattr(config, "compute_in_4bit", False) and getattr(config, "gather_once", False):
        convert_to_4bit_compute(model, coordinator, wrapper)
        wrapper = None
    model._zeroq_wrapper = wrapper
    model._zeroq_coordinator = coordinator
    model._zeroq_config = config
    return model


def get_zeroq_memory_stats(model: nn.Module) -> Dict[str, float]:
    coord = getattr(model, "_zeroq_coordinator", None)
    return coord.get_memory_stats() if coord is not None else {}


def apply_lora_with_zeroq(model: nn.Module, lora_config, zeroq_config: Optional[ZeroQConfig] = None,
                          **kwargs) -> nn.Module:
    """Add LoRA adapters, then :func:`prepare_model_for_zeroq` (reference :164-209)."""
    if HAS_PEFT and lora_config.__class__.__module__.startswith("peft"):
        model = get_peft_model(model, lora_config)
    else:
        r = int(_lora_cfg_value(lora_config, "r", 8))
        alpha = float(_lora_cfg_value(lora_config, "lora_alpha", 16))
        targets = _lora_cfg_value(lora_config, "target_modules", ["q_proj", "v_proj"])
        inject_lora(model, r, alpha, targets)
    return prepare_model_for_zeroq(model, zeroq_config, freeze_base=True, **kwargs)


def initialize(model: nn.Module, config: Optional[ZeroQConfig] = None, lora_config=None,
               **kwargs) -> nn.Module:
    """One-call setup (reference :213-237)."""
    if lora_config is not None:
        return apply_lora_with_zeroq(model, lora_config, config, **kwargs)
    return prepare_model_for_zeroq(model, config, **kwargs)


class ZeroQTrainer(_HFTrainer):
    """HF ``Trainer`` that prepares the model for ZeRO-Q first (reference :100-161)."""

    def __init__(self, model: nn.Module = None, args=None, zeroq_config: Optional[ZeroQConfig] = None,
                 **kwargs):
        if not HAS_TRANSFORMERS:
            raise ImportError("ZeroQTrainer requires transformers")
        self.zeroq_config = zeroq_config or B200_CONFIG
        if model is not None and not hasattr(model, "_zeroq_coordinator"):
            model = prepare_model_for_zeroq(model, self.zeroq_config)
        super().__init__(model=model, args=args, **kwargs)

    def log_zeroq_stats(self):
        st = get_zeroq_memory_stats(self.model)
        if st:
            self.log({"zeroq/local_memory_mb": st.get("local_memory_mb", 0),
                      "zeroq/compression_ratio": st.get("compression_ratio", 1),
                      "zeroq/num_params": st.get("num_params", 0)})

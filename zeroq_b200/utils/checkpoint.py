"""Activation checkpointing and training-state checkpoints.

Activation checkpointing keeps the reference's API (``src/checkpoint.py``):
:func:`enable_gradient_checkpointing` finds the layer list (``model.layers``,
``transformer.h``, ``encoder.layer``, ``decoder.layers``, or a model's own
``layers``) and wraps each layer's forward in ``torch.utils.checkpoint``;
:class:`ZeroQCheckpointedModule` and :func:`estimate_checkpoint_memory` as there.

State checkpoints (the reference only saves PEFT adapters, and its
``gather_full_state_dict`` keys tensors by ``id(module)``):

* :func:`save_sharded_checkpoint` / :func:`load_sharded_checkpoint` - one file
  per rank with every parameter's shard (NF4 packed bytes in bitsandbytes
  layout, fp32 absmax, quantisation metadata, shard plans), master shards,
  the trainable parameters, optimizer state and the step, written with
  safetensors for tensors plus a JSON manifest.  Resuming requires the same
  world size and plans; the manifest records both.
* :func:`save_adapters` / :func:`load_adapters` - LoRA weights under PEFT's
  ``base_model.model.<path>.lora_A.weight`` key names.
"""

from __future__ import annotations

import json
import os
from typing import Dict, List, Optional

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint

_LAYER_PATTERNS = ["model.layers", "transformer.h", "encoder.layer", "decoder.layers", "layers"]


def _auto_detect_layers(model: nn.Module) -> List[str]:
    for pat in _LAYER_PATTERNS:
        cur = model
        ok = True
        for part in pat.split("."):
            if not hasattr(cur, part):
                ok = False
                break
            cur = getattr(cur, part)
        if ok and isinstance(cur, (nn.ModuleList, list)):
            return [f"{pat}.{i}" for i in range(len(cur))]
    return []


def _get_layer_by_name(model: nn.Module, name: str) -> Optional[nn.Module]:
    cur = model
    for part in name.split("."):
        if hasattr(cur, part):
            cur = getattr(cur, part)
        elif isinstance(cur, (nn.ModuleList, list)) and part.isdigit():
            cur = cur[int(part)]
        else:
            return None
    return cur


def _wrap_layer_with_checkpoint(layer: nn.Module, use_reentrant: bool):
    if getattr(layer, "_zq_ckpt_wrapped", False):
        return
    original = layer.forward

    def checkpointed_forward(*args, **kwargs):
        if torch.is_grad_enabled():
            return checkpoint(original, *args, use_reentrant=use_reentrant, **kwargs)
        return original(*args, **kwargs)

    layer.forward = checkpointed_forward
    layer._zq_ckpt_wrapped = True


def enable_gradient_checkpointing(model: nn.Module, checkpoint_layers: Optional[List[str]] = None,
                                  use_reentrant: bool = False):
    if checkpoint_layers is None:
        checkpoint_layers = _auto_detect_layers(model)
    if not checkpoint_layers:
        if hasattr(model, "gradient_checkpointing_enable"):
            model.gradient_checkpointing_enable(
                gradient_checkpointing_kwargs={"use_reentrant": use_reentrant})
        return
    for name in checkpoint_layers:
        layer = _get_layer_by_name(model, name)
        if layer is not None:
            _wrap_layer_with_checkpoint(layer, use_reentrant)


class ZeroQCheckpointedModule(nn.Module):
    def __init__(self, module: nn.Module, coordinator=None,
                 checkpoint_layers: Optional[List[str]] = None, use_reentrant: bool = False):
        super().__init__()
        self.module = module
        self.coordinator = coordinator
        self.checkpoint_layers = checkpoint_layers or _auto_detect_layers(module)
        self.use_reentrant = use_reentrant
        enable_gradient_checkpointing(self.module, self.checkpoint_layers, use_reentrant)

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    @property
    def memory_estimate(self) -> dict:
        q = sum(p.numel() * 0.5 for p in self.module.parameters() if not p.requires_grad)
        t = sum(p.numel() * p.element_size() for p in self.module.parameters() if p.requires_grad)
        n = len(self.checkpoint_layers) if self.checkpoint_layers else 32
        f = n ** 0.5 / n
        return {"quantized_params_mb": q / 2 ** 20, "trainable_params_mb": t / 2 ** 20,
                "activation_reduction": f"{1 / f:.1f}x fewer stored activations"}


def estimate_checkpoint_memory(hidden_size: int, num_layers: int, batch_size: int, seq_len: int,
                               with_checkpointing: bool = True) -> dict:
    """Rough activation bytes (fp16), O(sqrt(L)) layers stored with checkpointing."""
    bpe = 2
    attn = batch_size * seq_len * hidden_size * 4 + batch_size * seq_len * seq_len
    mlp = batch_size * seq_len * hidden_size * 3
    per_layer = (attn + mlp) * bpe
    eff = num_layers ** 0.5 if with_checkpointing else num_layers
    return {"per_layer_mb": per_layer / 2 ** 20, "total_mb": per_layer * eff / 2 ** 20,
            "effective_layers": eff,
            "savings": num_layers / eff if with_checkpointing else 1.0}


# ----------------------------------------------------------------------------
# training-state checkpoints
# ----------------------------------------------------------------------------

def _flatten_for_safetensors(prefix: str, d: Dict, tensors: Dict, meta: Dict):
    for k, v in d.items():
        key = f"{prefix}{k}"
        if isinstance(v, torch.Tensor):
            tensors[key] = v.detach().cpu().clone()
        elif isinstance(v, dict):
            _flatten_for_safetensors(key + "/", v, tensors, meta)
        else:
            meta[key] = v


def save_sharded_checkpoint(path: str, model: nn.Module, optimizer=None, step: int = 0,
                            config=None, rank: Optional[int] = None,
                            world_size: Optional[int] = None) -> str:
    """Write this rank's shards + trainable params + optimizer state to ``path``."""
    from safetensors.torch import save_file
    import torch.distributed as dist

    rank = rank if rank is not None else (dist.get_rank() if dist.is_initialized() else 0)
    world_size = world_size if world_size is not None else (
        dist.get_world_size() if dist.is_initialized() else 1)
    os.makedirs(path, exist_ok=True)
    tensors: Dict[str, torch.Tensor] = {}
    meta: Dict = {"step": int(step), "rank": rank, "world_size": world_size, "format": 1}
    coord = getattr(model, "_zeroq_coordinator", None)
    if coord is not None:
        for pid, zq in coord._params.items():
            _flatten_for_safetensors(f"shard/{pid}/", zq.shard_state(), tensors, meta)
    for name, mod in model.named_modules():
        if getattr(mod, "has_nf4", False) and mod.weight_packed is not None:
            tensors[f"nf4/{name}/packed"] = mod.weight_packed.detach().cpu().clone()
            tensors[f"nf4/{name}/absmax"] = mod.weight_absmax.detach().cpu().clone()
    for name, p in model.named_parameters():
        if p.requires_grad:
            tensors[f"param/{name}"] = p.detach().cpu().clone()
    if optimizer is not None and hasattr(optimizer, "state_dict"):
        _flatten_for_safetensors("optim/", optimizer.state_dict(), tensors, meta)
    if config is not None and hasattr(config, "to_dict"):
        meta["config"] = config.to_dict()
    fn = os.path.join(path, f"rank{rank:05d}.safetensors")
    save_file(tensors, fn)
    with open(os.path.join(path, f"rank{rank:05d}.json"), "w") as f:
        json.dump(meta, f, default=str, indent=1)
    return fn


def load_sharded_checkpoint(path: str, model: nn.Module, optimizer=None,
                            rank: Optional[int] = None) -> int:
    """Restore what :func:`save_sharded_checkpoint` wrote for this rank; returns the step."""
    from safetensors.torch import load_file
    import torch.distributed as dist

    rank = rank if rank is not None else (dist.get_rank() if dist.is_initialized() else 0)
    tensors = load_file(os.path.join(path, f"rank{rank:05d}.safetensors"))
    with open(os.path.join(path, f"rank{rank:05d}.json")) as f:
        meta = json.load(f)
    ws = dist.get_world_size() if dist.is_initialized() else 1
    if int(meta["world_size"]) != ws:
        raise ValueError(f"checkpoint was written by {meta['world_size']} ranks, running {ws}")
    coord = getattr(model, "_zeroq_coordinator", None)
    if coord is not None:
        for pid, zq in coord._params.items():
            pre = f"shard/{pid}/"
            st = {k[len(pre):]: v for k, v in tensors.items() if k.startswith(pre)}
            st.update({k[len(pre):]: v for k, v in meta.items() if k.startswith(pre)})
            if st:
                if "local_packed" in st:
                    qm = {k[len("quant_meta/"):]: v for k, v in st.items()
                          if k.startswith("quant_meta/")}
                    st["quant_meta"] = qm
                zq.load_shard_state(st)
    mods = dict(model.named_modules())
    for k, v in tensors.items():
        if k.startswith("nf4/") and k.endswith("/packed"):
            name = k[len("nf4/"):-len("/packed")]
            mods[name].set_nf4(v.to(_module_device(mods[name])),
                               tensors[f"nf4/{name}/absmax"].to(_module_device(mods[name])))
    zcfg = getattr(model, "_zeroq_config", None)
    if (coord is not None and getattr(model, "_zeroq_wrapper", "hooks") is None
            and getattr(zcfg, "gather_once", False)):
        # gather-once mode has no hooks to gather again: rebuild the resident
        # weights (NF4 for Linear4bit, dequantised for the rest) from the shards
        from ..integration import convert_to_4bit_compute

        convert_to_4bit_compute(model, coord, None)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for k, v in tensors.items():
            if k.startswith("param/"):
                params[k[len("param/"):]].copy_(v)
    if optimizer is not None and hasattr(optimizer, "load_state_dict"):
        st = {k[len("optim/"):]: v for k, v in tensors.items() if k.startswith("optim/")}
        st.update({k[len("optim/"):]: v for k, v in meta.items() if k.startswith("optim/")})
        optimizer.load_state_dict(st)
    return int(meta["step"])


def _module_device(mod: nn.Module) -> torch.device:
    for t in list(mod.parameters()) + list(mod.buffers()):
        if t is not None and t.numel():
            return t.device
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def save_adapters(model: nn.Module, path: str, prefix: str = "base_model.model.") -> str:
    """LoRA weights in PEFT's key layout (``<prefix><module>.lora_A.weight``)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    out = {}
    cfg = {"r": None, "lora_alpha": None, "target_modules": set()}
    for name, mod in model.named_modules():
        if getattr(mod, "lora_r", 0):
            out[f"{prefix}{name}.lora_A.weight"] = mod.lora_A.detach().cpu().contiguous()
            out[f"{prefix}{name}.lora_B.weight"] = mod.lora_B.detach().cpu().contiguous()
            cfg["r"] = mod.lora_r
            cfg["lora_alpha"] = mod.scaling * mod.lora_r
            cfg["target_modules"].add(name.rsplit(".", 1)[-1])
    save_file(out, os.path.join(path, "adapter_model.safetensors"))
    cfg["target_modules"] = sorted(cfg["target_modules"])
    cfg["peft_type"] = "LORA"
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path


def load_adapters(model: nn.Module, path: str, prefix: str = "base_model.model.") -> int:
    from safetensors.torch import load_file

    sd = load_file(os.path.join(path, "adapter_model.safetensors"))
    n = 0
    mods = dict(model.named_modules())
    with torch.no_grad():
        for k, v in sd.items():
            name = k[len(prefix):] if k.startswith(prefix) else k
            mname, which, _ = name.rsplit(".", 2)
            mod = mods[mname]
            getattr(mod, which).copy_(v)
            n += 1
    return n

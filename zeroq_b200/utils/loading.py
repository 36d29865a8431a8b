"""Streamed checkpoint loading straight into ZeRO-Q shards.

The reference's production trainer builds a meta-device skeleton, then reads
the safetensors files tensor by tensor and hands each frozen weight to
``partition_from_full_precision`` so that no rank ever holds the full model in
full precision (``examples/train_32b_maxwell.py:413-470`` there).  This module
does the same for :class:`zeroq_b200.models.DecoderLM`:

* :func:`hf_to_decoder_name` maps Hugging Face Llama/Qwen2 parameter names
  (``model.layers.3.self_attn.q_proj.weight`` ...) to this framework's names
  (``layers.3.q_proj.weight`` ...);
* :func:`stream_load` walks ``*.safetensors`` files one tensor at a time: a
  weight registered with the coordinator is quantised and sharded on arrival
  (this rank keeps only its shard), anything else (norms, embeddings, the head,
  biases that are not registered) is copied into the module; the vocabulary
  padding rows stay zero.
"""

from __future__ import annotations

import glob
import os
import re
from typing import Callable, Dict, Iterable, Optional, Tuple

import torch
import torch.nn as nn

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
_SUFFIX = {
    "input_layernorm.weight": "attn_norm.weight",
    "post_attention_layernorm.weight": "mlp_norm.weight",
    "self_attn.q_proj.weight": "q_proj.weight",
    "self_attn.k_proj.weight": "k_proj.weight",
    "self_attn.v_proj.weight": "v_proj.weight",
    "self_attn.o_proj.weight": "o_proj.weight",
    "self_attn.q_proj.bias": "q_proj.bias",
    "self_attn.k_proj.bias": "k_proj.bias",
    "self_attn.v_proj.bias": "v_proj.bias",
    "mlp.gate_proj.weight": "gate_proj.weight",
    "mlp.up_proj.weight": "up_proj.weight",
    "mlp.down_proj.weight": "down_proj.weight",
}


def hf_to_decoder_name(name: str) -> Optional[str]:
    """Hugging Face Llama/Qwen2 parameter name -> DecoderLM name (None if unused)."""
    if name == "model.embed_tokens.weight":
        return "embed_tokens.weight"
    if name == "model.norm.weight":
        return "norm.weight"
    if name == "lm_head.weight":
        return "lm_head.weight"
    m = _LAYER.match(name)
    if m and m.group(2) in _SUFFIX:
        return f"layers.{m.group(1)}.{_SUFFIX[m.group(2)]}"
    return None


def _iter_safetensors(path: str) -> Iterable[Tuple[str, torch.Tensor]]:
    from safetensors import safe_open

    files = sorted(glob.glob(os.path.join(path, "*.safetensors"))) if os.path.isdir(path) else [path]
    if not files:
        raise FileNotFoundError(f"no .safetensors files under {path}")
    for fn in files:
        with safe_open(fn, framework="pt", device="cpu") as f:
            for key in f.keys():
                yield key, f.get_tensor(key)


def _resolve(model: nn.Module, name: str) -> Tuple[nn.Module, str]:
    mod_path, _, attr = name.rpartition(".")
    return (model.get_submodule(mod_path) if mod_path else model), attr


def stream_load(model: nn.Module, checkpoint: str, coordinator=None,
                device: Optional[torch.device] = None,
                name_map: Callable[[str], Optional[str]] = hf_to_decoder_name) -> Dict[str, int]:
    """Load ``checkpoint`` (a directory of safetensors files or one file) into
    ``model``; weights registered with ``coordinator`` are sharded as they arrive.

    Returns counts: ``sharded``, ``copied``, ``skipped``.
    """
    registered = {}
    if coordinator is not None:
        for zq in coordinator._params.values():
            if zq.module is not None and zq.param_name is not None:
                registered[(id(zq.module), zq.param_name)] = zq
    counts = {"sharded": 0, "copied": 0, "skipped": 0}
    for key, tensor in _iter_safetensors(checkpoint):
        name = name_map(key)
        if name is None:
            counts["skipped"] += 1
            continue
        try:
            module, attr = _resolve(model, name)
        except AttributeError:
            counts["skipped"] += 1
            continue
        if getattr(module, attr, None) is None:
            counts["skipped"] += 1
            continue
        zq = registered.get((id(module), attr))
        if zq is not None:
            if device is not None:
                target = device
            elif torch.cuda.is_available():
                target = torch.device("cuda", torch.cuda.current_device())
            else:
                target = torch.device("cpu")
            zq.partition_from_full_precision(tensor.to(target))
            counts["sharded"] += 1
            continue
        param = getattr(module, attr)
        with torch.no_grad():
            if param.device.type == "meta":
                new = nn.Parameter(torch.empty(param.shape, dtype=param.dtype,
                                               device=device or "cpu"),
                                   requires_grad=param.requires_grad)
                setattr(module, attr, new)
                param = new
            src = tensor.to(device=param.device, dtype=param.dtype)
            if src.shape != param.shape:
                if src.dim() == 2 and param.dim() == 2 and src.shape[1] == param.shape[1] \
                        and src.shape[0] <= param.shape[0]:
                    param.zero_()                  # vocabulary padding rows stay zero
                    param[: src.shape[0]].copy_(src)
                else:
                    raise ValueError(f"{key}: checkpoint shape {tuple(src.shape)} does not fit "
                                     f"{name} {tuple(param.shape)}")
            else:
                param.copy_(src)
        counts["copied"] += 1
    return counts


def save_hf_checkpoint(model: nn.Module, path: str, vocab_size: Optional[int] = None) -> None:
    """Write a dense DecoderLM (before quantisation) as one safetensors file with
    Hugging Face Llama/Qwen2 names (the inverse of :func:`hf_to_decoder_name`)."""
    from safetensors.torch import save_file

    inv = {}
    for i in range(len(getattr(model, "layers", []))):
        for hf, ours in _SUFFIX.items():
            inv[f"layers.{i}.{ours}"] = f"model.layers.{i}.{hf}"
    inv["embed_tokens.weight"] = "model.embed_tokens.weight"
    inv["norm.weight"] = "model.norm.weight"
    inv["lm_head.weight"] = "lm_head.weight"
    out = {}
    for name, p in model.named_parameters():
        if name in inv and p.numel() and p.device.type != "meta":
            t = p.detach().cpu().contiguous()
            if vocab_size is not None and name in ("embed_tokens.weight", "lm_head.weight"):
                t = t[:vocab_size].contiguous()
            out[inv[name]] = t
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    save_file(out, path)


__all__ = ["hf_to_decoder_name", "stream_load", "save_hf_checkpoint"]

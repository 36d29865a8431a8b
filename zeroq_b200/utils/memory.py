"""Analytical per-GPU memory model (reference ``tools/memory_calculator.py`` and
``src/partition.py:413-451``), sized for 180 GB B200s.

:func:`estimate_zeroq_memory` returns bytes per GPU for the weights (NF4 shards
or resident NF4 in 4-bit compute mode, plus the transient gathered layer),
trainable parameters with fp32 AdamW state, activations (with or without
activation checkpointing) and the logits buffer.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

from ..parallel.partition import estimate_memory_savings  # noqa: F401  (re-export)

GiB = 1024 ** 3


@dataclass
class MemoryEstimate:
    weights_gb: float
    gathered_layer_gb: float
    trainable_gb: float
    optimizer_gb: float
    activations_gb: float
    logits_gb: float

    @property
    def total_gb(self) -> float:
        return (self.weights_gb + self.gathered_layer_gb + self.trainable_gb + self.optimizer_gb
                + self.activations_gb + self.logits_gb)

    def as_dict(self) -> dict:
        d = dict(self.__dict__)
        d["total_gb"] = self.total_gb
        return d


def estimate_zeroq_memory(cfg, batch: int, seq: int, world_size: int = 1, mode: str = "4bit",
                          activation_checkpointing: Optional[bool] = None,
                          blocksize: int = 64) -> MemoryEstimate:
    """``mode``: ``"4bit"`` (NF4 resident, replicated), ``"gather"`` (NF4 sharded, one
    layer gathered at a time) or ``"bf16"`` (dense replicated, for comparison)."""
    d, L = cfg.d_model, cfg.n_layers
    per_layer = (d * cfg.n_heads * cfg.head_dim * 2 + d * cfg.n_kv_heads * cfg.head_dim * 2
                 + d * cfg.ffn_dim * (3 if cfg.ffn_act == "swiglu" else 2))
    nf4_bpe = 0.5 + 4.0 / blocksize
    if mode == "4bit":
        weights = per_layer * L * nf4_bpe
        gathered = 0.0
    elif mode == "gather":
        weights = per_layer * L * nf4_bpe / world_size
        gathered = per_layer * (nf4_bpe + 2.0) * 2  # current + prefetched layer
    else:
        weights = per_layer * L * 2.0
        gathered = 0.0
    emb = cfg.vocab_padded * d * 2 * (1 if cfg.tie_embeddings else 2)
    lora = 0
    if cfg.lora_r:
        for t in cfg.lora_targets:
            if t in ("q_proj", "o_proj"):
                i, o = d, cfg.n_heads * cfg.head_dim
            elif t in ("k_proj", "v_proj"):
                i, o = d, cfg.n_kv_heads * cfg.head_dim
            else:
                i, o = d, cfg.ffn_dim
            lora += cfg.lora_r * (i + o)
        lora *= L
    trainable = (lora + 2 * d * L + d) * 4.0
    optim = trainable * 2 / world_size
    ckpt = cfg.activation_checkpointing if activation_checkpointing is None else activation_checkpointing
    tok = batch * seq
    # saved per layer (bf16): residual, 2 norm outputs, q, k, v, o, 2 ffn tensors, LoRA U
    act_layer = tok * (d * 4 + cfg.n_heads * cfg.head_dim * 2 + cfg.n_kv_heads * cfg.head_dim * 2
                       + cfg.ffn_dim * (3 if cfg.ffn_act == "swiglu" else 2)) * 2.0
    acts = tok * d * 2.0 * L + act_layer if ckpt else act_layer * L
    logits = tok * cfg.vocab_padded * 2.0
    return MemoryEstimate(weights_gb=(weights + emb) / GiB, gathered_layer_gb=gathered / GiB,
                          trainable_gb=trainable / GiB, optimizer_gb=optim / GiB,
                          activations_gb=acts / GiB, logits_gb=logits / GiB)


def main(argv=None):  # pragma: no cover - CLI
    import argparse
    import json

    from ..models.decoder import get_config

    ap = argparse.ArgumentParser(description="Per-GPU memory estimate")
    ap.add_argument("--model", default="4.7b")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--mode", default="4bit", choices=["4bit", "gather", "bf16"])
    ap.add_argument("--lora-r", type=int, default=16)
    a = ap.parse_args(argv)
    cfg = get_config(a.model, lora_r=a.lora_r)
    print(json.dumps(estimate_zeroq_memory(cfg, a.batch, a.seq, a.gpus, a.mode).as_dict(), indent=1))


if __name__ == "__main__":  # pragma: no cover
    main()

"""Decoder-only language models built on this framework's kernels.

One module family covers every model shape the framework is measured on:

* ``tiny``      - vocab 1024, d 256, 4 layers, 4 heads of 64, SwiGLU 688 (plumbing).
* ``4.7b``      - d 3072, 40 layers, 24 heads of 128, explicit Q/K/V/O, GELU FFN
                  12288, vocab 50257 (the compiled-hybrid-lm decoder shape the
                  reference quotes in ``README.md:33-45``), tied embeddings.
* ``qwen2.5-7b``  - d 3584, 28 layers, 28 Q / 4 KV heads of 128, SwiGLU 18944,
                    vocab 152064, RoPE theta 1e6.
* ``qwen2.5-32b`` - d 5120, 64 layers, 40 Q / 8 KV heads of 128, SwiGLU 27648,
                    vocab 152064, RoPE theta 1e6.

Every projection is a :class:`zeroq_b200.ops.qlinear.Linear4bit`; it holds a
frozen full-precision ``weight`` (before quantisation, or while a gather/release
coordinator has it gathered) or resident NF4 data (4-bit compute).  Weights are
random N(0, std) and can be generated layer by layer straight into NF4
(``init_nf4_``), so a 4.7B model never exists in bf16 on the device.

The vocabulary is padded to a multiple of 128 so logits rows are 16-byte
aligned for the tcgen05 GEMM's TMA store; the padded rows of the embedding are
zero and the loss ignores the padded columns.
"""

from __future__ import annotations

import math
import os
from dataclasses import asdict, dataclass, field, replace
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.utils.checkpoint as ckpt

from ..ops.activations import gelu, swiglu
from ..ops.attention import flash_attention
from ..ops.cross_entropy import cross_entropy, lm_head_cross_entropy
from ..ops.gemm import LMHeadFunction
from ..ops.norm import add_rmsnorm
from ..ops.qlinear import Linear4bit
from ..ops.qkv import qkv_fusable, qkv_projection
from ..ops.rope import RopeSpec, apply_rope, rope_table
from ..utils.metrics import nvtx_range


@dataclass
class DecoderConfig:
    vocab_size: int = 1024
    d_model: int = 256
    n_layers: int = 4
    n_heads: int = 4
    n_kv_heads: int = 4
    head_dim: int = 64
    ffn_dim: int = 688
    ffn_act: str = "swiglu"  # "swiglu" | "gelu"
    qkv_bias: bool = False   # Qwen2-family models carry Q/K/V biases
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    tie_embeddings: bool = True
    vocab_pad_multiple: int = 128
    # LoRA (PEFT naming); targets are projection names
    lora_r: int = 0
    lora_alpha: float = 32.0
    lora_targets: Tuple[str, ...] = ("q_proj", "k_proj", "v_proj", "o_proj")
    # quantisation of the frozen projections
    blocksize: int = 64
    quant_type: str = "nf4"
    # memory
    activation_checkpointing: bool = False
    # > 0: LM head + cross-entropy over vocabulary chunks of this many columns
    # (the [tokens, vocab] logits are never materialised; frozen head only).
    # Off by default: it trades one extra head GEMM for the logits' memory
    # (Qwen2.5-7B shape, 2 B200s: 29.4 vs 31.1 GB peak, 327 vs 314 ms/step)
    ce_chunk: int = 0
    train_norms: bool = True
    train_embeddings: bool = False

    @property
    def vocab_padded(self) -> int:
        m = self.vocab_pad_multiple
        return (self.vocab_size + m - 1) // m * m

    def num_params(self) -> int:
        d, L = self.d_model, self.n_layers
        attn = d * self.n_heads * self.head_dim * 2 + d * self.n_kv_heads * self.head_dim * 2
        if self.qkv_bias:
            attn += (self.n_heads + 2 * self.n_kv_heads) * self.head_dim
        mlp = d * self.ffn_dim * (3 if self.ffn_act == "swiglu" else 2)
        emb = self.vocab_size * d * (1 if self.tie_embeddings else 2)
        return L * (attn + mlp + 2 * d) + emb + d

    def to_dict(self) -> dict:
        return asdict(self)


PRESETS = {
    "tiny": DecoderConfig(),
    "4.7b": DecoderConfig(vocab_size=50257, d_model=3072, n_layers=40, n_heads=24,
                          n_kv_heads=24, head_dim=128, ffn_dim=12288, ffn_act="gelu",
                          rope_theta=10000.0, tie_embeddings=True,
                          lora_targets=("q_proj", "k_proj", "v_proj", "o_proj",
                                        "up_proj", "down_proj")),
    "qwen2.5-7b": DecoderConfig(vocab_size=152064, d_model=3584, n_layers=28, n_heads=28,
                                n_kv_heads=4, head_dim=128, ffn_dim=18944, ffn_act="swiglu",
                                qkv_bias=True, rope_theta=1e6, tie_embeddings=False,
                                lora_targets=("q_proj", "k_proj", "v_proj", "o_proj")),
    "qwen2.5-32b": DecoderConfig(vocab_size=152064, d_model=5120, n_layers=64, n_heads=40,
                                 n_kv_heads=8, head_dim=128, ffn_dim=27648, ffn_act="swiglu",
                                 qkv_bias=True, rope_theta=1e6, tie_embeddings=False,
                                 activation_checkpointing=True,
                                 lora_targets=("q_proj", "k_proj", "v_proj", "o_proj",
                                               "gate_proj", "up_proj", "down_proj")),
}


def get_config(name: str, **overrides) -> DecoderConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; choose from {sorted(PRESETS)}")
    return replace(PRESETS[name], **overrides)


class RMSNorm(nn.Module):
    """RMSNorm; ``forward(h, delta)`` fuses the residual add and returns
    ``(h + delta, norm(h + delta))``, ``forward(h)`` returns ``norm(h)``.

    Called as a module (never by reaching into ``.weight``) so that a
    gather/release coordinator's hooks gather a sharded weight first."""

    def __init__(self, d: int, eps: float, device=None, trainable: bool = True):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d, device=device, dtype=torch.float32),
                                   requires_grad=trainable)

    def forward(self, h: torch.Tensor, delta: Optional[torch.Tensor] = None):
        if delta is None:
            return add_rmsnorm(h, None, self.weight, self.eps)[1]
        return add_rmsnorm(h, delta, self.weight, self.eps)


# ZEROQ_FUSED_MLP=0 keeps the activation kernels between the MLP projections
# (the split forms with GEMM-epilogue activations are the default)
_FUSED_MLP = os.environ.get("ZEROQ_FUSED_MLP", "1") != "0"


def _hooked(m: nn.Module) -> bool:
    return bool(m._forward_hooks or m._forward_pre_hooks or m._backward_hooks
                or m._backward_pre_hooks)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: DecoderConfig, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        d, hd = cfg.d_model, cfg.head_dim

        def lin(name, i, o):
            r = cfg.lora_r if name in cfg.lora_targets else 0
            bias = cfg.qkv_bias and name in ("q_proj", "k_proj", "v_proj")
            return Linear4bit(i, o, bias=bias, blocksize=cfg.blocksize,
                              quant_type=cfg.quant_type, lora_r=r, lora_alpha=cfg.lora_alpha,
                              device=device, dtype=dtype)

        self.attn_norm = RMSNorm(d, cfg.norm_eps, device, cfg.train_norms)
        self.q_proj = lin("q_proj", d, cfg.n_heads * hd)
        self.k_proj = lin("k_proj", d, cfg.n_kv_heads * hd)
        self.v_proj = lin("v_proj", d, cfg.n_kv_heads * hd)
        self.o_proj = lin("o_proj", cfg.n_heads * hd, d)
        self.mlp_norm = RMSNorm(d, cfg.norm_eps, device, cfg.train_norms)
        if cfg.ffn_act == "swiglu":
            self.gate_proj = lin("gate_proj", d, cfg.ffn_dim)
        else:
            self.gate_proj = None
        self.up_proj = lin("up_proj", d, cfg.ffn_dim)
        self.down_proj = lin("down_proj", cfg.ffn_dim, d)

    def projections(self):
        out = [("q_proj", self.q_proj), ("k_proj", self.k_proj), ("v_proj", self.v_proj),
               ("o_proj", self.o_proj)]
        if self.gate_proj is not None:
            out.append(("gate_proj", self.gate_proj))
        out += [("up_proj", self.up_proj), ("down_proj", self.down_proj)]
        return out

    def forward(self, h: torch.Tensor, delta: Optional[torch.Tensor]):
        """``h`` is the residual stream, ``delta`` the previous block's output that
        still has to be added (fused into this layer's first norm)."""
        cfg = self.cfg
        B, S, d = h.shape
        if delta is None:
            x = self.attn_norm(h)
        else:
            h, x = self.attn_norm(h, delta)
        if self._fused_rope(x):
            # the q/k projection GEMMs apply the rotary embedding in their epilogue;
            # the attention backward could also rotate dQ/dK back (flash_attention
            # rope=spec) but measured slower than the RoPE kernel it replaces
            # (B=8 S=1024 H=24: +97 us against 2 x 25 us), so the projections'
            # backward un-rotates
            cs = rope_table(S, cfg.head_dim, cfg.rope_theta, x.device)
            mods = (self.q_proj, self.k_proj, self.v_proj)
            if not any(_hooked(m) for m in mods) and qkv_fusable(mods, x, S):
                # one GEMM for q, k and v (column slices of one output)
                if not hasattr(self, "_qkv_cache"):
                    self._qkv_cache = {}
                q, k, v = qkv_projection(x, mods, cs, self._qkv_cache)
            else:
                spec = RopeSpec(cs)
                q = self.q_proj(x, rope=spec).view(B, S, cfg.n_heads, cfg.head_dim)
                k = self.k_proj(x, rope=spec).view(B, S, cfg.n_kv_heads, cfg.head_dim)
                v = self.v_proj(x).view(B, S, cfg.n_kv_heads, cfg.head_dim)
            o = flash_attention(q, k, v, causal=True)
        else:
            q = self.q_proj(x).view(B, S, cfg.n_heads, cfg.head_dim)
            k = self.k_proj(x).view(B, S, cfg.n_kv_heads, cfg.head_dim)
            v = self.v_proj(x).view(B, S, cfg.n_kv_heads, cfg.head_dim)
            q, k = apply_rope(q, k, cfg.rope_theta)
            o = flash_attention(q, k, v, causal=True)
        a = self.o_proj(o.view(B, S, cfg.n_heads * cfg.head_dim))
        h, x = self.mlp_norm(h, a)
        if self.gate_proj is not None:
            if self._fused_mlp(with_gate=True):
                # up-projection epilogue writes u and silu(g)·u; the down-projection's
                # input-gradient epilogue writes dg and du: no SwiGLU kernels
                g = self.gate_proj(x)
                u, f = self.up_proj(x, act_out="swiglu", gate=g)
                return h, self.down_proj(f, pre=(g, u))
            f = swiglu(self.gate_proj(x), self.up_proj(x))
        elif self._fused_gelu_mlp():
            # up-projection epilogue writes h and gelu(h); the down-projection's
            # input-gradient epilogue applies gelu'(h): no GELU kernels
            pre, f = self.up_proj(x, act_out="gelu")
            return h, self.down_proj(f, pre=pre)
        else:
            f = gelu(self.up_proj(x))
        return h, self.down_proj(f)

    def _fused_rope(self, x: torch.Tensor) -> bool:
        from ..ops.qlinear import Linear4bit

        mods = (self.q_proj, self.k_proj)
        return (x.is_cuda and self.cfg.head_dim == 128
                and all(isinstance(m, Linear4bit) for m in mods)
                and not any(_hooked(m) for m in mods))

    def _fused_mlp(self, with_gate: bool = False) -> bool:
        """The MLP's projections are all ``Linear4bit`` without module hooks (the
        split activation forms pass the pre-activations as keyword arguments and
        return a non-differentiable activation, which per-module hooks do not see)."""
        from ..ops.qlinear import Linear4bit

        mods = (self.up_proj, self.down_proj) + ((self.gate_proj,) if with_gate else ())
        return (_FUSED_MLP and all(isinstance(m, Linear4bit) for m in mods)
                and not any(_hooked(m) for m in mods))

    def _fused_gelu_mlp(self) -> bool:
        return self._fused_mlp()


class DecoderLM(nn.Module):
    def __init__(self, cfg: DecoderConfig, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        self.dtype = dtype
        V = cfg.vocab_padded
        self.embed_tokens = nn.Embedding(V, cfg.d_model, device=device, dtype=dtype)
        self.embed_tokens.weight.requires_grad_(cfg.train_embeddings)
        self.layers = nn.ModuleList([DecoderLayer(cfg, device, dtype) for _ in range(cfg.n_layers)])
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps, device, cfg.train_norms)
        if cfg.tie_embeddings:
            self.lm_head = None
        else:
            self.lm_head = nn.Linear(cfg.d_model, V, bias=False, device=device, dtype=dtype)
            self.lm_head.weight.requires_grad_(cfg.train_embeddings)

    # -- weights ---------------------------------------------------------------
    def head_weight(self) -> torch.Tensor:
        return self.embed_tokens.weight if self.lm_head is None else self.lm_head.weight

    def _zero_vocab_padding(self):
        with torch.no_grad():
            self.embed_tokens.weight[self.cfg.vocab_size:].zero_()
            if self.lm_head is not None:
                self.lm_head.weight[self.cfg.vocab_size:].zero_()

    def init_dense_(self, std: float = 0.02, seed: int = 0):
        """Random N(0, std) full-precision projection weights (before partitioning)."""
        g = torch.Generator(device=self.embed_tokens.weight.device).manual_seed(seed)
        with torch.no_grad():
            self.embed_tokens.weight.normal_(0.0, std, generator=g)
            if self.lm_head is not None:
                self.lm_head.weight.normal_(0.0, std, generator=g)
            for layer in self.layers:
                for _, m in layer.projections():
                    w = torch.empty(m.out_features, m.in_features, device=m.weight.device,
                                    dtype=self.dtype)
                    w.normal_(0.0, std, generator=g)
                    m.weight = nn.Parameter(w, requires_grad=False)
        self._zero_vocab_padding()
        return self

    def init_nf4_(self, std: float = 0.02, seed: int = 0):
        """Random N(0, std) weights generated one projection at a time and
        quantised straight to NF4 (the bf16 model is never materialised)."""
        dev = self.embed_tokens.weight.device
        g = torch.Generator(device=dev).manual_seed(seed)
        with torch.no_grad():
            self.embed_tokens.weight.normal_(0.0, std, generator=g)
            if self.lm_head is not None:
                self.lm_head.weight.normal_(0.0, std, generator=g)
            for layer in self.layers:
                for _, m in layer.projections():
                    w = torch.empty(m.out_features, m.in_features, device=dev, dtype=self.dtype)
                    w.normal_(0.0, std, generator=g)
                    m.quantize_from(w)
                    del w
        self._zero_vocab_padding()
        return self

    def init_meta_(self):
        """Give every projection a meta-device weight of its full shape: the model
        can then be registered with a coordinator and filled tensor by tensor
        from a checkpoint (``zeroq_b200.utils.loading``) without ever holding a
        full-precision copy."""
        for layer in self.layers:
            for _, m in layer.projections():
                m.weight = nn.Parameter(torch.empty(m.out_features, m.in_features, device="meta",
                                                    dtype=self.dtype), requires_grad=False)
        return self

    def convert_to_4bit_(self):
        """Quantise every projection that still holds a dense weight (4-bit compute)."""
        for layer in self.layers:
            for _, m in layer.projections():
                if not m.has_nf4 and m.weight.numel():
                    m.quantize_from(m.weight.data)
                    m.weight = nn.Parameter(torch.empty(0, device=m.weight.device,
                                                        dtype=m.weight.dtype), requires_grad=False)
        return self

    # -- forward -----------------------------------------------------------------
    def _layer_call(self, layer, h, delta):
        if self.cfg.activation_checkpointing and self.training and torch.is_grad_enabled():
            if delta is None:
                return ckpt.checkpoint(lambda hh: layer(hh, None), h, use_reentrant=False)
            return ckpt.checkpoint(layer, h, delta, use_reentrant=False)
        return layer(h, delta)

    def forward(self, input_ids: torch.Tensor, targets: Optional[torch.Tensor] = None,
                ignore_index: int = -100):
        B, S = input_ids.shape
        h = self.embed_tokens(input_ids)
        delta = None
        cb = getattr(self, "_layer_grad_cb", None)
        for i, layer in enumerate(self.layers):
            if cb is not None and torch.is_grad_enabled() and h.requires_grad:
                # the gradient of a layer's input is complete once every kernel of
                # that layer's backward (its parameter gradients included) is queued
                h.register_hook(lambda g, i=i: cb(i))
            with nvtx_range(f"layer{i}"):
                h, delta = self._layer_call(layer, h, delta)
        x = self.norm(h) if delta is None else self.norm(h, delta)[1]
        W = self.head_weight()
        if W.numel() == 0:
            raise RuntimeError("the LM head weight is sharded and not gathered here; keep "
                               "'embed_tokens' and 'lm_head' in exclude_modules")
        if targets is not None and self.cfg.ce_chunk > 0:
            return lm_head_cross_entropy(x, W, targets.reshape(-1), vocab=self.cfg.vocab_size,
                                         ignore_index=ignore_index, chunk=self.cfg.ce_chunk)
        logits = LMHeadFunction.apply(x, W)
        if targets is None:
            return logits.view(B, S, -1)[..., : self.cfg.vocab_size]
        return cross_entropy(logits, targets.reshape(-1), vocab=self.cfg.vocab_size,
                             ignore_index=ignore_index)

    # -- bookkeeping ---------------------------------------------------------------
    def trainable_parameters(self):
        return [p for p in self.parameters() if p.requires_grad]

    def layer_parameter_groups(self):
        """The trainable parameters of each decoder layer (``overlap_buckets`` of
        :class:`~zeroq_b200.parallel.optimizer.ShardedAdamW`)."""
        return [[p for p in layer.parameters() if p.requires_grad] for layer in self.layers]

    def pack_lora_operands(self) -> bool:
        """Repack the bf16 LoRA operands of every adapter that already has them (the
        fused q/k/v blocks and each other projection's own) in ONE launch, and mark
        those caches current, so the next forward packs nothing.  Call after an
        optimizer step (the :class:`~zeroq_b200.train.Trainer` does).  Adapters
        without operands yet pack themselves on first use.  Returns False when
        nothing was launched (the lazy per-module packs then run)."""
        from ..ops.qkv import lora_block_views, lora_blocks_key
        from ..ops.qlinear import Linear4bit, LoraPackBatch

        jobs = []
        for layer in self.layers:
            cache = getattr(layer, "_qkv_cache", None)
            mods = (layer.q_proj, layer.k_proj, layer.v_proj)
            if cache and "A_cat" in cache and all(getattr(m, "lora_r", 0) for m in mods):
                views = lora_block_views(mods, cache)

                def done_qkv(cache=cache, mods=mods):
                    cache["key"] = lora_blocks_key(mods)

                for i, (m, a_v, b_v, t_v) in enumerate(views):
                    jobs.append((m.lora_A.detach(), m.lora_B.detach(), m.scaling, a_v, b_v, t_v,
                                 done_qkv if i == len(views) - 1 else (lambda: None)))
            for _, m in layer.projections():
                ops = getattr(m, "_lora_ops", None) if isinstance(m, Linear4bit) else None
                if ops is not None and m.lora_r:
                    jobs.append((m.lora_A.detach(), m.lora_B.detach(), m.scaling, ops[0], ops[1], ops[2],
                                 lambda m=m: setattr(m, "_lora_key", m._lora_state_key())))
        if not jobs:
            return False
        if not hasattr(self, "_lora_batch"):
            self._lora_batch = LoraPackBatch()
        with torch.no_grad():
            return self._lora_batch.run(jobs)

    def set_layer_grad_callback(self, fn):
        """``fn(i)`` runs in the backward when layer ``i``'s input gradient is
        computed - every gradient of layer ``i`` is written by then (e.g.
        ``ShardedAdamW.bucket_ready``).  Layer 0's input (the frozen embedding)
        takes no gradient, so layer 0 gets no call.  ``None`` removes it."""
        self._layer_grad_cb = fn

    def flops_per_token(self, seq_len: int) -> float:
        """Training FLOPs per token: frozen projections run forward + input-grad
        (4·params), the head likewise, attention fwd (causal) + bwd (2.5x fwd);
        LoRA adds 6·r·(in+out) per adapted projection."""
        c = self.cfg
        proj = 0
        lora = 0
        for name, m in self.layers[0].projections():
            proj += m.in_features * m.out_features
            if m.lora_r:
                lora += m.lora_r * (m.in_features + m.out_features)
        proj *= c.n_layers
        lora *= c.n_layers
        head = c.d_model * c.vocab_padded
        attn_fwd = 2 * 2 * seq_len * c.n_heads * c.head_dim * c.n_layers * 0.5
        return 4 * proj + 4 * head + 6 * lora + attn_fwd * 3.5

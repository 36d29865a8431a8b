#!/usr/bin/env python
"""Training-throughput benchmark: the 4.7B NF4 decoder in 4-bit compute mode.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one rank per GPU with torchrun (``--master-addr 127.0.0.1``);
RANK / LOCAL_RANK / WORLD_SIZE come from the environment.

Workload (weak scaling, per GPU): batch 8 x seq 1024 uniform random token ids,
next-token cross-entropy, decoder d=3072, 40 layers, 24 heads of 128, explicit
Q/K/V/O, GELU FFN 12288, vocab 50257, random N(0, 0.02) weights quantised to NF4
(block 64, fp32 absmax) through the public ``initialize`` API with
``compute_in_4bit=True``; LoRA r=16 (alpha 32) on every projection and the RMSNorm
weights train under AdamW (reduce-scatter + sharded update + all-gather across
ranks).  The embedding (tied LM head) stays bf16 and frozen.

Reported (rank 0, one JSON line):
* ``value``: tokens/s over all ranks, device-timed with CUDA events around K
  steps (barrier + synchronize on both sides, max over ranks); inputs resident.
* ``e2e``: the same through ``Trainer.step`` - pinned host -> device copy of the
  batch and a device -> host read of the loss every step.
* ``gpu_launches``: this framework's kernel launches inside the timed region
  (with ``cuda_graph``, the kernels captured in one step times the steps).
* ``cuda_graph``: each step ran as one CUDA graph replay (the default for the
  resident-weight configs; ``--no-graph`` runs eagerly).
* ``clocks``: nvidia-smi SM clock median and throttle reasons sampled during it.
The step's working set (NF4 weights, activations, logits) is tens of GB, far
larger than the 126 MB L2, so no explicit L2 flush is needed between steps.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys

REFERENCE_PUBLISHED_TOK_S = 23.7  # the reference's published rate, README.md:41, 2x Tesla M40
METRIC = "train tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200; fused-path % roofline"


def _measured_peaks():
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
                "source": "fallback"}


# name -> (model preset, lora r, lora targets or None, batch, seq, mode, description)
CONFIGS = {
    "4.7b": ("4.7b", 16, None, 8, 1024, "4bit-once",
             "NF4 4-bit compute (weights gathered once, resident), LoRA r=16 on every "
             "projection + RMSNorm weights, AdamW"),
    "qwen7b-4bit": ("qwen2.5-7b", 16, ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                       "up_proj", "down_proj"), 4, 2048, "4bit-once",
                    "Qwen2.5-7B shape, NF4 4-bit compute (weights gathered once, resident), "
                    "SwiGLU MLP with its GEMM epilogues, LoRA r=16 on all linears + RMSNorm "
                    "weights, AdamW"),
    "qwen7b-hetero": ("qwen2.5-7b", 16, ("q_proj", "k_proj", "v_proj", "o_proj"), 4, 2048,
                      "hetero",
                      "Qwen2.5-7B shape, frozen NF4 base sharded by uneven rank weights "
                      "(rank_weights: [2,2,1,1,1,1,1,1] at 8 ranks) and gathered per use "
                      "(peer plan gather), LoRA r=16 alpha 32 on q/k/v/o, AdamW"),
    "qwen32b-gather": ("qwen2.5-32b", 64, ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                          "up_proj", "down_proj"), 2, 4096, "gather",
                       "Qwen2.5-32B shape, NF4 shards gathered per layer with one layer of "
                       "prefetch and released after use, activation checkpointing, LoRA r=64 "
                       "on all linears, AdamW"),
}


def hetero_weights(world: int):
    """Rank weights of the hetero config: the 8-rank plan [2,2,1,1,1,1,1,1] and, at
    fewer ranks, the same 2:1 split with a quarter of the ranks (at least one)
    holding double shares - [2,1] at 2 ranks, [2,1,1,1] at 4 - so every rank
    count measures a genuinely uneven plan."""
    heavy = max(1, world // 4)
    return [2.0] * heavy + [1.0] * (world - heavy)


def run_reference(args):
    """The reference's engine cannot be constructed on this image (see reason)."""
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "zero_q")):
        reason = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import zero_q  # noqa: F401
            import zero_q.coordinator  # noqa: F401  (needs bitsandbytes)
        except Exception as e:
            reason = (f"reference 4-bit engine unavailable: zero_q.coordinator imports bitsandbytes "
                      f"(src/coordinator.py:14), which is not installed and not in the offline "
                      f"wheelhouse ({type(e).__name__}: {e})")
    if reason is None:
        reason = "reference 4.7B decoder (compiled-hybrid-lm) is not part of the reference repo"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="4.7b", choices=sorted(CONFIGS),
                    help="4.7b: the headline; qwen7b-hetero / qwen32b-gather: the other "
                         "model configs (gather/release paths)")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="run the steps eagerly instead of as one CUDA graph replay each")
    ap.add_argument("--overlap-sync", action="store_true",
                    help="sync the trainable gradients per decoder layer during the backward "
                         "(fused backend, several GPUs)")
    ap.add_argument("--torch-profile", default=None,
                    help="after timing, profile one more step and write a per-kernel table here")
    ap.add_argument("--metrics-jsonl", default=None,
                    help="per-step JSONL (loss, device ms and tokens/s max over ranks, bytes "
                         "gathered / synced) written by the Trainer during the end-to-end pass")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from zeroq_b200 import ShardedAdamW, ZeroQConfig, initialize
    from zeroq_b200.models import DecoderLM, get_config
    from zeroq_b200.ops import _ext
    from zeroq_b200.train import ClockSampler, Trainer, device_time_ms, synthetic_batch
    from zeroq_b200.utils import metrics

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=10),
                                device_id=device)
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    _ext.ext()

    preset, lora_r, targets, B0, S0, mode, desc = CONFIGS[args.config]
    overrides = dict(lora_r=lora_r, lora_alpha=2.0 * lora_r)
    if targets is not None:
        overrides["lora_targets"] = targets
    cfg = get_config(preset, **overrides)
    model = DecoderLM(cfg, device=device)
    model.init_dense_(std=0.02, seed=1234)  # identical on every rank
    zq = ZeroQConfig(compute_dtype=torch.bfloat16, compute_in_4bit=True, double_quant=False,
                     gather_once=(mode == "4bit-once"), prefetch_count=1, async_gather=True,
                     exclude_modules=["lm_head", "embed_tokens"], backend="auto")
    rank_weights = hetero_weights(world) if mode == "hetero" else None
    trainable = ("lora_", "norm") if mode == "4bit-once" else ("lora_",)
    initialize(model, zq, trainable_patterns=trainable, rank_weights=rank_weights)
    torch.cuda.empty_cache()
    # --overlap-sync: one fused reduce-scatter + AdamW + all-gather per decoder layer,
    # launched during the backward (several ranks)
    okw = dict(overlap_buckets=model.layer_parameter_groups()) if args.overlap_sync else {}
    opt = ShardedAdamW(model.trainable_parameters(), lr=1e-4, betas=(0.9, 0.999),
                       weight_decay=0.0, **okw)
    if getattr(opt, "overlap", False):
        model.set_layer_grad_callback(opt.bucket_ready)
    trainer = Trainer(model, opt, device)

    B = args.batch or B0
    S = args.seq or S0
    x_host, y_host = synthetic_batch(B, S, cfg.vocab_size, seed=1000 + rank)
    x_dev, y_dev = x_host.to(device), y_host.to(device)

    # CUDA graph (weights resident, fixed shapes): warm-up step 0 runs eagerly,
    # step 1 runs eagerly on the capture stream and captures, later steps replay
    use_graph = not args.no_graph and mode == "4bit-once"
    losses = []
    for i in range(args.warmup):
        if use_graph and i == 1:
            trainer.enable_cuda_graph()
        losses.append(trainer.step_device(x_dev, y_dev))
    torch.cuda.synchronize()
    graphed = trainer._graph is not None

    metrics.reset_counters()
    with ClockSampler(local) as clk, _ext.LaunchCounter() as lc:
        ms = device_time_ms(lambda: trainer.step_device(x_dev, y_dev), args.steps)
    moved = {k: v // args.steps for k, v in metrics.snapshot().items()}
    e2e_ms = None
    if not args.no_e2e:
        if args.metrics_jsonl:
            trainer.logger = metrics.StepLogger(args.metrics_jsonl, flush_every=args.steps,
                                                flops_per_token=model.flops_per_token(S),
                                                peak_tflops=_measured_peaks()["bf16_tflops_sustained"])
        e2e_ms = device_time_ms(lambda: losses.append(trainer.step(x_host, y_host)), args.steps)
        if trainer.logger is not None:
            trainer.logger.flush()
            trainer.logger = None

    if args.torch_profile:
        # every rank runs the profiled step (its collectives need all ranks); rank r
        # writes its table to PATH (rank 0) or PATH.rank<r>
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            trainer.step_device(x_dev, y_dev)
            torch.cuda.synchronize()
        path = args.torch_profile if rank == 0 else f"{args.torch_profile}.rank{rank}"
        with open(path, "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=60,
                                              max_name_column_width=90))

    tokens = B * S * world * args.steps
    value = tokens / (ms / 1000.0)
    peaks = _measured_peaks()
    fpt = model.flops_per_token(S)
    tflops_per_gpu = fpt * value / world / 1e12
    mem = torch.tensor([torch.cuda.max_memory_allocated(device) / 1e9], device=device)
    if world > 1:
        dist.all_reduce(mem, op=dist.ReduceOp.MAX)
    mem_gb = float(mem.item())
    first_loss = float(losses[0]) if losses else float("nan")
    last_loss = float(losses[-1]) if losses else float("nan")
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / REFERENCE_PUBLISHED_TOK_S, 1) if args.config == "4.7b" else None,
        "dtype": "bf16",
        "data": "synthetic (uniform random token ids; random-init N(0,0.02) weights)",
        "impl": "ours",
        "config": {
            "model": f"{preset} decoder (d={cfg.d_model}, {cfg.n_layers} layers, "
                     f"{cfg.n_heads}/{cfg.n_kv_heads} heads of {cfg.head_dim}, {cfg.ffn_act} FFN "
                     f"{cfg.ffn_dim}, vocab {cfg.vocab_size}); {desc}",
            "config_name": args.config,
            "rank_weights": rank_weights,
            "global_batch": B * world,
            "seq_len": S,
            "parallelism": f"dp{world}",
            "l2": "no flush: per-step working set (NF4 weights + activations) >> 126 MB L2",
        },
        "e2e": None if e2e_ms is None else {
            "value": round(tokens / (e2e_ms / 1000.0), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size()
                                      + y_host.numel() * y_host.element_size()),
            "d2h_bytes_per_step": 4,
        },
        "gpu_launches": trainer.graph_launches * args.steps if graphed else lc.count,
        "cuda_graph": graphed,
        "clocks": clk.summary(),
        "achieved_tflops_per_gpu": round(tflops_per_gpu, 1),
        "frac_of_measured_bf16_sustained": round(tflops_per_gpu / peaks["bf16_tflops_sustained"], 3),
        "peak_mem_gb": round(mem_gb, 1),   # max over ranks
        "gather_bytes_per_step": moved.get("gather_bytes", 0),   # rank 0: read from other ranks
        "sync_bytes_per_step": moved.get("sync_bytes", 0),
        "loss_first_last": [round(first_loss, 4), round(last_loss, 4)],
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Train a decoder from scratch with ZeRO-3 style fp32 master shards.

Counterpart of the reference's train-from-scratch mode (``ZeroQTrainConfig``,
``SPEC_TRAIN_FROM_SCRATCH.md``): every projection weight lives as an fp32
master shard (ceil split, 1/W per rank); the full weight is all-gathered for
each use and released after it, the full gradient is reduce-scattered into the
shard's ``.grad`` by a hook, and the optimizer updates only the shards.

    torchrun --standalone --nproc-per-node 8 examples/train_from_scratch.py --model tiny --steps 200
    python examples/train_from_scratch.py --model tiny --layers 2 --steps 5 --optimizer lion-fused

``--optimizer adamw`` (torch AdamW over the master shards), ``lion-fused`` (the
Lion update with stochastic rounding runs inside the backward hook right after
the reduce-scatter, fp16 masters; the forward uses NF4 copies re-quantised from
the masters after each step) or ``adamw-offload`` (fp32 masters in host memory,
NF4 copies on the device re-quantised after each step).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import zeroq_b200 as zq  # noqa: E402
from zeroq_b200.models import DecoderLM, get_config  # noqa: E402


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model", default="tiny")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--seq", type=int, default=128)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--optimizer", choices=["adamw", "lion-fused", "adamw-offload"], default="adamw")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--fixed-batch", action="store_true", help="reuse one batch (memorisation smoke)")
    args = p.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    rank = dist.get_rank() if dist.is_initialized() else 0
    if torch.cuda.is_available():
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device("cpu")
    torch.manual_seed(args.seed)
    overrides = {"n_layers": args.layers} if args.layers else {}
    cfg = get_config(args.model, **overrides)
    model = DecoderLM(cfg, device=device, dtype=torch.float32).init_dense_(seed=args.seed)
    for p_ in model.parameters():          # everything trains from scratch
        p_.requires_grad_(True)
    tcfg = zq.ZeroQTrainConfig(exclude_modules=["lm_head", "embed_tokens"],
                               fused_shard_step=args.optimizer == "lion-fused",
                               master_dtype=torch.float16 if args.optimizer == "lion-fused" else torch.float32,
                               cpu_offload=args.optimizer == "adamw-offload", lion_lr=args.lr)
    coord = zq.ZeroQCoordinator(tcfg)
    zq.ZeroQModuleWrapper(model, coord).partition()
    masters = coord.trainable_master_params()
    others = [p_ for n, p_ in model.named_parameters() if p_.requires_grad and p_.numel()
              and not any(p_ is m for m in masters)]
    opt = None
    if args.optimizer != "lion-fused":
        opt = torch.optim.AdamW(list(masters) + others, lr=args.lr)
    g = torch.Generator().manual_seed(args.seed + rank)
    fixed = torch.randint(0, cfg.vocab_size, (args.batch, args.seq), generator=g).to(device)
    first = last = None
    for step in range(args.steps):
        t0 = time.perf_counter()
        x = fixed if args.fixed_batch else \
            torch.randint(0, cfg.vocab_size, (args.batch, args.seq), generator=g).to(device)
        loss = model(x, x.roll(-1, dims=1))
        loss.backward()
        if opt is not None:
            if dist.is_initialized():        # replicated (unsharded) parameters: average
                for p_ in others:
                    if p_.grad is not None:
                        dist.all_reduce(p_.grad)
                        p_.grad /= dist.get_world_size()
            opt.step()
            opt.zero_grad(set_to_none=False)
        if args.optimizer in ("adamw-offload", "lion-fused"):
            # these modes run the forward from NF4 copies of the masters
            coord.update_4bit_from_masters()
        v = loss.item()
        first = v if first is None else first
        last = v
        if rank == 0:
            print(json.dumps({"step": step + 1, "loss": round(v, 4),
                              "step_s": round(time.perf_counter() - t0, 4)}), flush=True)
    if rank == 0:
        print(json.dumps({"event": "done", "first_loss": first, "last_loss": last,
                          "zeroq": coord.get_memory_stats()}), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

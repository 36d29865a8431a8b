#!/usr/bin/env python
"""Multi-node LoRA + ZeRO-Q smoke test: every rank must end each step with the same adapters.

Counterpart of the reference's ``run_smoke_lora_multinode.py``: a decoder with
NF4-sharded frozen weights (gather/release) and LoRA adapters trains a few
steps; LoRA gradients are averaged with an explicit all-reduce; after each step
the ranks compare an adapter checksum and fail loudly if they differ.

    torchrun --nnodes 2 --nproc-per-node 8 --rdzv-endpoint head:29500 examples/smoke_lora_multinode.py
    torchrun --standalone --nproc-per-node 2 examples/smoke_lora_multinode.py --model tiny
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import zeroq_b200 as zq  # noqa: E402
from zeroq_b200.models import DecoderLM, get_config  # noqa: E402


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model", default="tiny")
    p.add_argument("--layers", type=int, default=2)
    p.add_argument("--steps", type=int, default=int(os.environ.get("STEPS", "2")))
    p.add_argument("--seq-len", type=int, default=int(os.environ.get("SEQ_LEN", "128")))
    p.add_argument("--batch-size", type=int, default=int(os.environ.get("BATCH", "2")))
    p.add_argument("--lr", type=float, default=float(os.environ.get("LR", "1e-3")))
    p.add_argument("--seed", type=int, default=int(os.environ.get("SEED", "1234")))
    args = p.parse_args(argv)

    if "WORLD_SIZE" in os.environ and not dist.is_initialized():
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=300))
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    if torch.cuda.is_available():
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device("cpu")
    torch.manual_seed(args.seed)
    cfg = get_config(args.model, n_layers=args.layers, lora_r=8)
    model = DecoderLM(cfg, device=device).init_dense_(seed=args.seed)
    zq.prepare_model_for_zeroq(model, zq.ZeroQConfig(exclude_modules=["lm_head", "embed_tokens"]),
                               trainable_patterns=("lora_",))
    params = [p_ for p_ in model.parameters() if p_.requires_grad]
    opt = torch.optim.AdamW(params, lr=args.lr)
    g = torch.Generator().manual_seed(args.seed + 17 * rank)
    ok = True
    for step in range(args.steps):
        x = torch.randint(0, cfg.vocab_size, (args.batch_size, args.seq_len), generator=g).to(device)
        loss = model(x, x.roll(-1, dims=1))
        loss.backward()
        for p_ in params:                      # manual LoRA gradient averaging
            if p_.grad is not None and world > 1:
                dist.all_reduce(p_.grad)
                p_.grad /= world
        opt.step()
        opt.zero_grad()
        checksum = torch.stack([p_.detach().double().sum() for p_ in params]).sum().to(device)
        if world > 1:
            lo, hi = checksum.clone(), checksum.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            agree = bool((hi - lo).abs() <= 1e-9 * max(1.0, hi.abs().item()))
        else:
            agree = True
        ok = ok and agree
        if rank == 0:
            print(json.dumps({"step": step + 1, "loss_rank0": round(loss.item(), 5),
                              "adapter_checksum": round(checksum.item(), 6),
                              "ranks_agree_on_adapters": agree}), flush=True)
    if rank == 0:
        print(json.dumps({"event": "done", "world": world, "ok": ok,
                          "zeroq": zq.get_zeroq_memory_stats(model)}), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

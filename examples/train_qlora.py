#!/usr/bin/env python
"""Production QLoRA trainer: NF4-sharded frozen base, LoRA adapters, AdamW.

Counterpart of the reference's ``examples/train_32b_maxwell.py``: streamed
checkpoint loading into ZeRO-Q shards, data-parallel training with gradient
accumulation, all-ranks-agree finite checks before every optimizer step,
CUDA-event throughput (max over ranks), best-loss adapter snapshot, early stop
decided on rank 0 and broadcast, PEFT-named adapter export and sharded resume.

    # one node, 8 GPUs, Qwen2.5-32B shape, gather/release with prefetch
    timeout -k 60 7200 torchrun --standalone --nproc-per-node 8 examples/train_qlora.py \\
        --model qwen2.5-32b --mode gather --seq 4096 --batch 2 --checkpoint /path/to/hf/ckpt
    # 4-bit compute (weights gathered once, resident NF4), random weights
    torchrun --standalone --nproc-per-node 2 examples/train_qlora.py --model 4.7b --mode 4bit
    # CPU smoke run (tiny model, gloo)
    python examples/train_qlora.py --model tiny --steps 3 --seq 64 --batch 2

Data: ``--data FILE`` trains on the file's bytes (token id = byte value);
without it, uniform random token ids.  ``--hetero-weights 2,2,1,...`` switches
to VRAM-weighted shards.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import zeroq_b200 as zq  # noqa: E402
from zeroq_b200.models import DecoderLM, get_config  # noqa: E402
from zeroq_b200.utils.checkpoint import (load_sharded_checkpoint, save_adapters,  # noqa: E402
                                         save_sharded_checkpoint)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model", default="tiny")
    p.add_argument("--layers", type=int, default=None, help="override the preset's layer count")
    p.add_argument("--checkpoint", default=None, help="HF-format safetensors file or directory")
    p.add_argument("--mode", choices=["4bit", "gather"], default="4bit")
    p.add_argument("--hetero-weights", default=None)
    p.add_argument("--data", default=None)
    p.add_argument("--seq", type=int, default=1024)
    p.add_argument("--batch", type=int, default=4, help="micro-batch per rank")
    p.add_argument("--accum", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--lr", type=float, default=2e-4)
    p.add_argument("--weight-decay", type=float, default=0.0)
    p.add_argument("--max-grad-norm", type=float, default=None,
                   help="global-norm gradient clipping (computed on the device, every backend)")
    p.add_argument("--lora-r", type=int, default=16)
    p.add_argument("--lora-alpha", type=float, default=32.0)
    p.add_argument("--lora-targets", default=None, help="comma list (default: the preset's)")
    p.add_argument("--grad-checkpointing", action="store_true")
    p.add_argument("--patience", type=int, default=0, help="early stop after N non-improving logs")
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--save", default=None, help="directory for adapters + sharded state")
    p.add_argument("--resume", default=None, help="sharded checkpoint directory to resume from")
    p.add_argument("--seed", type=int, default=1234)
    return p.parse_args(argv)


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
    return rank, world, device


class TokenChunks:
    """Fixed-length ``seq + 1`` token windows; rank-strided, reshuffled per epoch
    with a seed shared by all ranks (a DistributedSampler without the dataset)."""

    def __init__(self, tokens: torch.Tensor, seq: int, rank: int, world: int, seed: int):
        n = (tokens.numel() - 1) // seq
        if n < world:
            raise ValueError("not enough data for one window per rank")
        self.tokens, self.seq, self.rank, self.world, self.seed = tokens, seq, rank, world, seed
        self.n = n
        self.epoch, self.pos, self.order = 0, 0, None
        self._reshuffle()

    def _reshuffle(self):
        g = torch.Generator().manual_seed(self.seed + self.epoch)
        self.order = torch.randperm(self.n, generator=g)[self.rank::self.world]
        self.pos = 0

    def next_batch(self, batch: int):
        xs = []
        for _ in range(batch):
            if self.pos >= self.order.numel():
                self.epoch += 1
                self._reshuffle()
            i = int(self.order[self.pos]) * self.seq
            self.pos += 1
            xs.append(self.tokens[i:i + self.seq + 1])
        w = torch.stack(xs)
        return w[:, :-1].contiguous(), w[:, 1:].contiguous()


def load_tokens(args, vocab: int) -> torch.Tensor:
    if args.data:
        with open(args.data, "rb") as f:
            data = torch.frombuffer(bytearray(f.read()), dtype=torch.uint8).long()
        return data % vocab
    g = torch.Generator().manual_seed(args.seed)
    return torch.randint(0, vocab, (max(64, args.steps * args.accum * args.batch * 4) * (args.seq + 1),),
                         generator=g)


def all_ranks_true(flag: bool, device) -> bool:
    if not dist.is_initialized():
        return flag
    t = torch.tensor([1 if flag else 0], device=device, dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def main(argv=None) -> int:
    args = parse_args(argv)
    rank, world, device = setup_dist()
    torch.manual_seed(args.seed)
    overrides = dict(lora_r=args.lora_r, lora_alpha=args.lora_alpha)
    if args.layers:
        overrides["n_layers"] = args.layers
    if args.lora_targets:
        overrides["lora_targets"] = tuple(args.lora_targets.split(","))
    if args.grad_checkpointing:
        overrides["activation_checkpointing"] = True
    cfg = get_config(args.model, **overrides)
    model = DecoderLM(cfg, device=device)
    if args.checkpoint:
        model.init_meta_()
    else:
        model.init_dense_(seed=args.seed)
    zcfg = zq.ZeroQConfig(compute_dtype=torch.bfloat16 if device.type == "cuda" else torch.float32,
                          compute_in_4bit=args.mode == "4bit", gather_once=args.mode == "4bit",
                          exclude_modules=["lm_head", "embed_tokens"])
    weights = [float(w) for w in args.hetero_weights.split(",")] if args.hetero_weights else None
    zq.prepare_model_for_zeroq(model, zcfg, trainable_patterns=("lora_",), rank_weights=weights,
                               checkpoint=args.checkpoint)
    opt = zq.ShardedAdamW(model.trainable_parameters(), lr=args.lr, weight_decay=args.weight_decay,
                          max_grad_norm=args.max_grad_norm)
    start = 0
    if args.resume:
        start = load_sharded_checkpoint(args.resume, model, opt)
    data = TokenChunks(load_tokens(args, cfg.vocab_size), args.seq, rank, world, args.seed)
    stats = zq.get_zeroq_memory_stats(model)
    if rank == 0:
        print(json.dumps({"event": "start", "model": args.model, "mode": args.mode, "world": world,
                          "params": cfg.num_params(), "trainable": sum(p.numel() for p in
                                                                       model.trainable_parameters()),
                          "zeroq": stats, "resume_step": start}), flush=True)

    best, best_state, bad_logs = math.inf, None, 0
    tokens_per_step = args.batch * args.seq * args.accum * world
    for step in range(start, args.steps):
        t0 = time.perf_counter()
        if device.type == "cuda":
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        loss_sum = torch.zeros((), device=device)
        for _ in range(args.accum):
            x, y = data.next_batch(args.batch)
            loss = model(x.to(device, non_blocking=True), y.to(device, non_blocking=True))
            (loss / args.accum).backward()
            loss_sum += loss.detach().float()
        local_ok = bool(torch.isfinite(loss_sum).item())
        grads = [p.grad for p in model.trainable_parameters() if p.grad is not None]
        if local_ok and grads:
            local_ok = bool(torch.isfinite(torch.stack([g.float().abs().max() for g in grads]).max()).item())
        if all_ranks_true(local_ok, device):  # every rank steps or none does
            opt.step()
        elif rank == 0:
            print(json.dumps({"event": "skip_nonfinite", "step": step}), flush=True)
        opt.zero_grad()
        if device.type == "cuda":
            ev1.record()
            torch.cuda.synchronize()
            dt = ev0.elapsed_time(ev1) / 1000.0
        else:
            dt = time.perf_counter() - t0
        mean_loss = loss_sum / args.accum
        if dist.is_initialized():
            pack = torch.tensor([mean_loss.item(), dt], device=device, dtype=torch.float64)
            dist.all_reduce(pack[:1], op=dist.ReduceOp.SUM)
            dist.all_reduce(pack[1:], op=dist.ReduceOp.MAX)
            mean_loss_v, dt = pack[0].item() / world, pack[1].item()
        else:
            mean_loss_v = mean_loss.item()
        stop = False
        if (step + 1) % args.log_every == 0:
            if rank == 0:
                print(json.dumps({"step": step + 1, "loss": round(mean_loss_v, 4),
                                  "tokens_per_s": round(tokens_per_step / dt, 1),
                                  "step_s": round(dt, 4)}), flush=True)
            if mean_loss_v < best:
                best, bad_logs = mean_loss_v, 0
                best_state = {n: p.detach().cpu().clone() for n, p in model.named_parameters()
                              if p.requires_grad}
            else:
                bad_logs += 1
            stop = args.patience > 0 and bad_logs >= args.patience
        if dist.is_initialized():  # rank 0 decides, everybody follows
            flag = torch.tensor([1 if stop else 0], device=device, dtype=torch.int32)
            dist.broadcast(flag, src=0)
            stop = bool(flag.item())
        if stop:
            if rank == 0:
                print(json.dumps({"event": "early_stop", "step": step + 1, "best_loss": best}),
                      flush=True)
            break

    if args.save:
        os.makedirs(args.save, exist_ok=True)
        save_sharded_checkpoint(args.save, model, opt, step=step + 1)
        if best_state is not None:
            with torch.no_grad():
                for n, p in model.named_parameters():
                    if n in best_state:
                        p.copy_(best_state[n].to(p.device))
        if rank == 0:
            save_adapters(model, os.path.join(args.save, "adapter_model.safetensors"))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

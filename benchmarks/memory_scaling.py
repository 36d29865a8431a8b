#!/usr/bin/env python
"""Per-rank weight memory, fp16 replicated vs NF4-sharded (ZeRO-Q), across world sizes.

Counterpart of the reference's ``benchmarks/benchmark_memory.py`` (memory scaling
of a multi-layer MLP under partitioning).  For each world size W the MLP is
registered with a coordinator and really quantised and sharded on W ranks (gloo
processes on CPU, or NCCL on W GPUs with ``--cuda``); every rank reports the
bytes it holds and rank 0 prints one JSON line per W with the fp16 replicated
size, the measured per-rank NF4 shard bytes and the ratio.  ``--model`` adds
the analytic per-GPU estimate for a decoder preset.

    python benchmarks/memory_scaling.py --hidden 2048 --layers 8 --world 1 2 4
    python benchmarks/memory_scaling.py --cuda --world 2 4 8 --hidden 8192 --layers 16
    python benchmarks/memory_scaling.py --model qwen2.5-32b --world 8 --seq 4096 --batch 2
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import socket
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


class SimpleMLP(torch.nn.Module):
    def __init__(self, hidden: int, layers: int):
        super().__init__()
        self.layers = torch.nn.ModuleList([torch.nn.Linear(hidden, hidden, bias=False)
                                           for _ in range(layers)])

    def forward(self, x):
        for l in self.layers:
            x = torch.relu(l(x))
        return x


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, args, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    backend = "nccl" if args.cuda else "gloo"
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    device = torch.device("cuda", rank) if args.cuda else torch.device("cpu")
    if args.cuda:
        torch.cuda.set_device(device)
    import zeroq_b200 as zq

    torch.manual_seed(0)
    model = SimpleMLP(args.hidden, args.layers).to(device)
    for p in model.parameters():   # frozen base weights are what ZeRO-Q shards
        p.requires_grad_(False)
    coord = zq.ZeroQCoordinator(zq.ZeroQConfig(exclude_modules=[]))
    zq.ZeroQModuleWrapper(model, coord).partition()
    local = 0
    for p in coord._params.values():
        for t in (p.local_packed, p.local_absmax):
            if t is not None:
                local += t.numel() * t.element_size()
    t = torch.tensor([float(local)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        out[world] = {"max_local_bytes": t.item(), "stats": coord.get_memory_stats()}
    dist.barrier()
    dist.destroy_process_group()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--world", type=int, nargs="+", default=[1, 2, 4])
    ap.add_argument("--cuda", action="store_true", help="NCCL ranks on GPUs (one per rank)")
    ap.add_argument("--model", default=None, help="also print the analytic estimate for a preset")
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=8)
    args = ap.parse_args(argv)

    fp16_bytes = args.hidden * args.hidden * args.layers * 2
    ctx = mp.get_context("spawn")
    for W in args.world:
        mgr = ctx.Manager()
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(W, _free_port(), args, out), nprocs=W, join=True,
                           start_method="spawn")
        res = dict(out[W])
        mgr.shutdown()
        print(json.dumps({"world": W, "hidden": args.hidden, "layers": args.layers,
                          "fp16_replicated_bytes": fp16_bytes,
                          "nf4_shard_bytes_per_rank": int(res["max_local_bytes"]),
                          "ratio_vs_fp16": round(fp16_bytes / max(1.0, res["max_local_bytes"]), 2),
                          "coordinator_stats": res["stats"]}), flush=True)
    if args.model:
        from zeroq_b200.models import get_config
        from zeroq_b200.utils.memory import estimate_zeroq_memory

        cfg = get_config(args.model)
        for W in args.world:
            for mode in ("bf16", "4bit", "gather"):
                est = estimate_zeroq_memory(cfg, args.batch, args.seq, world_size=W, mode=mode)
                print(json.dumps({"model": args.model, "world": W, "mode": mode,
                                  **{k: round(v, 3) for k, v in est.as_dict().items()}}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

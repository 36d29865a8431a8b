#!/usr/bin/env python
"""Fused collective microbenchmarks on 2/4/8 GPUs of one node (run with torchrun).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/collectives.py --op ag_gemm
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/collectives.py --op rs_adamw

``ag_gemm``: a weight ``W [N, K]`` quantised to NF4 (block 64) and sharded over the
ranks (uniform split), activations ``X [M, K]`` bf16, output ``Y = X Wᵀ``.
  * ours: ONE kernel (gather mode of the tcgen05 pair GEMM): warps of every CTA
    read the owners' NF4 bytes over NVLink, dequantise them into a local bf16
    operand and publish per-N-tile counters that the TMA producer waits on, so
    the transfer overlaps the MMAs tile by tile (each rank starts on its own rows);
  * two_kernel: the peer gather+dequantise kernel, then the same GEMM;
  * nccl: the reference's path - NCCL all-gather of packed bytes and absmax,
    dequantise, cuBLAS GEMM.
Roofline = max(2MNK / measured bf16 peak, K·N·0.5625·(W-1)/W / 770 GB/s).

``master_gemm``: an fp32 weight ``W [N, K]`` sharded over the ranks as
train-from-scratch masters (ceil split), activations ``X [M, K]`` bf16, ``Y = X bf16(W)ᵀ``.
  * ours: ONE kernel gathers the fp32 master pieces over NVLink, casts them to bf16
    into a local operand and runs the GEMM as each N tile's rows arrive;
  * nccl: NCCL all-gather of the fp32 shards, cast, cuBLAS GEMM.
Roofline = max(2MNK / measured bf16 peak, 4·K·N·(W-1)/W / 770 GB/s).

``rs_adamw``: a flat bf16 gradient of S bytes per rank, fp32 parameters and AdamW
moments sharded 1/W.
  * ours: one peer kernel per rank sums its shard's slices from every peer, scales
    by 1/W and applies AdamW (``rs``), optionally also writing the updated shard
    into every peer's parameter buffer (``rs+ag``);
  * nccl: NCCL reduce-scatter + torch AdamW (+ NCCL all-gather of the parameters).
Roofline = max(NVLink bytes / 770 GB/s, local HBM bytes / measured copy bandwidth).

Times are CUDA-event device times after warm-up, max over ranks; inputs are far
larger than L2 for the large cases.  Rank 0 prints one JSON line per case.
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

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU on this pool


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        return json.load(open(p))
    except Exception:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def timed(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def ag_gemm(args, rank, world):
    import zeroq_b200 as zq
    from zeroq_b200.ops import _ext
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.parallel.peer import PeerShardPool

    E = _ext.ext()
    pk = peaks()
    for KN in args.kn:
        lin = Linear4bit(KN, KN, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(0)
        lin.weight = torch.nn.Parameter(torch.randn(KN, KN, device="cuda", generator=g) * 0.02,
                                        requires_grad=False)
        coord = zq.ZeroQCoordinator(zq.ZeroQConfig(exclude_modules=[], backend="nccl"))
        zq.ZeroQModuleWrapper(torch.nn.Sequential(lin), coord).partition()
        zp = coord._params[0]
        pool = PeerShardPool(coord)
        N = K = KN
        for M in args.m:
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            wb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)

            def ours():
                pool.ag_gemm(zp, x, out=y, wbuf=wb)

            def two_kernel():
                w = pool.gather_dequant(zp, N, K, out=wb.view(-1))
                E.gemm_bf16_tn(x, w, y)

            packed_full = torch.empty(zp.packed_plan.total, dtype=torch.uint8, device="cuda")
            absmax_full = torch.empty(zp.absmax_plan.total, dtype=torch.float32, device="cuda")
            wbuf = torch.empty(N * K, dtype=torch.bfloat16, device="cuda")
            equal = len(set(zp.packed_plan.lengths)) == 1 and len(set(zp.absmax_plan.lengths)) == 1

            def nccl():
                if equal:
                    dist.all_gather_into_tensor(packed_full, zp.local_packed)
                    dist.all_gather_into_tensor(absmax_full, zp.local_absmax)
                else:
                    from zeroq_b200.parallel.varlen import all_gather_by_plan
                    all_gather_by_plan(zp.local_packed, zp.packed_plan, out=packed_full)
                    all_gather_by_plan(zp.local_absmax, zp.absmax_plan, out=absmax_full)
                E.nf4_to_bf16(packed_full, absmax_full, wbuf, N, K, 64, 0, False)
                torch.matmul(x, wbuf.view(N, K).t(), out=y)

            t_ours = timed(ours, args.iters, args.warmup)
            y_ours = y.clone()
            code, detail = E.gemm_status(torch.cuda.current_device())
            if code:
                raise RuntimeError(f"ag_gemm kernel reported error {code} (detail {detail})")
            t_two = timed(two_kernel, args.iters, args.warmup)
            t_nccl = timed(nccl, args.iters, args.warmup)
            err = (y_ours.float() - y.float()).abs().max().item()
            flops = 2.0 * M * N * K
            t_comp = flops / (pk["bf16_tflops"] * 1e12) * 1e3
            t_link = K * N * 0.5625 * (world - 1) / world / (LINK_GBS * 1e9) * 1e3
            roof = max(t_comp, t_link)
            if rank == 0:
                print(json.dumps({
                    "op": "ag_dequant_gemm", "n_gpus": world, "M": M, "K": K, "N": N,
                    "ours_ms": round(t_ours, 4), "two_kernel_ms": round(t_two, 4),
                    "nccl_cublas_ms": round(t_nccl, 4),
                    "speedup": round(t_nccl / t_ours, 3),
                    "ours_tflops": round(flops / t_ours / 1e9, 1),
                    "roofline_ms": round(roof, 4), "bound": "compute" if t_comp >= t_link else "nvlink",
                    "frac_of_roofline": round(roof / t_ours, 3),
                    "roofline_basis": f"max(2MNK/{pk['bf16_tflops']} TFLOP/s measured, "
                                      f"NF4 bytes (W-1)/W / {LINK_GBS} GB/s measured)",
                    "max_abs_diff_vs_nccl": round(err, 4)}), flush=True)
            del x, y
        pool.close()
        torch.cuda.empty_cache()


def master_gemm(args, rank, world):
    from zeroq_b200.parallel.peer import PeerBuffer, ag_gemm_f32_pieces

    pk = peaks()
    for KN in args.kn:
        N = K = KN
        chunk = (N * K + world - 1) // world
        buf = PeerBuffer(chunk * 4, None)
        g = torch.Generator(device="cuda").manual_seed(0)
        full = torch.randn(N * K, device="cuda", generator=g) * 0.02
        mine = buf.tensor(chunk, torch.float32)
        mine.zero_()
        lo, hi = rank * chunk, min((rank + 1) * chunk, N * K)
        mine[: hi - lo].copy_(full[lo:hi])
        torch.cuda.synchronize()
        dist.barrier()
        starts = [q * chunk for q in range(world)]
        gathered = torch.empty(chunk * world, device="cuda")
        wb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        for M in args.m:
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

            def ours():
                ag_gemm_f32_pieces(x, buf.ptrs, starts, chunk * world, N, K, rank, out=y, wbuf=wb)

            def nccl():
                dist.all_gather_into_tensor(gathered, mine)
                w = gathered[: N * K].view(N, K).to(torch.bfloat16)
                torch.matmul(x, w.t(), out=y)

            t_ours = timed(ours, args.iters, args.warmup)
            y_ours = y.clone()
            t_nccl = timed(nccl, args.iters, args.warmup)
            err = (y_ours.float() - y.float()).abs().max().item()
            flops = 2.0 * M * N * K
            t_comp = flops / (pk["bf16_tflops"] * 1e12) * 1e3
            t_link = K * N * 4.0 * (world - 1) / world / (LINK_GBS * 1e9) * 1e3
            roof = max(t_comp, t_link)
            if rank == 0:
                print(json.dumps({
                    "op": "master_gather_cast_gemm", "n_gpus": world, "M": M, "K": K, "N": N,
                    "ours_ms": round(t_ours, 4), "nccl_cublas_ms": round(t_nccl, 4),
                    "speedup": round(t_nccl / t_ours, 3),
                    "roofline_ms": round(roof, 4), "bound": "compute" if t_comp >= t_link else "nvlink",
                    "frac_of_roofline": round(roof / t_ours, 3),
                    "max_abs_diff_vs_nccl": round(err, 4)}), flush=True)
            del x, y
        torch.cuda.synchronize()
        dist.barrier()
        buf.close()
        torch.cuda.empty_cache()


def rs_adamw(args, rank, world):
    from zeroq_b200.ops.optim import adamw_step
    from zeroq_b200.parallel.peer import PeerBuffer, PeerFlags, PeerReduceScatterAdamW

    pk = peaks()
    for mb in args.sizes_mb:
        n = int(mb * 2 ** 20) // 2
        n = (n + 4 * world - 1) // (4 * world) * (4 * world)
        shard = n // world
        gbuf = PeerBuffer(n * 2, None)
        pbuf = PeerBuffer(n * 4, None)
        grads = gbuf.tensor(n, torch.bfloat16)
        params = pbuf.tensor(n, torch.float32)
        g = torch.Generator(device="cuda").manual_seed(rank)
        grads.copy_(torch.randn(n, device="cuda", generator=g).to(torch.bfloat16))
        params.copy_(torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7)))
        m = torch.zeros(shard, device="cuda")
        v = torch.zeros(shard, device="cuda")
        op = PeerReduceScatterAdamW(gbuf, pbuf, PeerFlags(None), grad_is_bf16=True)
        lo = rank * shard
        kw = dict(lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, step=1,
                  grad_scale=1.0 / world)

        def ours_rs():
            op.run(lo, shard, m, v, push=False, **kw)

        def ours_rs_ag():
            op.run(lo, shard, m, v, push=True, **kw)

        shard_g = torch.empty(shard, dtype=torch.bfloat16, device="cuda")
        p_shard = torch.nn.Parameter(params[lo:lo + shard].clone())
        topt = torch.optim.AdamW([p_shard], lr=1e-4, foreach=True)

        def nccl_rs():
            dist.reduce_scatter_tensor(shard_g, grads, op=dist.ReduceOp.SUM)
            p_shard.grad = shard_g.float().div_(world)
            topt.step()

        def nccl_rs_ag():
            nccl_rs()
            dist.all_gather_into_tensor(params, p_shard.data)

        res = {}
        for name, fn in (("ours_rs", ours_rs), ("ours_rs_ag", ours_rs_ag), ("nccl_rs", nccl_rs),
                         ("nccl_rs_ag", nccl_rs_ag)):
            res[name] = timed(fn, args.iters, args.warmup)
        op.flags.check()
        link_rs = (world - 1) / world * n * 2 / (LINK_GBS * 1e9) * 1e3
        link_ag = (world - 1) / world * n * 4 / (LINK_GBS * 1e9) * 1e3
        hbm = (shard * (2 + 8 + 16)) / (pk["hbm_gbs"] * 1e9) * 1e3
        roof_rs = max(link_rs, hbm)
        roof_rsag = max(link_rs + link_ag, hbm)
        if rank == 0:
            print(json.dumps({
                "op": "rs_adamw", "n_gpus": world, "grad_bytes_per_rank": n * 2,
                **{k + "_ms": round(t, 4) for k, t in res.items()},
                "speedup_rs": round(res["nccl_rs"] / res["ours_rs"], 3),
                "speedup_rs_ag": round(res["nccl_rs_ag"] / res["ours_rs_ag"], 3),
                "roofline_rs_ms": round(roof_rs, 4), "roofline_rs_ag_ms": round(roof_rsag, 4),
                "frac_of_roofline_rs": round(roof_rs / res["ours_rs"], 3),
                "frac_of_roofline_rs_ag": round(roof_rsag / res["ours_rs_ag"], 3),
                "roofline_basis": f"max(NVLink bytes / {LINK_GBS} GB/s, shard HBM bytes / "
                                  f"{pk['hbm_gbs']} GB/s measured)"}), flush=True)
        del topt, p_shard
        op.flags.close()
        gbuf.close()
        pbuf.close()
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["ag_gemm", "master_gemm", "rs_adamw"], required=True)
    ap.add_argument("--kn", type=int, nargs="+", default=[4096, 8192, 12288])
    ap.add_argument("--m", type=int, nargs="+", default=[1024, 4096, 16384])
    ap.add_argument("--sizes-mb", type=float, nargs="+", default=[1, 16, 256, 1024])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=5),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    try:
        if args.op == "ag_gemm":
            ag_gemm(args, rank, world)
        elif args.op == "master_gemm":
            master_gemm(args, rank, world)
        else:
            rs_adamw(args, rank, world)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

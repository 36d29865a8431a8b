#!/usr/bin/env python
"""Run one hot kernel a few times on one GPU - the small cases profiled with ncu.

    python benchmarks/kernel_case.py gemm --m 8192 --n 3072 --k 3072 [--pair 0|1] [--nn]
    python benchmarks/kernel_case.py attention --b 8 --s 1024 --h 24 --d 128
    python benchmarks/kernel_case.py nf4_operand --n 12288 --k 3072 [--transpose]
    python benchmarks/kernel_case.py rmsnorm --m 8192 --d 3072
    python benchmarks/kernel_case.py gelu --m 8192 --n 12288

Each case allocates at most a few GB, runs ``--reps`` launches (default 4) and
prints the mean CUDA-event time of the last ``--reps - 1`` launches.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


_PROFILE = False


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    if _PROFILE:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=10))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps - 1):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / max(1, reps - 1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "attention", "nf4_operand", "rmsnorm", "gelu"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--pair", type=int, default=1)
    ap.add_argument("--b", type=int, default=8)
    ap.add_argument("--s", type=int, default=1024)
    ap.add_argument("--h", type=int, default=24)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--transpose", action="store_true")
    ap.add_argument("--nn", action="store_true", help="gemm: B given as [K, N] (MN-major read)")
    ap.add_argument("--reps", type=int, default=4)
    ap.add_argument("--profile", action="store_true", help="print one call's kernels (torch profiler)")
    a = ap.parse_args()
    global _PROFILE
    _PROFILE = a.profile

    from zeroq_b200.ops import _ext

    E = _ext.ext()
    dev = torch.device("cuda", 0)
    if a.case == "gemm":
        E.set_gemm_pair_mode(a.pair)
        x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
        y = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        if a.nn:
            w = torch.randn(a.k, a.n, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: E.gemm_bf16_nn(x, w, y, None, None), a.reps)
        else:
            w = torch.randn(a.n, a.k, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: E.gemm_bf16_tn(x, w, y), a.reps)
        print(f"gemm {a.m}x{a.n}x{a.k} pair={a.pair} nn={a.nn}: {ms:.4f} ms, "
              f"{2 * a.m * a.n * a.k / ms / 1e9:.0f} TFLOP/s, status {E.gemm_status(0)}")
    elif a.case == "attention":
        from zeroq_b200.ops.attention import flash_attention

        q = torch.randn(a.b, a.s, a.h, a.d, device=dev, dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn_like(q, requires_grad=True)
        v = torch.randn_like(q, requires_grad=True)
        go = torch.randn_like(q)

        def step():
            o = flash_attention(q, k, v, causal=True)
            o.backward(go)

        ms = _time(step, a.reps)
        fl = 4 * a.b * a.h * a.s * a.s * a.d / 2 * 3.5
        print(f"attention fwd+bwd B={a.b} S={a.s} H={a.h} D={a.d}: {ms:.4f} ms, "
              f"{fl / ms / 1e9:.0f} TFLOP/s (causal)")
    elif a.case == "nf4_operand":
        from zeroq_b200.ops.nf4 import quantize_4bit

        w = torch.randn(a.n, a.k, device=dev) * 0.02
        packed, st = quantize_4bit(w, 64, "nf4")
        out = torch.empty(a.n * a.k, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: E.nf4_to_bf16(packed, st.absmax, out, a.n, a.k, 64, 0, a.transpose), a.reps)
        byts = a.n * a.k * (0.5 + 4 / 64 + 2)
        print(f"nf4_operand {a.n}x{a.k} transpose={a.transpose}: {ms:.4f} ms, {byts / ms / 1e6:.0f} GB/s")
    elif a.case == "gelu":
        from zeroq_b200.ops.activations import gelu

        x = torch.randn(a.m, a.n, device=dev, dtype=torch.bfloat16, requires_grad=True)
        g = torch.randn_like(x)

        def step():
            gelu(x).backward(g)

        ms = _time(step, a.reps)
        print(f"gelu fwd+bwd {a.m}x{a.n}: {ms:.4f} ms, {5 * 2 * a.m * a.n / ms / 1e6:.0f} GB/s (5 passes)")
    elif a.case == "rmsnorm":
        from zeroq_b200.ops.norm import add_rmsnorm

        h = torch.randn(a.m, a.d, device=dev, dtype=torch.bfloat16, requires_grad=True)
        d = torch.randn_like(h, requires_grad=True)
        w = torch.ones(a.d, device=dev, requires_grad=True)

        def step():
            hn, y = add_rmsnorm(h, d, w)
            torch.autograd.backward([hn, y], [torch.ones_like(hn), torch.ones_like(y)])

        ms = _time(step, a.reps)
        print(f"add_rmsnorm fwd+bwd {a.m}x{a.d}: {ms:.4f} ms")


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Run one hot kernel on one GPU: CUDA-event timings and the small cases profiled with ncu.

    python benchmarks/kernel_case.py gemm --m 8192 --n 3072 --k 3072 [--pair 0|1] [--nn] [--cublas]
    python benchmarks/kernel_case.py attention --b 8 --s 1024 --h 24 --d 128
    python benchmarks/kernel_case.py nf4_operand --n 12288 --k 3072 [--transpose]
    python benchmarks/kernel_case.py rmsnorm --m 8192 --n 3072
    python benchmarks/kernel_case.py gelu --m 8192 --n 12288
    python benchmarks/kernel_case.py q4gemm --m 8192 --n 3072 --k 12288 [--nn]
    python benchmarks/kernel_case.py lora --m 8192 --k 3072 --n 3072 --r 16 [--cublas]

Each case allocates at most a few GB and times ``--reps`` launches of the kernel
itself with CUDA events on the launching stream.  Before every timed launch a
256 MB buffer (twice the 126 MB L2) is overwritten so each launch starts with a
cold L2; the flush is outside the events.  The first launch is an untimed warm-up.
``--profile`` prints the kernels of one extra call (torch profiler) for reading
only; the reported numbers never come from a profiled run.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

_FLUSH = None


def _flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def _time(fn, reps, profile=False):
    """Mean CUDA-event time (ms) of ``fn`` over ``reps`` cold-L2 launches."""
    fn()
    torch.cuda.synchronize()
    if profile:
        from torch.profiler import ProfilerActivity, profile as tprof

        with tprof(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=10))
    total = 0.0
    for _ in range(reps):
        _flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / reps


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _report(name, ms, byts=None, flops=None, extra=""):
    hbm, tf, basis = _peaks()
    parts = [f"{name}: {ms * 1e3:.1f} us"]
    if byts is not None:
        gbs = byts / ms / 1e6
        parts.append(f"{gbs:.0f} GB/s = {gbs / hbm:.2f} of {basis} HBM {hbm:.0f}")
    if flops is not None:
        t = flops / ms / 1e9
        parts.append(f"{t:.0f} TFLOP/s = {t / tf:.2f} of {basis} bf16 {tf:.0f}")
    print(", ".join(parts) + (f" {extra}" if extra else ""), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "attention", "attn_trace", "attn2_trace", "attn_bwd_trace",
                                     "nf4_operand", "rmsnorm", "gelu", "q4gemm", "gelu_gemm",
                                     "ag_gemm", "lora", "rs_adamw"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--pair", type=int, default=1)
    ap.add_argument("--nn", action="store_true", help="gemm: B given as [K, N] (MN-major read)")
    ap.add_argument("--cublas", action="store_true", help="gemm: also time torch.matmul (cuBLAS)")
    ap.add_argument("--b", type=int, default=8)
    ap.add_argument("--s", type=int, default=1024)
    ap.add_argument("--h", type=int, default=24)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--transpose", action="store_true")
    ap.add_argument("--bhsd", action="store_true", help="attn_trace: K/V as [B, H, S, D]")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--r", type=int, default=16, help="lora: adapter rank (packed width)")
    ap.add_argument("--sweep", action="store_true",
                    help="lora: time every launch shape (cluster size / splits, ring depth, "
                         "K boxes per stage) of the three kernels, read-only L2 flush")
    ap.add_argument("--world", type=int, default=4, help="ag_gemm: emulated ranks (pieces)")
    ap.add_argument("--profile", action="store_true", help="print one call's kernels (torch profiler)")
    a = ap.parse_args()

    from zeroq_b200.ops import _ext

    E = _ext.ext()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.case == "gemm":
        E.set_gemm_pair_mode(a.pair)
        x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
        y = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        fl = 2.0 * a.m * a.n * a.k
        if a.nn:
            w = torch.randn(a.k, a.n, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: E.gemm_bf16_nn(x, w, y, None, None), a.reps, a.profile)
            ref = lambda: torch.matmul(x, w, out=y)  # noqa: E731
        else:
            w = torch.randn(a.n, a.k, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: E.gemm_bf16_tn(x, w, y), a.reps, a.profile)
            ref = lambda: torch.matmul(x, w.t(), out=y)  # noqa: E731
        _report(f"gemm {a.m}x{a.n}x{a.k} pair={a.pair} nn={a.nn}", ms, flops=fl,
                extra=f"status {E.gemm_status(0)}")
        if a.cublas:
            _report(f"cublas {a.m}x{a.n}x{a.k} nn={a.nn}", _time(ref, a.reps), flops=fl)
    elif a.case == "gelu_gemm":
        # GELU MLP halves: up-projection with the GELU-output epilogue vs GEMM + GELU
        # kernel, and the down-projection input gradient with the GELU-gradient
        # epilogue vs GEMM + GELU-backward kernel (M x N output, K reduction)
        x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
        w = (torch.randn(a.n, a.k, device=dev) * 0.05).to(torch.bfloat16)
        wd = (torch.randn(a.k, a.n, device=dev) * 0.05).to(torch.bfloat16)
        h = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        act = torch.empty_like(h)
        dh = torch.empty_like(h)
        fl = 2.0 * a.m * a.n * a.k
        _report("gemm tn", _time(lambda: E.gemm_bf16_tn(x, w, h), a.reps), flops=fl)
        _report("gemm tn + gelu_fwd kernel",
                _time(lambda: (E.gemm_bf16_tn(x, w, h), E.gelu_fwd(h, act)), a.reps), flops=fl)
        _report("gemm tn, GELU-output epilogue",
                _time(lambda: E.gemm_gelu(x, w, h, act, False, None, None), a.reps, a.profile),
                flops=fl)
        _report("gemm nn", _time(lambda: E.gemm_bf16_nn(x, wd, dh, None, None), a.reps), flops=fl)
        _report("gemm nn + gelu_bwd kernel",
                _time(lambda: (E.gemm_bf16_nn(x, wd, act, None, None), E.gelu_bwd(act, h, dh)),
                      a.reps), flops=fl)
        _report("gemm nn, GELU-gradient epilogue",
                _time(lambda: E.gemm_gelu(x, wd, dh, h, True, None, None), a.reps, a.profile),
                flops=fl, extra=f"status {E.gemm_status(0)}")
    elif a.case == "ag_gemm":
        # one-kernel gather + dequantise + GEMM over `world` pieces held in separate
        # allocations of this GPU (the kernel sees only pointers, as with peers),
        # against the standalone dequantise followed by the same GEMM
        from zeroq_b200.ops.nf4 import quantize_4bit
        from zeroq_b200.parallel.peer import ag_gemm_pieces

        N, K = a.n, a.k
        packed, st = quantize_4bit(torch.randn(N, K, device=dev) * 0.02, 64, "nf4")
        packed, absmax = packed.reshape(-1), st.absmax.reshape(-1)
        pp = [packed.numel() * q // a.world // 16 * 16 for q in range(a.world)]
        ap_ = [absmax.numel() * q // a.world for q in range(a.world)]
        pk = [packed[pp[q]:(pp[q + 1] if q + 1 < a.world else None)].clone() for q in range(a.world)]
        am = [absmax[ap_[q]:(ap_[q + 1] if q + 1 < a.world else None)].clone() for q in range(a.world)]
        x = torch.randn(a.m, K, device=dev, dtype=torch.bfloat16)
        y = torch.empty(a.m, N, device=dev, dtype=torch.bfloat16)
        wb = torch.empty(N, K, device=dev, dtype=torch.bfloat16)
        fl = 2.0 * a.m * N * K
        ms = _time(lambda: ag_gemm_pieces(x, [t.data_ptr() for t in pk], pp,
                                          [t.data_ptr() for t in am], ap_, N, K, 64, "nf4", 0,
                                          out=y, wbuf=wb), a.reps, a.profile)
        _report(f"ag_gemm one kernel {a.m}x{N}x{K} pieces={a.world}", ms, flops=fl,
                extra=f"status {E.gemm_status(0)}")

        def two():
            E.nf4_to_bf16(packed, absmax, wb.view(-1), N, K, 64, 0, False)
            E.gemm_bf16_tn(x, wb, y)
        _report(f"dequantise + gemm {a.m}x{N}x{K}", _time(two, a.reps), flops=fl)
        _report(f"gemm only {a.m}x{N}x{K}", _time(lambda: E.gemm_bf16_tn(x, wb, y), a.reps), flops=fl)
    elif a.case == "q4gemm":
        # C[M, N] = X[M, K] · op(W) with W 4-bit: in-kernel decode vs operand kernel + GEMM
        from zeroq_b200.ops.nf4 import quantize_4bit

        rows, cols = (a.k, a.n) if a.nn else (a.n, a.k)
        w = torch.randn(rows, cols, device=dev) * 0.02
        packed, st = quantize_4bit(w, 64, "nf4")
        del w
        x = torch.randn(a.m, a.k, device=dev, dtype=torch.bfloat16)
        y = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        wb = torch.empty(rows * cols, device=dev, dtype=torch.bfloat16)
        fl = 2.0 * a.m * a.n * a.k
        ms = _time(lambda: E.gemm_nf4(x, packed, st.absmax, rows, cols, 64, 0, a.nn, y, None, None),
                   a.reps, a.profile)
        _report(f"gemm_nf4 (decode in kernel) {a.m}x{a.n}x{a.k} nn={a.nn}", ms, flops=fl,
                extra=f"status {E.gemm_status(0)}")

        def two_step():
            E.nf4_to_bf16(packed, st.absmax, wb, rows, cols, 64, 0, False)
            if a.nn:
                E.gemm_bf16_nn(x, wb.view(rows, cols), y, None, None)
            else:
                E.gemm_bf16_tn(x, wb.view(rows, cols), y)

        _report(f"operand kernel + gemm {a.m}x{a.n}x{a.k} nn={a.nn}", _time(two_step, a.reps), flops=fl)
    elif a.case == "attn_trace":
        # per-CTA timeline of the tcgen05 forward from its optional timestamp trace
        q = torch.randn(a.b, a.s, a.h, a.d, device=dev, dtype=torch.bfloat16)
        k, v = torch.randn_like(q), torch.randn_like(q)
        o = torch.empty_like(q)
        lse = torch.empty(a.b, a.h, a.s, device=dev)
        grid = a.b * a.h * (a.s // 128)
        tr = torch.zeros(grid, 32, dtype=torch.int64, device=dev)
        scale = a.d ** -0.5
        if a.bhsd:  # K/V handed over head-major: every key tile is one contiguous block
            k, v = k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous()
        for _ in range(3):
            E.attn_fwd_tc(q, k, v, o, lse, True, scale, None, a.bhsd)
        torch.cuda.synchronize()
        ms = _time(lambda: E.attn_fwd_tc(q, k, v, o, lse, True, scale, None, a.bhsd), a.reps)
        _report(f"attn_fwd_tc kv_bhsd={a.bhsd}", ms, flops=4.0 * a.b * a.h * a.s * a.s * a.d / 2)
        E.attn_fwd_tc(q, k, v, o, lse, True, scale, tr, a.bhsd)
        torch.cuda.synchronize()
        t = tr.cpu().double()
        n = t[:, 31].long()
        print(f"attn trace B={a.b} S={a.s} H={a.h}: kernel span "
              f"{(t[:, 30].max() - t[:, 0].min()) / 1e3:.1f} us over {grid} CTAs")
        print(f"  CTA start -> first S ready: mean {((t[:, 1] - t[:, 0]) / 1e3).mean():.2f} us")
        names = ["S ready", "max exchanged", "exps done", "P stored", "p_full arrived",
                 "MMA: K_next seen", "MMA: S_next issued", "MMA: p_full seen", "MMA: V seen",
                 "MMA: PV issued", "K_next load issued", "V load issued"]
        sel = n >= 4  # CTAs that ran tiles 0..3
        if sel.any():
            base = t[sel]
            for j in range(1, 3):
                s0 = base[:, 2 + 12 * (j - 1)]
                row = [f"{nm} {((base[:, 2 + 12 * (j - 1) + i] - s0) / 1e3).mean():+.3f}"
                       for i, nm in enumerate(names) if i > 0]
                nxt = ((base[:, 2 + 12 * j] - s0) / 1e3).mean() if j < 2 else float("nan")
                print(f"  tile {j} (us from S ready): " + ", ".join(row) + f"; next S ready +{nxt:.3f}")
        last_end = t[:, 30]
        print(f"  CTA duration mean {((last_end - t[:, 0]) / 1e3).mean():.2f} us")
    elif a.case == "attn2_trace":
        # per-CTA timeline of the two-query-tile forward (S a multiple of 256)
        q = torch.randn(a.b, a.s, a.h, a.d, device=dev, dtype=torch.bfloat16)
        k, v = torch.randn_like(q), torch.randn_like(q)
        o = torch.empty_like(q)
        lse = torch.empty(a.b, a.h, a.s, device=dev)
        grid = a.b * a.h * (a.s // 256)
        tr = torch.zeros(grid, 32, dtype=torch.int64, device=dev)
        scale = a.d ** -0.5
        for _ in range(3):
            E.attn_fwd_tc(q, k, v, o, lse, True, scale)
        torch.cuda.synchronize()
        ms = _time(lambda: E.attn_fwd_tc(q, k, v, o, lse, True, scale), a.reps)
        _report("attn_fwd_tc (two query tiles)", ms, flops=4.0 * a.b * a.h * a.s * a.s * a.d / 2)
        E.attn_fwd_tc(q, k, v, o, lse, True, scale, tr)
        torch.cuda.synchronize()
        t = tr.cpu().double()
        n = t[:, 31].long()
        print(f"attn2 trace B={a.b} S={a.s} H={a.h}: kernel span "
              f"{(t[:, 30].max() - t[:, 0].min()) / 1e3:.1f} us over {grid} CTAs")
        base = t[n >= 4]
        names = ["in registers", "row max", "exps", "P stored", "p_full arrived"]
        for x, tile in ((0, "A"), (1, "B")):
            for j in (1, 2):
                o0 = 1 + 6 * (2 * x + j - 1)
                s0 = base[:, o0]
                row = [f"{nm} {((base[:, o0 + i + 1] - s0) / 1e3).mean():+.3f}" for i, nm in enumerate(names)]
                print(f"  tile {tile} key {j} (us from S ready): " + ", ".join(row))
            per = ((base[:, 1 + 6 * (2 * x + 1)] - base[:, 1 + 6 * (2 * x)]) / 1e3).mean()
            print(f"  tile {tile}: S ready(2) - S ready(1) = {per:.3f} us")
        a1, b1 = base[:, 6], base[:, 18]
        print(f"  MMA: p_full A(1) seen {((base[:, 25] - a1) / 1e3).mean():+.3f} us after the arrival, "
              f"PV A(1) + S A(2) issued {((base[:, 26] - a1) / 1e3).mean():+.3f}; "
              f"S A(2) ready {((base[:, 7] - a1) / 1e3).mean():+.3f}")
        print(f"  MMA: p_full B(1) seen {((base[:, 27] - b1) / 1e3).mean():+.3f} us after the arrival, "
              f"PV B(1) + S B(2) issued {((base[:, 28] - b1) / 1e3).mean():+.3f}; "
              f"S B(2) ready {((base[:, 19] - b1) / 1e3).mean():+.3f}")
        print(f"  CTA duration mean {((t[:, 30] - t[:, 0]) / 1e3).mean():.2f} us, "
              f"start -> S A(1) ready {((base[:, 1] - base[:, 0]) / 1e3).mean():.2f} us")
    elif a.case == "attn_bwd_trace":
        # per-CTA timelines of the tcgen05 backward kernels (dQ, then dK/dV)
        q = torch.randn(a.b, a.s, a.h, a.d, device=dev, dtype=torch.bfloat16)
        k, v, do = torch.randn_like(q), torch.randn_like(q), torch.randn_like(q)
        o = torch.empty_like(q)
        lse = torch.empty(a.b, a.h, a.s, device=dev)
        scale = a.d ** -0.5
        E.attn_fwd_tc(q, k, v, o, lse, True, scale)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        g = a.b * a.h * (a.s // 128)
        tr = torch.zeros(2 * g, 32, dtype=torch.int64, device=dev)
        for _ in range(3):
            E.attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, True, scale)
        torch.cuda.synchronize()
        ms = _time(lambda: E.attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, True, scale), a.reps)
        _report("attn_bwd_tc (delta + dQ + dK/dV)", ms,
                flops=2.5 * 4.0 * a.b * a.h * a.s * a.s * a.d / 2)
        E.attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, True, scale, tr)
        torch.cuda.synchronize()
        t = tr.cpu().double()
        names = ["S/dP seen", "loaded", "computed", "arrived", "MMA: inputs seen", "MMA: S/dP issued",
                 "MMA: dS seen", "MMA: grads issued"]
        for label, part in (("dQ", t[:g]), ("dK/dV", t[g:])):
            sel = (part[:, 1] > 0) & (part[:, 9] > 0) & (part[:, 16] > 0)
            print(f"{label}: CTA span mean {((part[:, 30] - part[:, 0]) / 1e3).mean():.2f} us")
            if sel.any():
                p = part[sel]
                for j in (1, 2):
                    s0 = p[:, 1 + 8 * (j - 1)]
                    row = [f"{nm} {((p[:, 1 + 8 * (j - 1) + i] - s0) / 1e3).mean():+.3f}"
                           for i, nm in enumerate(names) if i > 0]
                    print(f"  tile {j}: " + ", ".join(row))
                print(f"  tile 1 -> tile 2 S/dP seen: {((p[:, 9] - p[:, 1]) / 1e3).mean():.3f} us")
    elif a.case == "attention":
        from zeroq_b200.ops.attention import flash_attention

        q = torch.randn(a.b, a.s, a.h, a.d, device=dev, dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn_like(q, requires_grad=True)
        v = torch.randn_like(q, requires_grad=True)
        go = torch.randn_like(q)
        fwd_fl = 4.0 * a.b * a.h * a.s * a.s * a.d / 2  # causal
        with torch.no_grad():
            ms_f = _time(lambda: flash_attention(q, k, v, causal=True), a.reps, a.profile)
        _report(f"attention fwd B={a.b} S={a.s} H={a.h} D={a.d} causal", ms_f, flops=fwd_fl)

        def step():
            o = flash_attention(q, k, v, causal=True)
            o.backward(go)

        ms = _time(step, a.reps, a.profile)
        _report(f"attention fwd+bwd B={a.b} S={a.s} H={a.h} D={a.d} causal", ms,
                flops=fwd_fl * 3.5)
        if a.d == 128:
            # backward kernels alone, plain and with the inverse-RoPE dQ/dK epilogue
            from zeroq_b200.ops.rope import rope_table

            qd, kd, vd = q.detach(), k.detach(), v.detach()
            o = torch.empty_like(qd)
            lse = torch.empty(a.b, a.h, a.s, device=dev)
            E.attn_fwd_tc(qd, kd, vd, o, lse, True, a.d ** -0.5)
            dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
            cs = rope_table(a.s, a.d, 10000.0, dev)
            for name, t in (("plain", None), ("inverse-RoPE epilogue", cs)):
                ms_b = _time(lambda: E.attn_bwd_tc(go, qd, kd, vd, o, lse, dq, dk, dv, True,
                                                   a.d ** -0.5, None, t), a.reps)
                _report(f"attention bwd kernels ({name})", ms_b, flops=fwd_fl * 2.5)
    elif a.case == "rs_adamw":
        # the fused reduce-scatter + AdamW (+ all-gather) kernel on one GPU: world 1,
        # epoch 0 (no cross-rank barrier), so it runs its memory traffic alone:
        # per element it reads the gradient, master, m and v and writes master, m,
        # v and the pushed parameter copy (here the same buffer)
        n = a.n * a.k
        g = torch.randn(n, device=dev) * 1e-3
        master = torch.randn(n, device=dev)
        m_ = torch.zeros(n, device=dev)
        v_ = torch.zeros(n, device=dev)
        flags = torch.zeros(64, dtype=torch.int32, device=dev)

        def run():
            E.rs_adamw([g.data_ptr()], [master.data_ptr()], [flags.data_ptr()], 0, 0, 0, n,
                       m_, v_, 0, 1e-4, 0.9, 0.999, 1e-8, 0.0, 0.1, 0.001, 1.0, True, 0)

        ms = _time(run, a.reps, a.profile)
        _report(f"rs_adamw world 1, {n} fp32 elements", ms, byts=7 * 4 * n)
    elif a.case == "nf4_operand":
        from zeroq_b200.ops.nf4 import quantize_4bit

        w = torch.randn(a.n, a.k, device=dev) * 0.02
        packed, st = quantize_4bit(w, 64, "nf4")
        out = torch.empty(a.n * a.k, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: E.nf4_to_bf16(packed, st.absmax, out, a.n, a.k, 64, 0, a.transpose),
                   a.reps, a.profile)
        _report(f"nf4_operand {a.n}x{a.k} transpose={a.transpose}", ms,
                byts=a.n * a.k * (0.5 + 4 / 64 + 2))
    elif a.case == "rmsnorm":
        M, D = a.m, a.n
        h = torch.randn(M, D, device=dev, dtype=torch.bfloat16)
        d = torch.randn_like(h)
        w = torch.ones(D, device=dev)
        hout, y = torch.empty_like(h), torch.empty_like(h)
        rstd = torch.empty(M, device=dev)
        ms = _time(lambda: E.add_rmsnorm_fwd(h, d, w, hout, y, rstd, 1e-6), a.reps, a.profile)
        _report(f"add_rmsnorm fwd {M}x{D}", ms, byts=4 * M * D * 2)
        gy, gh, dx = torch.randn_like(h), torch.randn_like(h), torch.empty_like(h)
        part = torch.empty(2 * torch.cuda.get_device_properties(dev).multi_processor_count, D,
                           device=dev)
        ms = _time(lambda: E.rmsnorm_bwd(gy, hout, w, rstd, gh, dx, part), a.reps)
        _report(f"rmsnorm bwd (+residual grad) {M}x{D}", ms, byts=4 * M * D * 2)
    elif a.case == "lora":
        # the four rank-space products of one adapter on x [M, K] -> y [M, N]
        from zeroq_b200.ops import lora as L

        M, K, N, r = a.m, a.k, a.n, a.r
        r16 = L.round16(r)
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        gy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        sa = (0.02 * torch.randn(r16, K, device=dev)).bfloat16()
        bt = (0.02 * torch.randn(r16, N, device=dev)).bfloat16()
        u, ut = L.down(x, sa)
        v, vt = L.down(gy, bt)
        gA = torch.zeros(r, K, device=dev)
        gB = torch.zeros(N, r, device=dev)
        ms = _time(lambda: L.down(x, sa), a.reps, a.profile)
        _report(f"lora_down U=x·Aᵀ {M}x{K} r={r}", ms, byts=M * K * 2 + M * (64 + r16) * 2)
        ms = _time(lambda: L.down(gy, bt), a.reps)
        _report(f"lora_down V=dY·B {M}x{N} r={r}", ms, byts=M * N * 2 + M * (64 + r16) * 2)
        ms = _time(lambda: L.wgrad(x, vt, r16, [(0, K, 0, 1.0)], [gA], r16, r, True), a.reps)
        _report(f"lora_wgrad dA=Vᵀ·x {M}x{K} r={r}", ms, byts=M * K * 2 + M * r16 * 2)
        ms = _time(lambda: L.wgrad(gy, ut, r16, [(0, N, 0, 1.0)], [gB], r16, r, False), a.reps)
        _report(f"lora_wgrad dB=dYᵀ·U {M}x{N} r={r}", ms, byts=M * N * 2 + M * r16 * 2)
        if L.vdb(gy, bt, ut, 64, [(0, N, 0)], [gB], r16, r) is not None:
            ms = _time(lambda: L.vdb(gy, bt, ut, 64, [(0, N, 0)], [gB], r16, r), a.reps)
            _report(f"lora_vdb V and dB {M}x{N} r={r}", ms, byts=M * N * 2 + M * (64 + 2 * r16) * 2)
        if a.sweep:
            flush = torch.ones(64 << 20, device=dev)  # 256 MB read between launches

            def tro(fn, reps=10):
                fn()
                torch.cuda.synchronize()
                tot = 0.0
                for _ in range(reps):
                    flush.sum()
                    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s0.record()
                    fn()
                    e0.record()
                    torch.cuda.synchronize()
                    tot += s0.elapsed_time(e0)
                return tot / reps

            import itertools

            ut2 = torch.empty(r16, M, device=dev, dtype=torch.bfloat16)
            u2 = torch.empty(M, 64, device=dev, dtype=torch.bfloat16)
            for cs, st, kb in itertools.product((1, 2, 4, 8), (4, 6), (1, 2)):
                _report(f"sweep lora_down {M}x{K} cs={cs} stages={st} kb={kb}",
                        tro(lambda: E.lora_down(x, sa, u2, ut2, cs, st, kb)), byts=M * K * 2)
            for sp, st, kb in itertools.product((0, 6, 13, 26), (4, 6), (1, 2)):
                _report(f"sweep lora_wgrad dA {M}x{K} splits={sp} stages={st} kb={kb}",
                        tro(lambda: E.lora_wgrad(x, vt, r16, [0], [K], [0], [1.0], [gA], r16, r,
                                                 True, sp, st, kb)), byts=M * K * 2)
            for cs, st in itertools.product((1, 2, 4, 8), (4, 6)):
                v2 = torch.empty(M, 64, device=dev, dtype=torch.bfloat16)
                vt2 = torch.empty(r16, M, device=dev, dtype=torch.bfloat16)
                if E.lora_vdb(gy, bt, ut, v2, vt2, r16, [0], [N], [0], [gB], r, cs, st):
                    _report(f"sweep lora_vdb {M}x{N} cs={cs} stages={st}",
                            tro(lambda: E.lora_vdb(gy, bt, ut, v2, vt2, r16, [0], [N], [0], [gB], r,
                                                   cs, st)), byts=M * N * 2)
                else:
                    print(f"sweep lora_vdb {M}x{N} cs={cs} stages={st}: declined (TMEM)")
        if a.cublas:
            ap_, bp_ = torch.zeros(64, K, device=dev, dtype=torch.bfloat16), torch.zeros(
                N, 64, device=dev, dtype=torch.bfloat16)
            _report(f"cublas x·A_padᵀ {M}x{K}x64", _time(lambda: x @ ap_.t(), a.reps),
                    byts=M * K * 2 + M * 64 * 2)
            _report(f"cublas dY·B_pad {M}x{N}x64", _time(lambda: gy @ bp_, a.reps),
                    byts=M * N * 2 + M * 64 * 2)
        print(f"status {E.gemm_status(0)}", flush=True)
    elif a.case == "gelu":
        x = torch.randn(a.m, a.n, device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        ms = _time(lambda: E.gelu_fwd(x, y), a.reps, a.profile)
        _report(f"gelu fwd {a.m}x{a.n}", ms, byts=2 * a.m * a.n * 2)
        g, dx = torch.randn_like(x), torch.empty_like(x)
        ms = _time(lambda: E.gelu_bwd(g, x, dx), a.reps)
        _report(f"gelu bwd {a.m}x{a.n}", ms, byts=3 * a.m * a.n * 2)


if __name__ == "__main__":
    main()

"""Numerics of each sm_100a kernel against a plain PyTorch fp32 reference of the same op."""

import math

import pytest
import torch

from zeroq_b200.ops import _ext
from zeroq_b200.ops.nf4 import (dequantize_4bit_reference, quantize_4bit,
                                quantize_4bit_reference)

pytestmark = pytest.mark.gpu


def _status_ok(dev):
    code, detail = _ext.ext().gemm_status(dev.index or 0)
    assert code == 0, f"device status error {code} (detail {detail})"


@pytest.mark.parametrize("quant_type", ["nf4", "fp4"])
@pytest.mark.parametrize("blocksize", [64, 256, 1024])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_matches_oracle_bit_exact(cuda, quant_type, blocksize, dtype):
    torch.manual_seed(0)
    x = (torch.randn(1000003, dtype=torch.float32) * 0.02).to(dtype)
    x[:blocksize] = 0  # an all-zero block
    p_ref, a_ref = quantize_4bit_reference(x, blocksize, quant_type)
    p, st = quantize_4bit(x.to(cuda), blocksize, quant_type)
    assert torch.equal(p.cpu(), p_ref)
    assert torch.equal(st.absmax.cpu(), a_ref)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dequantize_matches_oracle(cuda, out_dtype):
    torch.manual_seed(1)
    x = torch.randn(4096 * 33 + 7) * 0.02
    p, a = quantize_4bit_reference(x, 64, "nf4")
    ref = dequantize_4bit_reference(p, a, x.numel(), 64, "nf4", out_dtype)
    out = torch.empty(x.numel(), dtype=out_dtype, device=cuda)
    _ext.ext().nf4_dequantize(p.to(cuda), a.to(cuda), out, x.numel(), 64, 0)
    assert torch.equal(out.cpu(), ref)


@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 512, 128), (1000, 768, 320),
                                   (8192 // 4, 3072, 3072), (333, 200, 64), (4096, 12288, 3072),
                                   (300, 136, 256), (2048, 50304, 128)])
def test_gemm_bf16_tn(cuda, shape):
    M, N, K = shape
    torch.manual_seed(2)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda, dtype=torch.bfloat16)
    c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    _ext.ext().gemm_bf16_tn(a, b, c)
    torch.cuda.synchronize()
    _status_ok(cuda)
    # strided output (a column block of a wider matrix) through the TMA-store epilogue
    wide = torch.zeros(M, N + 64, device=cuda, dtype=torch.bfloat16)
    _ext.ext().gemm_bf16_tn(a, b, wide[:, 32:32 + N])
    torch.cuda.synchronize()
    assert torch.equal(wide[:, 32:32 + N], c)
    assert torch.all(wide[:, :32] == 0) and torch.all(wide[:, 32 + N:] == 0)
    ref = a.float() @ b.float().t()
    err = (c.float() - ref).abs().max().item()
    tol = 2e-2 * math.sqrt(K) + 1e-2 * ref.abs().max().item()
    assert err < tol, (err, tol)


@pytest.mark.parametrize("K", [192, 256, 3072])
def test_gemm_extra_slab(cuda, K):
    M, N = 640, 448
    torch.manual_seed(3)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=cuda, dtype=torch.bfloat16)
    a2 = torch.zeros(M, 64, device=cuda, dtype=torch.bfloat16)
    b2 = torch.zeros(N, 64, device=cuda, dtype=torch.bfloat16)
    a2[:, :16] = torch.randn(M, 16, device=cuda).bfloat16()
    b2[:, :16] = torch.randn(N, 16, device=cuda).bfloat16()
    c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    _ext.ext().gemm_bf16_tn_extra(a, b, c, a2, b2)
    torch.cuda.synchronize()
    _status_ok(cuda)
    ref = a.float() @ b.float().t() + a2.float() @ b2.float().t()
    tol = 2e-2 * math.sqrt(K) + 1e-2 * ref.abs().max().item()
    assert (c.float() - ref).abs().max().item() < tol


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("R,C,bs,qt", [(384, 1280, 64, "nf4"), (33, 48, 64, "nf4"),
                                       (640, 1024, 128, "fp4"), (1000, 3072, 256, "nf4")])
def test_nf4_to_bf16(cuda, transpose, R, C, bs, qt):
    """Flat (non-transposed, 32-aligned) and tiled paths, both code tables."""
    from zeroq_b200.ops.nf4 import QUANT_TYPE_ID

    if transpose and R % 16:
        pytest.skip("transposed output needs rows % 16 == 0")
    w = torch.randn(R, C) * 0.02
    p, a = quantize_4bit_reference(w, bs, qt)
    ref = dequantize_4bit_reference(p, a, R * C, bs, qt, torch.bfloat16).view(R, C)
    out = torch.empty(R * C, dtype=torch.bfloat16, device=cuda)
    _ext.ext().nf4_to_bf16(p.to(cuda), a.to(cuda), out, R, C, bs, QUANT_TYPE_ID[qt], transpose)
    got = out.view(C, R).t() if transpose else out.view(R, C)
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("M,D", [(300, 3072), (1001, 256), (77, 2056), (513, 3584), (130, 5120),
                                 (64, 8192), (4099, 3072), (20001, 512), (333, 1024), (1500, 2048),
                                 (200, 6144)])
def test_add_rmsnorm_fwd_bwd(cuda, M, D):
    """Every team width (32/64/128 lanes) and chunk count, ragged row counts."""
    from zeroq_b200.ops.norm import add_rmsnorm

    torch.manual_seed(4)
    h = torch.randn(M, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    d = torch.randn(M, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device=cuda)).requires_grad_(True)
    hn, y = add_rmsnorm(h, d, w, 1e-6)
    g_h = torch.randn_like(hn)
    g_y = torch.randn_like(y)
    (hn.float() * g_h.float()).sum().add((y.float() * g_y.float()).sum()).backward()
    hr = h.detach().float().requires_grad_(True)
    dr = d.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    s = (hr + dr).bfloat16().float()
    yr = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    ((hr + dr) * g_h.float()).sum().add((yr * g_y.float()).sum()).backward()
    assert (y.float() - yr).abs().max() < 3e-2
    assert (h.grad.float() - hr.grad).abs().max() < 5e-2
    assert (d.grad.float() - dr.grad).abs().max() < 5e-2
    assert (w.grad - wr.grad).abs().max() / wr.grad.abs().max() < 1e-2


def test_rope(cuda):
    from zeroq_b200.ops.rope import apply_rope, rope_reference

    q = torch.randn(2, 64, 4, 128, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(2, 64, 2, 128, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    qo, ko = apply_rope(q, k, 1e6)
    assert (qo.float() - rope_reference(q.detach(), 1e6).float()).abs().max() < 2e-2
    assert (ko.float() - rope_reference(k.detach(), 1e6).float()).abs().max() < 2e-2
    (qo.float().sum() + ko.float().sum()).backward()
    qr = q.detach().float().requires_grad_(True)
    rope_reference(qr, 1e6).sum().backward()
    assert (q.grad.float() - qr.grad).abs().max() < 3e-2


def test_gelu_cdf_pdf_error_bound(cuda):
    """The GELU CDF (Abramowitz & Stegun 7.1.26 erf, |e| <= 1.5e-7) and PDF in
    fp32 against CUDA's erf/exp as called by PyTorch."""
    x = torch.linspace(-12.0, 12.0, 1 << 20, device=cuda)
    cdf = torch.empty_like(x)
    pdf = torch.empty_like(x)
    _ext.ext().gelu_cdf_pdf(x, cdf, pdf)
    torch.cuda.synchronize()
    xd = x.double()
    ref_cdf = 0.5 * (1.0 + torch.special.erf(xd / math.sqrt(2.0)))
    ref_pdf = torch.exp(-0.5 * xd * xd) / math.sqrt(2.0 * math.pi)
    assert (cdf.double() - ref_cdf).abs().max().item() < 1e-6
    rel = ((pdf.double() - ref_pdf).abs() / ref_pdf.clamp_min(1e-30))[ref_pdf > 1e-30]
    assert rel.max().item() < 1e-5


@pytest.mark.parametrize("n", [8, 8 * 1023, 8 * 4097, 3 * 1024 * 1024])
def test_gelu_ragged_sizes(cuda, n):
    from zeroq_b200.ops.activations import gelu

    torch.manual_seed(5)
    x = torch.randn(n, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = gelu(x)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    yr = torch.nn.functional.gelu(xr)
    yr.backward(g.float())
    assert (y.float() - yr).abs().max().item() < 2e-2
    assert (x.grad.float() - xr.grad).abs().max().item() < 3e-2


def test_gelu_swiglu(cuda):
    from zeroq_b200.ops.activations import gelu, swiglu

    x = torch.randn(4096, 1024, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    u = torch.randn(4096, 1024, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = gelu(x)
    xr = x.detach().float().requires_grad_(True)
    yr = torch.nn.functional.gelu(xr)
    assert (y.float() - yr).abs().max() < 2e-2
    y.float().sum().backward()
    yr.sum().backward()
    assert (x.grad.float() - xr.grad).abs().max() < 2e-2
    x.grad = None
    z = swiglu(x, u)
    xr2 = x.detach().float().requires_grad_(True)
    ur2 = u.detach().float().requires_grad_(True)
    zr = torch.nn.functional.silu(xr2) * ur2
    assert (z.float() - zr).abs().max() < 5e-2
    z.float().sum().backward()
    zr.sum().backward()
    assert (x.grad.float() - xr2.grad).abs().max() < 5e-2
    assert (u.grad.float() - ur2.grad).abs().max() < 5e-2


def test_cross_entropy(cuda):
    from zeroq_b200.ops.cross_entropy import cross_entropy

    torch.manual_seed(5)
    M, V, Vp = 257, 50257, 50304
    logits = torch.randn(M, Vp, device=cuda, dtype=torch.bfloat16) * 3
    t = torch.randint(0, V, (M,), device=cuda)
    t[5] = -100
    lg = logits.clone().requires_grad_(True)
    loss = cross_entropy(lg, t, vocab=V)
    lr = logits[:, :V].float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(lr, t, ignore_index=-100)
    assert abs(loss.item() - ref.item()) < 1e-3
    loss.backward()
    ref.backward()
    g = lg.grad.float()
    assert (g[:, :V] - lr.grad).abs().max() < 1e-4
    assert g[:, V:].abs().max() == 0


def test_adamw_lion(cuda):
    from zeroq_b200.ops.optim import adamw_step, lion_step

    n = 100003
    p = torch.randn(n, device=cuda)
    g = torch.randn(n, device=cuda)
    m = torch.zeros(n, device=cuda)
    v = torch.zeros(n, device=cuda)
    pc, gc, mc, vc = p.cpu(), g.cpu(), m.cpu(), v.cpu()
    for step in (1, 2):
        adamw_step(p, g, m, v, lr=1e-3, weight_decay=0.1, step=step, grad_scale=0.5)
        adamw_step(pc, gc, mc, vc, lr=1e-3, weight_decay=0.1, step=step, grad_scale=0.5)
    assert (p.cpu() - pc).abs().max() < 1e-6
    mom = torch.zeros(n, device=cuda)
    mom_c = mom.cpu()
    w = torch.randn(n, device=cuda)
    wc = w.cpu()
    lion_step(w, g, mom, lr=1e-3, wd=0.01, seed=7)
    lion_step(wc, gc, mom_c, lr=1e-3, wd=0.01, seed=7)
    assert (w.cpu() - wc).abs().max() < 1e-6
    # fp16 master: stochastic rounding stays within one fp16 ulp of the fp32 update
    w16 = torch.randn(n, device=cuda).half()
    ref = w16.float().cpu()
    m16 = torch.zeros(n, device=cuda)
    lion_step(w16, g, m16, lr=1e-3, wd=0.0, seed=3)
    upd = ref - 1e-3 * torch.sign(0.1 * g.cpu())
    assert ((w16.float().cpu() - upd).abs() <= upd.abs() * 2e-3 + 1e-4).all()


@pytest.mark.parametrize("cfg", [(2, 256, 4, 4, 128), (1, 512, 8, 2, 128), (2, 128, 4, 4, 64),
                                 (1, 384, 6, 3, 64)])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_attention_fwd_bwd(cuda, cfg, causal):
    from zeroq_b200.ops.attention import attention_reference, flash_attention

    B, S, Hq, Hk, D = cfg
    torch.manual_seed(6)
    q = torch.randn(B, S, Hq, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    o = flash_attention(q, k, v, causal=causal)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    orf = attention_reference(qr, kr, vr, causal=causal)
    assert (o.float() - orf).abs().max().item() < 2e-2
    go = torch.randn_like(o)
    o.backward(go)
    orf.backward(go.float())
    for a, r in ((q.grad, qr.grad), (k.grad, kr.grad), (v.grad, vr.grad)):
        err = (a.float() - r).abs().max().item()
        assert err < 5e-2 * max(1.0, r.abs().max().item()), err


@pytest.mark.parametrize("shape", [(256, 128, 64), (512, 384, 192), (1000, 768, 320),
                                   (2048, 3072, 3072), (8192, 3072, 12288)])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_bf16_nn_mn_major_b(cuda, shape, extra):
    """C = A @ B with B row-major [K, N] (the tensor core reads B MN-major)."""
    M, N, K = shape
    torch.manual_seed(8)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(K, N, device=cuda, dtype=torch.bfloat16)
    c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = torch.zeros(M, 64, device=cuda, dtype=torch.bfloat16)
        b2 = torch.zeros(64, N, device=cuda, dtype=torch.bfloat16)
        a2[:, :16] = torch.randn(M, 16, device=cuda).bfloat16()
        b2[:16] = torch.randn(16, N, device=cuda).bfloat16()
    _ext.ext().gemm_bf16_nn(a, b, c, a2, b2)
    torch.cuda.synchronize()
    _status_ok(cuda)
    ref = a.float() @ b.float()
    if extra:
        ref = ref + a2.float() @ b2.float()
    tol = 2e-2 * math.sqrt(K) + 1e-2 * ref.abs().max().item()
    assert (c.float() - ref).abs().max().item() < tol


@pytest.mark.parametrize("M", [96, 512, 2048])
@pytest.mark.parametrize("lora_r", [0, 16])
def test_nf4_linear_fwd_bwd_vs_fp32(cuda, M, lora_r):
    """Fused NF4 linear (operand kernel + tcgen05 GEMM + LoRA slab) against the
    fp32 oracle of the same op: output, input gradient and LoRA gradients."""
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(11)
    K, N = 768, 1280
    lin = Linear4bit(K, N, lora_r=lora_r, lora_alpha=32.0, device=cuda)
    lin.quantize_from(torch.randn(N, K, device=cuda) * 0.05)
    if lora_r:
        with torch.no_grad():
            lin.lora_B.normal_(0.0, 0.05)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(M, N, device=cuda, dtype=torch.bfloat16)
    y = lin(x)
    y.backward(gy)
    torch.cuda.synchronize()
    _status_ok(cuda)

    w = lin.dequantized_weight(torch.float32)
    xf = x.detach().float().requires_grad_(True)
    params = []
    yr = xf @ w.t()
    if lora_r:
        A = lin.lora_A.detach().clone().requires_grad_(True)
        B = lin.lora_B.detach().clone().requires_grad_(True)
        params = [A, B]
        yr = yr + (xf @ A.t()) @ B.t() * lin.scaling
    yr.backward(gy.float())

    def close(a, b, rel):
        return (a.float() - b).abs().max().item() <= rel * b.abs().max().item() + 1e-3

    assert close(y, yr.detach(), 2e-2)
    assert close(x.grad, xf.grad, 2e-2)
    if lora_r:
        assert close(lin.lora_A.grad, params[0].grad, 3e-2)
        assert close(lin.lora_B.grad, params[1].grad, 3e-2)


def test_lm_head_grad_vs_fp32(cuda):
    """Tied LM head: logits = h·Eᵀ and dh = dlogits·E (E read MN-major in place)."""
    from zeroq_b200.ops.gemm import LMHeadFunction

    torch.manual_seed(12)
    M, d, V = 1024, 512, 4096
    h = torch.randn(M, d, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    E = (torch.randn(V, d, device=cuda) * 0.05).bfloat16().requires_grad_(True)
    g = torch.randn(M, V, device=cuda, dtype=torch.bfloat16)
    logits = LMHeadFunction.apply(h, E)
    logits.backward(g)
    torch.cuda.synchronize()
    _status_ok(cuda)
    hf, Ef = h.detach().float(), E.detach().float()
    ref_dh = g.float() @ Ef
    ref_dE = g.float().t() @ hf
    assert (logits.float() - hf @ Ef.t()).abs().max().item() < 2e-2 * (hf @ Ef.t()).abs().max().item() + 1e-2
    assert (h.grad.float() - ref_dh).abs().max().item() < 2e-2 * ref_dh.abs().max().item() + 1e-2
    assert (E.grad.float() - ref_dE).abs().max().item() < 2e-2 * ref_dE.abs().max().item() + 1e-2


def test_nf4_linear_flat_grads_and_lora_cache(cuda):
    """FlatParams-bound LoRA weights: gradients accumulate in place in fp32 over
    two backward passes, and the cached padded operands follow an update
    written by a kernel once the optimizer marks the buffers updated."""
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.parallel.optimizer import FlatParams

    torch.manual_seed(13)
    K, N, M = 512, 768, 512
    lin = Linear4bit(K, N, lora_r=8, lora_alpha=16.0, device=cuda)
    lin.quantize_from(torch.randn(N, K, device=cuda) * 0.05)
    with torch.no_grad():
        lin.lora_B.normal_(0.0, 0.05)
    flat = FlatParams([lin.lora_A, lin.lora_B])
    w = lin.dequantized_weight(torch.float32)

    def ref_grads(x, gy):
        xf = x.float()
        A = lin.lora_A.detach().clone().requires_grad_(True)
        B = lin.lora_B.detach().clone().requires_grad_(True)
        y = xf @ w.t() + (xf @ A.t()) @ B.t() * lin.scaling
        y.backward(gy.float())
        return y.detach(), A.grad, B.grad

    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    gy = torch.randn(M, N, device=cuda, dtype=torch.bfloat16)
    _, rA, rB = ref_grads(x, gy)
    for _ in range(2):
        lin(x).backward(gy)
    torch.cuda.synchronize()
    assert lin.lora_A.grad.data_ptr() == flat.grad.data_ptr()
    tolA = 3e-2 * rA.abs().max().item()
    tolB = 3e-2 * rB.abs().max().item()
    assert (lin.lora_A.grad - 2 * rA).abs().max().item() < 2 * tolA
    assert (lin.lora_B.grad - 2 * rB).abs().max().item() < 2 * tolB

    # an update that bypasses autograd's counters, then the optimizer's notice
    with torch.no_grad():
        flat.data.mul_(1.5)
    flat.mark_updated()
    y = lin(x)
    yr, _, _ = ref_grads(x, gy)
    assert (y.float() - yr).abs().max().item() < 2e-2 * yr.abs().max().item()


@pytest.mark.parametrize("M,rows,cols", [(256, 256, 128), (300, 320, 384), (1000, 1280, 768),
                                         (2048, 3072, 3072), (512, 12288, 3072)])
@pytest.mark.parametrize("w_is_kn", [False, True])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_nf4_in_kernel_decode_matches_operand_path(cuda, M, rows, cols, w_is_kn, extra):
    """The GEMM that decodes the 4-bit weight inside its B producer gives exactly
    the result of the standalone operand kernel followed by the bf16 GEMM (same
    decoded bits, same MMA order), forward (C = A·Wᵀ) and input-gradient (C = A·W)."""
    from zeroq_b200.ops.nf4 import quantize_4bit

    E = _ext.ext()
    torch.manual_seed(21)
    w = torch.randn(rows, cols, device=cuda) * 0.05
    packed, st = quantize_4bit(w, 64, "nf4")
    K, N = (rows, cols) if w_is_kn else (cols, rows)
    if K % 128 or N % 64:
        pytest.skip("shape outside the in-kernel decode's tiling")
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = torch.randn(M, 64, device=cuda, dtype=torch.bfloat16)
        b2 = torch.randn(64, N, device=cuda, dtype=torch.bfloat16) if w_is_kn else \
            torch.randn(N, 64, device=cuda, dtype=torch.bfloat16)
    c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    E.gemm_nf4(a, packed, st.absmax, rows, cols, 64, 0, w_is_kn, c, a2, b2)
    wb = torch.empty(rows * cols, device=cuda, dtype=torch.bfloat16)
    E.nf4_to_bf16(packed, st.absmax, wb, rows, cols, 64, 0, False)
    ref = torch.empty_like(c)
    if w_is_kn:
        E.gemm_bf16_nn(a, wb.view(rows, cols), ref, a2, b2)
    elif extra:
        E.gemm_bf16_tn_extra(a, wb.view(rows, cols), ref, a2, b2)
    else:
        E.set_gemm_pair_mode(1)
        E.gemm_bf16_tn(a, wb.view(rows, cols), ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(c, ref)
    exact = a.float() @ (wb.view(rows, cols).float() if w_is_kn else wb.view(rows, cols).float().t())
    if extra:
        exact = exact + a2.float() @ (b2.float() if w_is_kn else b2.float().t())
    assert (c.float() - exact).abs().max().item() < 2e-2 * exact.abs().max().item() + 1e-2


@pytest.mark.parametrize("quant_type,blocksize", [("fp4", 64), ("nf4", 128), ("nf4", 256)])
def test_gemm_nf4_fp4_and_block_sizes(cuda, quant_type, blocksize):
    from zeroq_b200.ops.nf4 import QUANT_TYPE_ID, quantize_4bit

    E = _ext.ext()
    torch.manual_seed(22)
    rows, cols, M = 768, 1024, 512
    w = torch.randn(rows, cols, device=cuda) * 0.05
    packed, st = quantize_4bit(w, blocksize, quant_type)
    qt = QUANT_TYPE_ID[quant_type]
    wb = torch.empty(rows * cols, device=cuda, dtype=torch.bfloat16)
    E.nf4_to_bf16(packed, st.absmax, wb, rows, cols, blocksize, qt, False)
    for w_is_kn in (False, True):
        K, N = (rows, cols) if w_is_kn else (cols, rows)
        a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
        c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        E.gemm_nf4(a, packed, st.absmax, rows, cols, blocksize, qt, w_is_kn, c, None, None)
        ref = torch.empty_like(c)
        if w_is_kn:
            E.gemm_bf16_nn(a, wb.view(rows, cols), ref, None, None)
        else:
            E.set_gemm_pair_mode(1)
            E.gemm_bf16_tn(a, wb.view(rows, cols), ref)
        torch.cuda.synchronize()
        _status_ok(cuda)
        assert torch.equal(c, ref), (quant_type, blocksize, w_is_kn)



@pytest.mark.parametrize("B,S,Hq,Hk", [(2, 256, 4, 4), (1, 1024, 8, 2), (2, 512, 3, 1), (1, 2048, 2, 2),
                                       (2, 384, 4, 2)])
@pytest.mark.parametrize("causal", [True, False])
def test_attention_forward_tcgen05_vs_fp32(cuda, B, S, Hq, Hk, causal):
    """tcgen05 forward: output and row log-sum-exp against an fp32 reference (S a
    multiple of 256: the two-query-tile kernel; S = 384: the one-tile kernel)."""
    torch.manual_seed(31)
    D = 128
    q = torch.randn(B, S, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, device=cuda)
    scale = 1.0 / math.sqrt(D)
    _ext.ext().attn_fwd_tc(q, k, v, o, lse, causal, scale)
    # the same with K/V handed over head-major ([B, Hk, S, D])
    o2 = torch.empty_like(q)
    lse2 = torch.empty_like(lse)
    _ext.ext().attn_fwd_tc(q, k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous(), o2,
                           lse2, causal, scale, None, True)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    rep = Hq // Hk
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        mask = torch.ones(S, S, device=cuda, dtype=torch.bool).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    ref_lse = torch.logsumexp(s, dim=-1)
    ref_o = (torch.softmax(s, dim=-1) @ vf).transpose(1, 2)
    assert (o.float() - ref_o).abs().max().item() < 2e-2
    assert (lse - ref_lse).abs().max().item() < 1e-3



@pytest.mark.parametrize("B,S,Hq,Hk", [(2, 256, 4, 4), (1, 1024, 8, 2), (1, 512, 8, 2), (2, 384, 4, 1)])
@pytest.mark.parametrize("causal", [True, False])
def test_attention_backward_tcgen05_vs_fp32(cuda, B, S, Hq, Hk, causal):
    """tcgen05 backward (dQ kernel + dK/dV kernel) against fp32 autograd of the
    same attention, with the forward's lse; GQA groups of 1, 2 and 4."""
    from zeroq_b200.ops.attention import attention_reference

    torch.manual_seed(41)
    D = 128
    q = torch.randn(B, S, Hq, D, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(B, S, Hk, D, device=cuda, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, device=cuda)
    E = _ext.ext()
    E.attn_fwd_tc(q, k, v, o, lse, causal, scale)
    do = torch.randn_like(q)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    E.attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, causal, scale)
    torch.cuda.synchronize()
    _status_ok(cuda)
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    attention_reference(qr, kr, vr, causal=causal, scale=scale).backward(do.float())
    for got, ref in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        err = (got.float() - ref).abs().max().item()
        assert err < 3e-2 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("M,N,K", [(8192, 3072, 6144), (2048, 3072, 12288), (4096, 1536, 8192)])
@pytest.mark.parametrize("nn", [False, True])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_stream_k_tail(cuda, M, N, K, nn, extra):
    """Shapes whose last wave of 256x256 tiles is split along K over the idle
    clusters (partials in fp32, added by the last part): against fp32, twice in
    a row (the arrival counters reset themselves)."""
    torch.manual_seed(51)
    E = _ext.ext()
    E.set_gemm_pair_mode(1)
    a = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    b = torch.randn(K, N, device=cuda, dtype=torch.bfloat16) if nn else \
        torch.randn(N, K, device=cuda, dtype=torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = torch.randn(M, 64, device=cuda, dtype=torch.bfloat16)
        b2 = torch.randn(64, N, device=cuda, dtype=torch.bfloat16) if nn else \
            torch.randn(N, 64, device=cuda, dtype=torch.bfloat16)
    ref = a.float() @ (b.float() if nn else b.float().t())
    if extra:
        ref = ref + a2.float() @ (b2.float() if nn else b2.float().t())
    tol = 2e-2 * math.sqrt(K) + 1e-2 * ref.abs().max().item()
    for _ in range(2):
        c = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        if nn:
            E.gemm_bf16_nn(a, b, c, a2, b2)
        elif extra:
            E.gemm_bf16_tn_extra(a, b, c, a2, b2)
        else:
            E.gemm_bf16_tn(a, b, c)
        torch.cuda.synchronize()
        _status_ok(cuda)
        assert (c.float() - ref).abs().max().item() < tol


def _split_pieces(t: torch.Tensor, starts):
    """Copies of t[starts[q]:starts[q+1]] in separate allocations (one per emulated
    rank, each at a 16-byte-aligned base), plus their device addresses."""
    bounds = list(starts) + [t.numel()]
    pieces = [t[bounds[q]:bounds[q + 1]].clone() for q in range(len(starts))]
    # an empty piece still needs an address; the kernel never reads it
    ptrs = [p.data_ptr() if p.numel() else t.data_ptr() for p in pieces]
    return pieces, ptrs


@pytest.mark.parametrize("M,N,K,starts_frac", [
    (512, 384, 512, [0.0, 0.5]),                 # two even pieces
    (1024, 4096, 4096, [0.0, 0.25, 0.5, 0.75]),  # four ranks, several N tiles each
    (768, 1000, 1536, [0.0, 0.3, 0.31, 0.8]),    # uneven pieces, N and K not tile multiples
    (300, 520, 384, [0.0, 0.0, 0.6]),            # an empty piece, ragged M
    (2048, 3072, 12288, [0.0, 0.5]),             # stream-K tail active
])
@pytest.mark.parametrize("extra", [False, True])
def test_ag_gemm_one_kernel_matches_dequant_then_gemm(cuda, M, N, K, starts_frac, extra):
    """The gather + dequantise + GEMM kernel over per-rank pieces (emulated on one
    GPU as separate allocations) against the standalone dequantise and the same
    GEMM: the assembled operand is bit-identical, the product too (up to the
    stream-K reduction order), for every rank's tile rotation, launched twice in a
    row (the counters reset themselves)."""
    from zeroq_b200.parallel.peer import ag_gemm_pieces

    torch.manual_seed(3)
    W = torch.randn(N, K, device=cuda) * 0.02
    packed, st = quantize_4bit(W, 64, "nf4")
    packed, absmax = packed.reshape(-1), st.absmax.reshape(-1)
    # packed starts at odd byte offsets exercise the byte-wise path at boundaries
    pst = [int(f * packed.numel()) | (1 if 0 < f < 0.5 else 0) for f in starts_frac]
    pst[0] = 0
    ast = [int(f * absmax.numel()) for f in starts_frac]
    ppieces, pptrs = _split_pieces(packed, pst)
    apieces, aptrs = _split_pieces(absmax, ast)
    full = torch.empty(N * K, dtype=torch.bfloat16, device=cuda)
    _ext.ext().nf4_to_bf16(packed, absmax, full, N, K, 64, 0, False)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    ex = None
    ref = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    if extra:
        ex = ((torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16),
              (torch.randn(N, 64, device=cuda) * 0.1).to(torch.bfloat16))
        _ext.ext().gemm_bf16_tn_extra(x, full.view(N, K), ref, ex[0], ex[1])
    else:
        _ext.ext().gemm_bf16_tn(x, full.view(N, K), ref)
    streamk = K >= 128 * 48
    for rank in range(len(pst)):
        for _ in range(2):
            y, wbuf = ag_gemm_pieces(x, pptrs, pst, aptrs, ast, N, K, 64, "nf4", rank=rank,
                                     extra=ex)
            torch.cuda.synchronize()
            _status_ok(cuda)
            assert torch.equal(wbuf.reshape(-1), full)
            if streamk:
                torch.testing.assert_close(y.float(), ref.float(), rtol=1e-2, atol=1e-2)
            else:
                assert torch.equal(y, ref), (rank, (y.float() - ref.float()).abs().max().item())
    # sanity against fp32
    want = x.float() @ full.view(N, K).float().t()
    if extra:
        want += ex[0].float() @ ex[1].float().t()
    assert (y.float() - want).abs().max().item() < 2e-2 * want.abs().max().item() + 1e-2


def test_lora_pack_batch_matches_per_module_packs(cuda):
    """One lora_pack_many launch over several adapters writes exactly what the
    per-adapter lora_pack launches write (padding stays zero)."""
    from zeroq_b200.ops import lora as lora_k
    from zeroq_b200.ops.qlinear import LoraPackBatch, _pack_lora

    torch.manual_seed(23)
    jobs, refs, bufs = [], [], []
    for r, K, N, sc in [(16, 512, 1024, 2.0), (16, 1024, 512, 0.5), (8, 256, 768, 1.0)]:
        A = torch.randn(r, K, device=cuda)
        B = torch.randn(N, r, device=cuda)
        out = (torch.zeros(64, K, dtype=torch.bfloat16, device=cuda),
               torch.zeros(N, 64, dtype=torch.bfloat16, device=cuda),
               torch.zeros(lora_k.round16(r), N, dtype=torch.bfloat16, device=cuda))
        jobs.append((A, B, sc, out[0], out[1], out[2], lambda: None))
        bufs.append(out)
        refs.append(_pack_lora(A, B, sc))
    assert LoraPackBatch().run(jobs)
    torch.cuda.synchronize()
    for out, ref in zip(bufs, refs):
        for a, b in zip(out, ref):
            assert torch.equal(a, b)


def test_trainer_batch_pack_keeps_lora_operands_current(cuda):
    """After Trainer steps (each ending with one batched repack) every cached LoRA
    operand - the fused q/k/v blocks and each projection's own - equals a fresh
    pack of the adapter's current parameters."""
    import zeroq_b200 as zq
    from zeroq_b200.models import DecoderLM, get_config
    from zeroq_b200.ops.qkv import _lora_blocks
    from zeroq_b200.ops.qlinear import _pack_lora
    from zeroq_b200.train import Trainer, synthetic_batch

    cfg = get_config("4.7b", d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn_dim=1024,
                     vocab_size=1000, lora_r=16, lora_alpha=32.0)
    model = DecoderLM(cfg, device=cuda).init_dense_(seed=0)
    zq.initialize(model, zq.ZeroQConfig(compute_dtype=torch.bfloat16, compute_in_4bit=True,
                                        gather_once=True,
                                        exclude_modules=["lm_head", "embed_tokens"]),
                  trainable_patterns=("lora_", "norm"))
    with torch.no_grad():
        for n_, p in model.named_parameters():
            if "lora_B" in n_:
                p.normal_(0.0, 0.02)
    opt = zq.ShardedAdamW(model.trainable_parameters(), lr=1e-2)
    tr = Trainer(model, opt, cuda)
    x, y = synthetic_batch(2, 256, cfg.vocab_size, seed=0)
    for _ in range(3):
        tr.step(x, y)
    torch.cuda.synchronize()
    checked = 0
    for layer in model.layers:
        for _, m in layer.projections():
            if m._lora_ops is not None:
                assert m._lora_key == m._lora_state_key()     # marked current by the batch
                for a, b in zip(m._lora_ops, _pack_lora(m.lora_A.detach(), m.lora_B.detach(), m.scaling)):
                    assert torch.equal(a, b)
                checked += 1
        cache = layer._qkv_cache
        mods = (layer.q_proj, layer.k_proj, layer.v_proj)
        got = [t.clone() for t in _lora_blocks(mods, cache)[1:]]   # current key: no repack
        cache["key"] = None                                           # force a fresh pack
        fresh = _lora_blocks(mods, cache)[1:]
        for a, b in zip(got, fresh):
            assert torch.equal(a, b)
    assert checked > 0


def test_rope_into2_matches_two_rope_into(cuda):
    """The q and k gradients un-rotated by one launch equal two separate launches,
    into column slices of one fused gradient buffer."""
    from zeroq_b200.ops.rope import rope_table

    torch.manual_seed(22)
    B, S, Hq, Hk, D = 2, 256, 4, 2, 128
    dq = torch.randn(B, S, Hq, D, device=cuda).to(torch.bfloat16)
    dk = torch.randn(B, S, Hk, D, device=cuda).to(torch.bfloat16)
    cs = rope_table(S, D, 10000.0, cuda)
    Nt = (Hq + 2 * Hk) * D
    g1 = torch.zeros(B * S, Nt, dtype=torch.bfloat16, device=cuda)
    g2 = torch.zeros_like(g1)
    o1, o2 = Hq * D, (Hq + Hk) * D
    _ext.ext().rope_into2(dq, g1[:, :o1], dk, g1[:, o1:o2], cs, -1.0)
    _ext.ext().rope_into(dq, g2[:, :o1], cs, -1.0)
    _ext.ext().rope_into(dk, g2[:, o1:o2], cs, -1.0)
    torch.cuda.synchronize()
    assert torch.equal(g1, g2)
    assert float(g1[:, o2:].abs().sum()) == 0.0


def test_nf4_segments_decode_matches_per_weight_decodes(cuda):
    """Three 4-bit weights decoded into one buffer by one launch equal the three
    separate decodes, byte for byte (the fused q/k/v operand)."""
    torch.manual_seed(21)
    shapes = [(1024, 512), (256, 512), (256, 512)]
    qs = [quantize_4bit(torch.randn(n, k, device=cuda) * 0.02, 64, "nf4") for n, k in shapes]
    total = sum(n * k for n, k in shapes)
    out = torch.empty(total, dtype=torch.bfloat16, device=cuda)
    _ext.ext().nf4_to_bf16_segments([p.reshape(-1) for p, _ in qs], [st.absmax.reshape(-1) for _, st in qs],
                                    [n * k for n, k in shapes], out, 64, 0)
    ref, off = torch.empty_like(out), 0
    for (n, k), (p, st) in zip(shapes, qs):
        _ext.ext().nf4_to_bf16(p.reshape(-1), st.absmax.reshape(-1), ref[off:off + n * k], n, k, 64, 0, False)
        off += n * k
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_gather_dequant_fast_path_matches_full(cuda):
    """The warp-per-item peer gather + dequantise (standalone kernel) over uneven
    pieces equals the full dequantise, for a row window too."""
    N, K = 1000, 1536
    torch.manual_seed(4)
    packed, st = quantize_4bit(torch.randn(N, K, device=cuda) * 0.02, 64, "nf4")
    packed, absmax = packed.reshape(-1), st.absmax.reshape(-1)
    pst = [0, 100003, 400000]
    ast = [0, 3125, 12500]
    ppieces, pptrs = _split_pieces(packed, pst)
    apieces, aptrs = _split_pieces(absmax, ast)
    full = torch.empty(N * K, dtype=torch.bfloat16, device=cuda)
    _ext.ext().nf4_to_bf16(packed, absmax, full, N, K, 64, 0, False)
    for row0, rows in ((0, N), (136, 264)):
        out = torch.empty(rows * K, dtype=torch.bfloat16, device=cuda)
        _ext.ext().plan_gather_dequant(pptrs, pst, aptrs, ast, rows, K, row0, 64, 0, False, out)
        torch.cuda.synchronize()
        assert torch.equal(out, full[row0 * K:(row0 + rows) * K])


@pytest.mark.parametrize("M,K,N", [(512, 384, 1024), (300, 1536, 640), (2048, 3072, 12288)])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_gelu_epilogues_match_separate_kernels(cuda, M, K, N, extra):
    """GELU-output epilogue (H and gelu(H) from one GEMM) and GELU-gradient
    epilogue ((dY·W) * gelu'(H)) against the plain GEMM followed by the GELU
    kernels: bit-identical (the epilogues round the accumulator to bf16 first)."""
    E = _ext.ext()
    torch.manual_seed(5)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.05).to(torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = (torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16)
        b2 = (torch.randn(N, 64, device=cuda) * 0.1).to(torch.bfloat16)
    h = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    act = torch.empty_like(h)
    E.gemm_gelu(x, w, h, act, False, a2, b2)
    h_ref = torch.empty_like(h)
    if extra:
        E.gemm_bf16_tn_extra(x, w, h_ref, a2, b2)
    else:
        E.gemm_bf16_tn(x, w, h_ref)
    act_ref = torch.empty_like(h)
    E.gelu_fwd(h_ref, act_ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    streamk = K >= 128 * 48
    if streamk:
        torch.testing.assert_close(h.float(), h_ref.float(), rtol=1e-2, atol=1e-2)
    else:
        assert torch.equal(h, h_ref) and torch.equal(act, act_ref)
    # backward: dH = (dY [M, N] · W [N, K]... here the GEMM is dY [M, K'] x Wd [K', N])
    gy = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    wd = (torch.randn(K, N, device=cuda) * 0.05).to(torch.bfloat16)  # [K', N] read MN-major
    a3 = b3 = None
    if extra:
        a3 = (torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16)
        b3 = (torch.randn(64, N, device=cuda) * 0.1).to(torch.bfloat16)
    dh = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    E.gemm_gelu(gy, wd, dh, h_ref, True, a3, b3)
    da = torch.empty_like(dh)
    E.gemm_bf16_nn(gy, wd, da, a3, b3)
    dh_ref = torch.empty_like(dh)
    E.gelu_bwd(da, h_ref, dh_ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(dh, dh_ref), (dh.float() - dh_ref.float()).abs().max().item()


@pytest.mark.parametrize("lora_r", [0, 16])
def test_fused_gelu_mlp_matches_unfused(cuda, lora_r):
    """up_proj(x, act_out='gelu') + down_proj(f, pre=h) equals gelu between two
    plain NF4 layers, values and gradients (input and LoRA)."""
    from zeroq_b200.ops.activations import gelu
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(6)
    d, f = 512, 1536
    up = Linear4bit(d, f, lora_r=lora_r, device=cuda)
    down = Linear4bit(f, d, lora_r=lora_r, device=cuda)
    up.quantize_from(torch.randn(f, d, device=cuda) * 0.03)
    down.quantize_from(torch.randn(d, f, device=cuda) * 0.03)
    if lora_r:
        with torch.no_grad():
            up.lora_B.normal_(0, 0.02)
            down.lora_B.normal_(0, 0.02)
    x = (torch.randn(2, 200, d, device=cuda)).to(torch.bfloat16).requires_grad_(True)
    hpre, a = up(x, act_out="gelu")
    y = down(a, pre=hpre)
    (y.float() ** 2).sum().backward()
    grads = [x.grad.clone()] + ([up.lora_A.grad.clone(), up.lora_B.grad.clone(),
                                 down.lora_A.grad.clone(), down.lora_B.grad.clone()] if lora_r else [])
    for p in [x] + ([up.lora_A, up.lora_B, down.lora_A, down.lora_B] if lora_r else []):
        p.grad = None
    y2 = down(gelu(up(x)))
    (y2.float() ** 2).sum().backward()
    grads2 = [x.grad] + ([up.lora_A.grad, up.lora_B.grad, down.lora_A.grad, down.lora_B.grad]
                         if lora_r else [])
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(y, y2)
    assert torch.equal(grads[0], grads2[0])
    for g1, g2 in zip(grads[1:], grads2[1:]):  # LoRA grads: atomic fp32 sums, no fixed order
        torch.testing.assert_close(g1, g2, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("M,K,N", [(512, 384, 1024), (300, 1536, 640), (2048, 3584, 4736)])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_swiglu_epilogues_match_separate_kernels(cuda, M, K, N, extra):
    """SwiGLU-output epilogue (u and silu(g)·u from the up-projection GEMM) and
    SwiGLU-gradient epilogue (dg, du from the down-projection's input-gradient
    GEMM) against the plain GEMMs followed by the SwiGLU kernels (bit-identical:
    the epilogues round the accumulator to bf16 first) and against fp32 torch."""
    E = _ext.ext()
    torch.manual_seed(15)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.05).to(torch.bfloat16)
    g = (torch.randn(M, N, device=cuda) * 2).to(torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = (torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16)
        b2 = (torch.randn(N, 64, device=cuda) * 0.1).to(torch.bfloat16)
    u = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    act = torch.empty_like(u)
    E.gemm_swiglu(x, w, u, act, g, None, False, a2, b2)
    u_ref = torch.empty_like(u)
    if extra:
        E.gemm_bf16_tn_extra(x, w, u_ref, a2, b2)
    else:
        E.gemm_bf16_tn(x, w, u_ref)
    act_ref = torch.empty_like(u)
    E.swiglu_fwd(g, u_ref, act_ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(u, u_ref) and torch.equal(act, act_ref)
    want = torch.nn.functional.silu(g.float()) * u_ref.float()
    torch.testing.assert_close(act.float(), want, rtol=1e-2, atol=1e-2)
    # backward: D = dY [M, K'] · Wd [K', N]; dg = D·u·silu'(g), du = D·silu(g)
    gy = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    wd = (torch.randn(K, N, device=cuda) * 0.05).to(torch.bfloat16)
    a3 = b3 = None
    if extra:
        a3 = (torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16)
        b3 = (torch.randn(64, N, device=cuda) * 0.1).to(torch.bfloat16)
    dg = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    du = torch.empty_like(dg)
    E.gemm_swiglu(gy, wd, dg, du, g, u_ref, True, a3, b3)
    d = torch.empty_like(dg)
    E.gemm_bf16_nn(gy, wd, d, a3, b3)
    dg_ref, du_ref = torch.empty_like(dg), torch.empty_like(dg)
    E.swiglu_bwd(d, g, u_ref, dg_ref, du_ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(dg, dg_ref), (dg.float() - dg_ref.float()).abs().max().item()
    assert torch.equal(du, du_ref), (du.float() - du_ref.float()).abs().max().item()
    gf, uf, df = g.float(), u_ref.float(), d.float()
    sg = torch.sigmoid(gf)
    torch.testing.assert_close(du.float(), df * gf * sg, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(dg.float(), df * uf * sg * (1 + gf * (1 - sg)), rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("lora_r", [0, 16])
def test_fused_swiglu_mlp_matches_unfused(cuda, lora_r):
    """gate(x); up(x, act_out='swiglu', gate=g); down(f, pre=(g, u)) equals
    swiglu between plain NF4 layers, values and gradients (input and LoRA)."""
    from zeroq_b200.ops.activations import swiglu
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(16)
    d, f = 512, 1408
    gate = Linear4bit(d, f, lora_r=lora_r, device=cuda)
    up = Linear4bit(d, f, lora_r=lora_r, device=cuda)
    down = Linear4bit(f, d, lora_r=lora_r, device=cuda)
    for m, shape in ((gate, (f, d)), (up, (f, d)), (down, (d, f))):
        m.quantize_from(torch.randn(*shape, device=cuda) * 0.03)
        if lora_r:
            with torch.no_grad():
                m.lora_B.normal_(0, 0.02)
    mods = (gate, up, down)
    x = (torch.randn(2, 200, d, device=cuda)).to(torch.bfloat16).requires_grad_(True)
    g = gate(x)
    u, a = up(x, act_out="swiglu", gate=g)
    assert not a.requires_grad
    y = down(a, pre=(g, u))
    (y.float() ** 2).sum().backward()

    def take():
        out = [x.grad.clone()]
        for m in mods:
            if lora_r:
                out += [m.lora_A.grad.clone(), m.lora_B.grad.clone()]
                m.lora_A.grad = m.lora_B.grad = None
        x.grad = None
        return out

    grads = take()
    y2 = down(swiglu(gate(x), up(x)))
    (y2.float() ** 2).sum().backward()
    grads2 = take()
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(y, y2)
    torch.testing.assert_close(grads[0], grads2[0], rtol=1e-2, atol=1e-3)  # summed in another order
    for g1, g2 in zip(grads[1:], grads2[1:]):  # LoRA grads: atomic fp32 sums, no fixed order
        torch.testing.assert_close(g1, g2, rtol=1e-3, atol=1e-5)


def test_ag_gemm_swiglu_epilogue_matches_separate_kernels(cuda):
    """The gather-mode GEMM with the SwiGLU-output epilogue (u and silu(g)·u, the
    weight assembled from pieces inside the kernel) against the plain GEMM on the
    dequantised weight and the SwiGLU kernel, for every rank's tile rotation."""
    from zeroq_b200.parallel.peer import ag_gemm_pieces

    torch.manual_seed(17)
    M, N, K = 512, 1408, 512
    W = torch.randn(N, K, device=cuda) * 0.02
    packed, st = quantize_4bit(W, 64, "nf4")
    packed, absmax = packed.reshape(-1), st.absmax.reshape(-1)
    pst = [0, packed.numel() // 3 + 1, 2 * packed.numel() // 3]
    ast = [0, absmax.numel() // 3, 2 * absmax.numel() // 3]
    ppieces, pptrs = _split_pieces(packed, pst)
    apieces, aptrs = _split_pieces(absmax, ast)
    full = torch.empty(N * K, dtype=torch.bfloat16, device=cuda)
    _ext.ext().nf4_to_bf16(packed, absmax, full, N, K, 64, 0, False)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    g = (torch.randn(M, N, device=cuda) * 2).to(torch.bfloat16)
    ex = ((torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16),
          (torch.randn(N, 64, device=cuda) * 0.1).to(torch.bfloat16))
    u_ref = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    _ext.ext().gemm_bf16_tn_extra(x, full.view(N, K), u_ref, ex[0], ex[1])
    act_ref = torch.empty_like(u_ref)
    _ext.ext().swiglu_fwd(g, u_ref, act_ref)
    for rank in range(3):
        act = torch.empty_like(u_ref)
        u, _ = ag_gemm_pieces(x, pptrs, pst, aptrs, ast, N, K, 64, "nf4", rank=rank, extra=ex,
                              swiglu=(g, act))
        torch.cuda.synchronize()
        _status_ok(cuda)
        assert torch.equal(u, u_ref) and torch.equal(act, act_ref), rank


@pytest.mark.parametrize("M,N,K,starts_frac", [
    (512, 384, 512, [0.0, 0.5]),
    (768, 1000, 1536, [0.0, 0.3, 0.31, 0.8]),   # uneven pieces, odd element starts
    (300, 520, 384, [0.0, 0.0, 0.6]),           # an empty piece, ragged M
])
def test_ag_gemm_f32_master_pieces_match_cast_then_gemm(cuda, M, N, K, starts_frac):
    """Gather of fp32 master pieces + bf16 cast + GEMM in one kernel against the
    cast weight and the same GEMM (bit-identical), for every rank's rotation, with
    a zero-padded tail on the last piece."""
    from zeroq_b200.parallel.peer import ag_gemm_f32_pieces

    torch.manual_seed(8)
    W = torch.randn(N, K, device=cuda) * 0.05
    flat = torch.cat([W.reshape(-1), torch.zeros(37, device=cuda)])   # padded tail
    starts = [int(f * N * K) | (1 if 0 < f < 0.5 else 0) for f in starts_frac]
    starts[0] = 0
    pieces, ptrs = _split_pieces(flat, starts)
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    wb = W.to(torch.bfloat16)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    _ext.ext().gemm_bf16_tn(x, wb, ref)
    for rank in range(len(starts)):
        y, wbuf = ag_gemm_f32_pieces(x, ptrs, starts, flat.numel(), N, K, rank)
        torch.cuda.synchronize()
        _status_ok(cuda)
        assert torch.equal(wbuf, wb)
        assert torch.equal(y, ref)


@pytest.mark.parametrize("B,S,H,K", [(2, 512, 8, 1024), (1, 384, 3, 512), (4, 1024, 24, 3072)])
@pytest.mark.parametrize("extra", [False, True])
def test_gemm_rope_epilogue_matches_rope_kernel(cuda, B, S, H, K, extra):
    """RoPE applied in the GEMM epilogue equals the GEMM followed by the RoPE
    kernel, bit for bit (both rotate the bf16-rounded output in fp32)."""
    from zeroq_b200.ops.rope import rope_table

    E = _ext.ext()
    torch.manual_seed(9)
    M, N = B * S, H * 128
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda) * 0.05).to(torch.bfloat16)
    a2 = b2 = None
    if extra:
        a2 = (torch.randn(M, 64, device=cuda) * 0.1).to(torch.bfloat16)
        b2 = (torch.randn(N, 64, device=cuda) * 0.1).to(torch.bfloat16)
    cs = rope_table(S, 128, 10000.0, cuda)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    E.gemm_rope(x, w, y, cs, a2, b2)
    h = torch.empty_like(y)
    if extra:
        E.gemm_bf16_tn_extra(x, w, h, a2, b2)
    else:
        E.gemm_bf16_tn(x, w, h)
    ref = torch.empty_like(h)
    E.rope(h.view(B, S, H, 128), ref.view(B, S, H, 128), cs, 1.0)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(y, ref), (y.float() - ref.float()).abs().max().item()


@pytest.mark.parametrize("lora_r", [0, 16])
def test_linear4bit_rope_output_matches_apply_rope(cuda, lora_r):
    """q/k projections with the rotary embedding in the GEMM epilogue give the
    same values and gradients as the projection followed by apply_rope."""
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.ops.rope import apply_rope, rope_table

    torch.manual_seed(10)
    B, S, d, Hq, Hk = 2, 256, 512, 4, 2
    q_proj = Linear4bit(d, Hq * 128, lora_r=lora_r, device=cuda)
    k_proj = Linear4bit(d, Hk * 128, lora_r=lora_r, device=cuda)
    for m in (q_proj, k_proj):
        m.quantize_from(torch.randn(m.out_features, d, device=cuda) * 0.05)
        if lora_r:
            with torch.no_grad():
                m.lora_B.normal_(0, 0.02)
    x = torch.randn(B, S, d, device=cuda).to(torch.bfloat16).requires_grad_(True)
    cs = rope_table(S, 128, 10000.0, cuda)
    q = q_proj(x, rope=cs).view(B, S, Hq, 128)
    k = k_proj(x, rope=cs).view(B, S, Hk, 128)
    (q.float().square().sum() + (k.float() * 0.5).sum()).backward()
    gx = x.grad.clone()
    gA = q_proj.lora_A.grad.clone() if lora_r else None
    x.grad = None
    if lora_r:
        q_proj.lora_A.grad = None
        k_proj.lora_A.grad = None
        q_proj.lora_B.grad = None
        k_proj.lora_B.grad = None
    q2, k2 = apply_rope(q_proj(x).view(B, S, Hq, 128), k_proj(x).view(B, S, Hk, 128), 10000.0)
    (q2.float().square().sum() + (k2.float() * 0.5).sum()).backward()
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(q, q2) and torch.equal(k, k2)
    assert torch.equal(gx, x.grad)
    if lora_r:
        # the LoRA weight-gradient kernel adds fp32 partial sums over token ranges
        # with atomics, in no fixed order: two runs agree to fp32 rounding only
        torch.testing.assert_close(gA, q_proj.lora_A.grad, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,S,Hq,Hk", [(2, 256, 4, 4), (1, 512, 8, 2)])
def test_attention_backward_inverse_rope_epilogue(cuda, B, S, Hq, Hk):
    """dQ/dK written rotated back by the attention backward (rope table given)
    equal the plain backward followed by the inverse RoPE kernel, bit for bit."""
    from zeroq_b200.ops.rope import rope_table

    E = _ext.ext()
    torch.manual_seed(11)
    q = torch.randn(B, S, Hq, 128, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, S, Hk, 128, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, S, Hk, 128, device=cuda).to(torch.bfloat16)
    do = torch.randn(B, S, Hq, 128, device=cuda).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, device=cuda)
    scale = 128 ** -0.5
    E.attn_fwd_tc(q, k, v, o, lse, True, scale)
    cs = rope_table(S, 128, 10000.0, cuda)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    E.attn_bwd_tc(do, q, k, v, o, lse, dq, dk, dv, True, scale)
    dq_r, dk_r, dv_r = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    E.attn_bwd_tc(do, q, k, v, o, lse, dq_r, dk_r, dv_r, True, scale, None, cs)
    ref_q, ref_k = torch.empty_like(dq), torch.empty_like(dk)
    E.rope(dq, ref_q, cs, -1.0)
    E.rope(dk, ref_k, cs, -1.0)
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(dv_r, dv)
    assert torch.equal(dq_r, ref_q), (dq_r.float() - ref_q.float()).abs().max().item()
    assert torch.equal(dk_r, ref_k), (dk_r.float() - ref_k.float()).abs().max().item()


def test_rope_spec_projection_attention_chain_matches_apply_rope(cuda):
    """q/k projections rotating in their epilogue + attention rotating dQ/dK back
    (shared RopeSpec) against projections, apply_rope and plain attention."""
    from zeroq_b200.ops.attention import flash_attention
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.ops.rope import RopeSpec, apply_rope, rope_table

    torch.manual_seed(12)
    B, S, d, Hq, Hk = 2, 256, 512, 4, 2
    qp = Linear4bit(d, Hq * 128, lora_r=8, device=cuda)
    kp = Linear4bit(d, Hk * 128, lora_r=8, device=cuda)
    vp = Linear4bit(d, Hk * 128, device=cuda)
    for m in (qp, kp, vp):
        m.quantize_from(torch.randn(m.out_features, d, device=cuda) * 0.05)
    with torch.no_grad():
        qp.lora_B.normal_(0, 0.02)
        kp.lora_B.normal_(0, 0.02)
    x = torch.randn(B, S, d, device=cuda).to(torch.bfloat16).requires_grad_(True)
    spec = RopeSpec(rope_table(S, 128, 10000.0, cuda))
    o = flash_attention(qp(x, rope=spec).view(B, S, Hq, 128), kp(x, rope=spec).view(B, S, Hk, 128),
                        vp(x).view(B, S, Hk, 128), causal=True, rope=spec)
    o.float().square().sum().backward()
    assert spec.grads_unrotated
    g1, gA1 = x.grad.clone(), qp.lora_A.grad.clone()
    x.grad = None
    qp.lora_A.grad = None
    kp.lora_A.grad = None
    qp.lora_B.grad = None
    kp.lora_B.grad = None
    q2, k2 = apply_rope(qp(x).view(B, S, Hq, 128), kp(x).view(B, S, Hk, 128), 10000.0)
    o2 = flash_attention(q2, k2, vp(x).view(B, S, Hk, 128), causal=True)
    o2.float().square().sum().backward()
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert torch.equal(o, o2)
    assert torch.equal(g1, x.grad)
    torch.testing.assert_close(gA1, qp.lora_A.grad, rtol=1e-4, atol=1e-5)  # atomic fp32 sums


@pytest.mark.parametrize("lora_r", [0, 16])
def test_fused_qkv_projection_matches_separate_projections(cuda, lora_r):
    """One GEMM for q, k, v (RoPE on the q/k columns, three LoRA slabs) and its
    backward (one input-gradient GEMM over the concatenated gradient) against the
    three projections + apply_rope, through the attention."""
    from zeroq_b200.ops.attention import flash_attention
    from zeroq_b200.ops.qkv import qkv_fusable, qkv_projection
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.ops.rope import apply_rope, rope_table

    torch.manual_seed(13)
    B, S, d, Hq, Hk = 2, 256, 512, 4, 2
    mods = [Linear4bit(d, h * 128, lora_r=lora_r, device=cuda) for h in (Hq, Hk, Hk)]
    for m in mods:
        m.quantize_from(torch.randn(m.out_features, d, device=cuda) * 0.05)
        if lora_r:
            with torch.no_grad():
                m.lora_B.normal_(0, 0.05)
    x = torch.randn(B, S, d, device=cuda).to(torch.bfloat16).requires_grad_(True)
    cs = rope_table(S, 128, 10000.0, cuda)
    assert qkv_fusable(mods, x, S)
    go = torch.randn(B, S, Hq, 128, device=cuda).to(torch.bfloat16)
    results = []
    cache = {}
    for fused in (True, False, True):   # fused twice: the LoRA block cache is reused
        x.grad = None
        for m in mods:
            if lora_r:
                m.lora_A.grad = None
                m.lora_B.grad = None
        if fused:
            q, k, v = qkv_projection(x, mods, cs, cache)
        else:
            q, k = apply_rope(mods[0](x).view(B, S, Hq, 128), mods[1](x).view(B, S, Hk, 128), 10000.0)
            v = mods[2](x).view(B, S, Hk, 128)
        o = flash_attention(q, k, v, causal=True)
        o.backward(go)
        results.append([o.detach().clone(), x.grad.clone()] +
                       ([g for m in mods for g in (m.lora_A.grad.clone(), m.lora_B.grad.clone())]
                        if lora_r else []))
    torch.cuda.synchronize()
    _status_ok(cuda)
    for a, b in zip(results[0], results[1]):
        scale = b.float().abs().max().item() + 1e-6
        assert (a.float() - b.float()).abs().max().item() <= 2e-2 * scale, (a.shape,)
    for i, (a, b) in enumerate(zip(results[0], results[2])):
        if i < 2:
            assert torch.equal(a, b)
        else:  # LoRA grads: atomic fp32 sums over token ranges, no fixed order
            torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)
    if lora_r:
        # an in-place update of the adapters (what an optimizer step does) must
        # repack the cached q/k/v blocks
        with torch.no_grad():
            for m in mods:
                m.lora_A.mul_(1.5)
                m.lora_B.add_(0.01)
        outs = []
        for fused in (True, False):
            if fused:
                q, k, v = qkv_projection(x, mods, cs, cache)
            else:
                q, k = apply_rope(mods[0](x).view(B, S, Hq, 128), mods[1](x).view(B, S, Hk, 128),
                                  10000.0)
                v = mods[2](x).view(B, S, Hk, 128)
            outs.append(flash_attention(q, k, v, causal=True).detach().float())
        torch.cuda.synchronize()
        scale = outs[1].abs().max().item() + 1e-6
        assert (outs[0] - outs[1]).abs().max().item() <= 2e-2 * scale
        assert (outs[0] - results[0][0].float()).abs().max().item() > 1e-3 * scale  # it changed


@pytest.mark.parametrize("E", [128, 192, 256])
@pytest.mark.parametrize("nn", [False, True])
def test_gemm_wide_extra_slab_matches_concatenated_k(cuda, E, nn):
    """An extra K slab of 2-4 x 64 columns (one pipeline stage each) equals the
    GEMM over the concatenated K dimension."""
    Ex = _ext.ext()
    torch.manual_seed(14)
    M, N, K = 512, 768, 1024
    x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
    a2 = (torch.randn(M, E, device=cuda) * 0.1).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    ref = torch.empty_like(y)
    if nn:
        w = (torch.randn(K, N, device=cuda) * 0.05).to(torch.bfloat16)
        b2 = (torch.randn(E, N, device=cuda) * 0.1).to(torch.bfloat16)
        Ex.gemm_bf16_nn(x, w, y, a2, b2)
        Ex.gemm_bf16_nn(torch.cat([x, a2], 1), torch.cat([w, b2], 0), ref, None, None)
    else:
        w = (torch.randn(N, K, device=cuda) * 0.05).to(torch.bfloat16)
        b2 = (torch.randn(N, E, device=cuda) * 0.1).to(torch.bfloat16)
        Ex.gemm_bf16_tn_extra(x, w, y, a2, b2)
        Ex.gemm_bf16_tn(torch.cat([x, a2], 1), torch.cat([w, b2], 1), ref)
    torch.cuda.synchronize()
    _status_ok(cuda)
    torch.testing.assert_close(y.float(), ref.float(), rtol=1e-2, atol=1e-2)


def test_cuda_graph_training_steps_match_eager(cuda):
    """Trainer steps replayed from one captured CUDA graph (device-side optimizer
    clock) track the same steps run eagerly.  Eager steps are not bitwise
    reproducible (floating-point atomics, and Adam's first updates are close to
    sign(grad), which amplifies last-bit differences), so the graph run must stay
    within a few times the spread between two eager runs."""
    from zeroq_b200 import ShardedAdamW, ZeroQConfig, initialize
    from zeroq_b200.models import DecoderLM, get_config
    from zeroq_b200.train import Trainer

    def run(graph: bool):
        cfg = get_config("4.7b", n_layers=2, lora_r=8, lora_alpha=16.0)
        model = DecoderLM(cfg, device=cuda)
        model.init_dense_(std=0.02, seed=7)
        zq = ZeroQConfig(compute_dtype=torch.bfloat16, compute_in_4bit=True, gather_once=True,
                         exclude_modules=["lm_head", "embed_tokens"], backend="auto")
        initialize(model, zq, trainable_patterns=("lora_", "norm"))
        opt = ShardedAdamW(model.trainable_parameters(), lr=1e-3)
        tr = Trainer(model, opt, cuda)
        g = torch.Generator().manual_seed(3)
        x = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).to(cuda)
        y = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).to(cuda)
        losses = [float(tr.step_device(x, y))]
        if graph:
            tr.enable_cuda_graph()
        for _ in range(5):
            losses.append(float(tr.step_device(x, y)))
        torch.cuda.synchronize()
        assert (tr._graph is not None) == graph
        assert opt.state_dict()["step"] == 6   # the device clock advanced on every replay
        return torch.tensor(losses), torch.cat([p.detach().float().reshape(-1) for p in opt.params])

    la, pa = run(False)
    lb, pb = run(False)
    lg, pg = run(True)
    _status_ok(cuda)
    assert lg[-1] < lg[0] - 1.0 and la[-1] < la[0] - 1.0
    spread_l = (lb - la).abs().max().item()
    spread_p = (pb - pa).abs().max().item()
    assert (lg - la).abs().max().item() <= 3 * spread_l + 2e-3, (lg, la, lb)
    assert (pg - pa).abs().max().item() <= 3 * spread_p + 1e-4


@pytest.mark.parametrize("vocab,chunk", [(1000, 256), (50257, 16384), (2048, 2048)])
def test_chunked_lm_head_cross_entropy_matches_full_logits(cuda, vocab, chunk):
    """LM head + CE over vocabulary chunks (no [M, V] logits) against the full
    logits path and an fp32 reference, with ignored rows."""
    from zeroq_b200.ops.cross_entropy import cross_entropy, lm_head_cross_entropy
    from zeroq_b200.ops.gemm import LMHeadFunction

    torch.manual_seed(21)
    M, d = 512, 256
    Vp = (vocab + 127) // 128 * 128
    W = (0.05 * torch.randn(Vp, d, device=cuda)).bfloat16()
    W[vocab:] = 0
    h = torch.randn(M, d, device=cuda).bfloat16()
    t = torch.randint(0, vocab, (M,), device=cuda)
    t[::7] = -100
    h1 = h.clone().requires_grad_(True)
    l1 = lm_head_cross_entropy(h1, W, t, vocab, chunk=chunk)
    l1.backward()
    h2 = h.clone().requires_grad_(True)
    l2 = cross_entropy(LMHeadFunction.apply(h2, W), t, vocab=vocab)
    l2.backward()
    h3 = h.float().clone().requires_grad_(True)
    l3 = torch.nn.functional.cross_entropy(h3 @ W.float()[:vocab].t(), t, ignore_index=-100)
    l3.backward()
    torch.cuda.synchronize()
    _status_ok(cuda)
    assert abs(l1.item() - l2.item()) < 2e-3 and abs(l1.item() - l3.item()) < 2e-2
    scale = h3.grad.abs().max().item()
    assert (h1.grad.float() - h2.grad.float()).abs().max().item() < 3e-2 * scale
    assert (h1.grad.float() - h3.grad).abs().max().item() < 3e-2 * scale

"""LoRA rank-space products (``zeroq_b200.ops.lora``): the tcgen05 kernels of
``csrc/lora_sm100.cu`` against fp32 PyTorch, and the CPU oracle path."""

import pytest
import torch

from zeroq_b200.ops import lora as L


def _ref_down(p, w):
    return p.float() @ w.float().t()


def test_cpu_down_and_wgrad_oracle():
    torch.manual_seed(0)
    T, K, nq = 70, 128, 16
    p = torch.randn(T, K).bfloat16()
    w = torch.randn(nq, K).bfloat16()
    u, ut = L.down(p, w, upad=64)
    assert u.shape == (T, 64) and torch.all(u[:, nq:] == 0)
    assert torch.equal(ut, u[:, :nq].t())
    out = torch.zeros(8, K)
    L.wgrad(p, ut, nq, [(0, K, 0, 0.5)], [out], 16, 8, True)
    ref = 0.5 * (ut[:8].float() @ p.float())
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("T,K,nq,upad", [(8192, 3072, 16, 64), (1000, 3072, 48, 64),
                                         (333, 12288, 16, 64), (640, 192, 64, 64),
                                         (300, 1024, 192, 192), (129, 9216, 48, 64)])
def test_lora_down_vs_fp32(cuda, T, K, nq, upad):
    torch.manual_seed(1)
    p = torch.randn(T, K, device=cuda).bfloat16()
    w = (0.05 * torch.randn(nq, K, device=cuda)).bfloat16()
    u, ut = L.down(p, w, upad=upad)
    torch.cuda.synchronize()
    from zeroq_b200.ops import _ext

    assert list(_ext.ext().gemm_status(cuda.index or 0)) == [0, 0]
    ref = _ref_down(p, w)
    err = (u[:, :nq].float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err
    assert torch.all(u[:, nq:] == 0)
    assert torch.equal(ut[:, :T], u[:, :nq].t())


@pytest.mark.gpu
def test_lora_down_strided_rows_and_second_call(cuda):
    """W given as the first rows of a wider padded buffer; P as a column slice."""
    torch.manual_seed(2)
    big = torch.randn(512, 4096 + 64, device=cuda).bfloat16()
    p = big[:, 64:]
    a_pad = torch.zeros(64, 4096, device=cuda, dtype=torch.bfloat16)
    a_pad[:16] = (0.1 * torch.randn(16, 4096, device=cuda)).bfloat16()
    for _ in range(2):
        u, ut = L.down(p, a_pad[:16])
        ref = _ref_down(p, a_pad[:16])
        assert (u[:, :16].float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("T,I,r,transposed", [(8192, 3072, 16, True), (8192, 12288, 16, False),
                                              (1000, 448, 8, True), (777, 3072, 16, False),
                                              (4096, 1024, 64, True)])
def test_lora_wgrad_vs_fp32(cuda, T, I, r, transposed):
    torch.manual_seed(3)
    r16 = L.round16(r)
    p = torch.randn(T, I, device=cuda).bfloat16()
    qt = torch.zeros(r16, (T + 7) // 8 * 8, device=cuda, dtype=torch.bfloat16)
    qt[:, :T] = torch.randn(r16, T, device=cuda).bfloat16()
    base = torch.randn(r, I, device=cuda) if transposed else torch.randn(I, r, device=cuda)
    out = base.clone()
    L.wgrad(p, qt, r16, [(0, I, 0, 0.25)], [out], r16, r, transposed)
    torch.cuda.synchronize()
    prod = 0.25 * (qt[:r, :T].float() @ p.float())      # [r, I]
    ref = base + (prod if transposed else prod.t())
    err = (out - ref).abs().max().item()
    assert err <= 1e-4 * prod.abs().max().item() + 1e-4, err


@pytest.mark.gpu
def test_lora_wgrad_jobs_and_groups_qkv_layout(cuda):
    """The fused q/k/v layouts: three dA in one pass (groups of 16 rank columns)
    and three dB as three jobs over column slices of dY."""
    torch.manual_seed(4)
    T, d, N, r = 2048, 1024, 512, 16
    x = torch.randn(T, d, device=cuda).bfloat16()
    g = torch.randn(T, 3 * N, device=cuda).bfloat16()
    vt = torch.randn(48, T, device=cuda).bfloat16()
    ut = torch.randn(48, T, device=cuda).bfloat16()
    dA = [torch.zeros(r, d, device=cuda) for _ in range(3)]
    L.wgrad(x, vt, 48, [(0, d, 0, 2.0)], dA, 16, r, True)
    dB = [torch.zeros(N, r, device=cuda) for _ in range(3)]
    L.wgrad(g, ut, 16, [(i * N, N, 16 * i, 1.0) for i in range(3)], dB, 16, r, False)
    torch.cuda.synchronize()
    for i in range(3):
        refA = 2.0 * vt[16 * i:16 * i + r].float() @ x.float()
        refB = g[:, i * N:(i + 1) * N].float().t() @ ut[16 * i:16 * i + r].float().t()
        assert (dA[i] - refA).abs().max().item() <= 1e-4 * refA.abs().max().item()
        assert (dB[i] - refB).abs().max().item() <= 1e-4 * refB.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("T,N,r,segs", [(8192, 3072, 16, 1), (1000, 6144, 16, 1),
                                        (2048, 3 * 1024, 16, 3), (777, 1536, 8, 1)])
def test_lora_vdb_matches_down_and_wgrad(cuda, T, N, r, segs):
    """One pass over dY: V and Vt as lora_down, dB as lora_wgrad (per segment)."""
    torch.manual_seed(5)
    g = torch.randn(T, N, device=cuda).bfloat16()
    nqv = 16 * segs
    bt = (0.05 * torch.randn(nqv, N, device=cuda)).bfloat16()
    ut = torch.zeros(nqv, (T + 7) // 8 * 8, device=cuda, dtype=torch.bfloat16)
    ut[:, :T] = torch.randn(nqv, T, device=cuda).bfloat16()
    w = N // segs
    sg = [(i * w, w, 16 * i) for i in range(segs)]
    outs = [torch.randn(w, r, device=cuda) for _ in range(segs)]
    base = [o.clone() for o in outs]
    res = L.vdb(g, bt, ut, 64, sg, outs, 16, r)
    assert res is not None
    # wider outputs (TMEM would need 8 CTAs per cluster) are declined, untouched
    wide = torch.zeros(12288, r, device=cuda)
    g2 = torch.zeros(64, 12288, device=cuda, dtype=torch.bfloat16)
    assert L.vdb(g2, torch.zeros(16, 12288, device=cuda, dtype=torch.bfloat16), ut[:, :64],
                 64, [(0, 12288, 0)], [wide], 16, r) is None
    assert torch.all(wide == 0)
    v, vt = res
    torch.cuda.synchronize()
    ref_v = g.float() @ bt.float().t()
    assert (v[:, :nqv].float() - ref_v).abs().max().item() <= 1e-2 * ref_v.abs().max().item() + 1e-3
    assert torch.all(v[:, nqv:] == 0) and torch.equal(vt[:, :T], v[:, :nqv].t())
    for i, (n0, n, q0) in enumerate(sg):
        ref = base[i] + g[:, n0:n0 + n].float().t() @ ut[q0:q0 + r, :T].float().t()
        err = (outs[i] - ref).abs().max().item()
        assert err <= 1e-4 * (ref - base[i]).abs().max().item() + 1e-4, (i, err)


@pytest.mark.gpu
@pytest.mark.parametrize("G,D", [(296, 3072), (7, 1000), (128, 8192)])
def test_colsum_accum_vs_torch(cuda, G, D):
    from zeroq_b200.ops import _ext

    part = torch.randn(G, D, device=cuda)
    out = torch.randn(D, device=cuda)
    ref = out + part.sum(0)
    _ext.ext().colsum_accum(part, out)
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-4)

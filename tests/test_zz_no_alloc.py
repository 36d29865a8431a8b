"""The allocation-free RMSNorm backward entry point, called through its exported C
symbol, against the regular entry point (which allocates its scratch through
PyTorch) and against a plain fp32 PyTorch backward.  Callers of the C symbol are
code that cannot allocate device memory itself, e.g. a runtime that owns the
whole device memory or must not trigger cudaMalloc's implicit synchronisation;
the symbol uses a static 4 MiB device array as scratch instead.  This file is
collected last on purpose."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    from zeroq_b200.ops import _ext

    _ext.ext()
    lib = ctypes.CDLL(_ext.so_path())
    fn = lib.zq_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    err = lib.zq_noalloc_error_string
    err.restype = ctypes.c_char_p
    return fn, err


def _regular(gy, x, w, rstd, gh):
    """The regular CUDA entry point (partial rows allocated by PyTorch)."""
    from zeroq_b200.ops import _ext

    dx = torch.empty_like(x)
    part = torch.empty(min(x.shape[0], 296), x.shape[1], dtype=torch.float32, device=x.device)
    _ext.ext().rmsnorm_bwd(gy, x, w, rstd, gh, dx, part)
    return dx, part.sum(0)


def _fp32_oracle(gy, x, w, rstd, gh):
    """RMSNorm backward in fp32 PyTorch: y = x * rstd * w."""
    xf, gf = x.float(), gy.float()
    xhat = xf * rstd[:, None]
    gxhat = gf * w
    dx = rstd[:, None] * (gxhat - xhat * (gxhat * xhat).mean(-1, keepdim=True))
    if gh is not None:
        dx = dx + gh.float()
    return dx, (gf * xhat).sum(0)


def _call(fn, err, gy, x, w, rstd, gh):
    M, D = x.shape
    dx = torch.empty_like(x)
    dw = torch.full((D,), float("nan"), device=x.device)
    rc = fn(gy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(),
            None if gh is None else gh.data_ptr(), dx.data_ptr(), dw.data_ptr(), M, D,
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, err()
    return dx, dw


# (M, D, with residual gradient): D = 1000 and 2056 are not multiples of the
# 128-lane team; D = 8192 caps the grid at 128 partial rows (4 MiB / (4 B * D)),
# below the 2 * SMs the regular entry point uses
CASES = [(1000, 3072, True), (777, 1024, True), (513, 1000, False), (77, 2056, True),
         (4099, 8192, False), (300, 8192, True)]


@pytest.mark.parametrize("M,D,with_gh", CASES)
def test_noalloc_matches_regular_entry_point_and_fp32_twice(cuda, M, D, with_gh):
    fn, err = _symbol()
    for call in range(2):  # the second call finds the scratch holding the first one's rows
        torch.manual_seed(1000 * call + D)
        x = torch.randn(M, D, device=cuda, dtype=torch.bfloat16)
        gy = torch.randn(M, D, device=cuda, dtype=torch.bfloat16)
        gh = torch.randn(M, D, device=cuda, dtype=torch.bfloat16) if with_gh else None
        w = 1 + 0.1 * torch.randn(D, device=cuda)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6)
        dx_reg, dw_reg = _regular(gy, x, w, rstd, gh)
        dx, dw = _call(fn, err, gy, x, w, rstd, gh)
        assert torch.equal(dx, dx_reg)
        assert torch.allclose(dw, dw_reg, rtol=1e-4, atol=1e-3)
        dx_ref, dw_ref = _fp32_oracle(gy, x, w, rstd, gh)
        assert (dx.float() - dx_ref).abs().max().item() < 5e-2
        assert ((dw - dw_ref).abs().max() / dw_ref.abs().max()).item() < 1e-3


def test_noalloc_rejects_oversized_problem(cuda):
    fn, err = _symbol()
    x = torch.zeros(4, 16, device=cuda, dtype=torch.bfloat16)
    w = torch.ones(16, device=cuda)
    rc = fn(x.data_ptr(), x.data_ptr(), w.data_ptr(), w.data_ptr(), None, x.data_ptr(),
            w.data_ptr(), 4, 8200, torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"8192" in err()

"""The allocation-free RMSNorm backward entry point, called through its exported C
symbol, against the regular entry point (which allocates its scratch through
PyTorch).  Callers of the C symbol are code that cannot allocate device memory
itself, e.g. a runtime that owns the whole device memory or must not trigger
cudaMalloc's implicit synchronisation; the symbol uses a static 4 MiB device array
as scratch instead.  This file is collected last on purpose."""

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


def _reference(gy, x, w, rstd, gh):
    from zeroq_b200.ops import _ext

    dx = torch.empty_like(x)
    part = torch.empty(min(x.shape[0], 296), x.shape[1], dtype=torch.float32, device=x.device)
    _ext.ext().rmsnorm_bwd(gy, x, w, rstd, gh, dx, part)
    return dx, part.sum(0)


def test_noalloc_matches_regular_entry_point_twice(cuda):
    fn, err = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (M, D) in enumerate([(1000, 3072), (777, 1024)]):
        torch.manual_seed(call)
        x = torch.randn(M, D, device=cuda, dtype=torch.bfloat16)
        gy = torch.randn(M, D, device=cuda, dtype=torch.bfloat16)
        gh = torch.randn(M, D, device=cuda, dtype=torch.bfloat16)
        w = 1 + 0.1 * torch.randn(D, device=cuda)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6)
        dx_ref, dw_ref = _reference(gy, x, w, rstd, gh)
        dx = torch.empty_like(x)
        dw = torch.full((D,), float("nan"), device=cuda)
        rc = fn(gy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), gh.data_ptr(),
                dx.data_ptr(), dw.data_ptr(), M, D, stream)
        torch.cuda.synchronize()
        assert rc == 0, err()
        assert torch.equal(dx, dx_ref)
        assert torch.allclose(dw, dw_ref, rtol=1e-4, atol=1e-3)


def test_noalloc_rejects_oversized_problem(cuda):
    fn, err = _symbol()
    x = torch.zeros(4, 16, device=cuda, dtype=torch.bfloat16)
    w = torch.ones(16, device=cuda)
    rc = fn(x.data_ptr(), x.data_ptr(), w.data_ptr(), w.data_ptr(), None, x.data_ptr(),
            w.data_ptr(), 4, 8200, torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"8192" in err()

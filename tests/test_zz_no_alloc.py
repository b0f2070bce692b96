"""The allocation-free RMSNorm backward (C symbol ``bb_rmsnorm_bwd_noalloc``) against the regular one.

The entry point exists for callers that cannot allocate device memory while the op runs (a host
runtime that owns every allocation, or a loop that must not allocate after start-up); its reduction
scratch is a static device array.  This file is collected last on purpose: if it fails, a run that
stops at the first failure has already run every other test.
"""

import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import bridge_b200

    here = os.path.dirname(bridge_b200.__file__)
    (so,) = glob.glob(os.path.join(here, "_C*.so"))
    lib = ctypes.CDLL(so)
    fn = lib.bb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_long, ctypes.c_int, ctypes.c_void_p]
    lib.bb_noalloc_last_error.restype = ctypes.c_char_p
    return lib, fn


def _case(rows, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).bfloat16()
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    return dy, x, w, rstd


def _call(fn, dy, x, w, rstd):
    dx = torch.empty_like(x)
    dw = torch.empty(x.shape[1], device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
            x.shape[0], x.shape[1], stream)
    return rc, dx, dw


def _fp32_reference(dy, x, w, rstd):
    """RMSNorm backward in plain FP32 PyTorch (autograd through y = x * rstd(x) * w)."""
    xf = x.float().requires_grad_()
    wf = w.float().requires_grad_()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    (xf * r * wf).backward(dy.float())
    return xf.grad, wf.grad


def _check(dx, dw, ref_dx, ref_dw):
    assert (dx.float() - ref_dx).abs().max().item() <= 2e-2 + 1e-2 * ref_dx.abs().max().item()
    assert (dw - ref_dw).abs().max().item() <= 1e-3 + 1e-3 * ref_dw.abs().max().item()


def test_noalloc_matches_regular_entry_point_twice():
    """Two calls in a row (different shapes) against the regular CUDA entry point and FP32 PyTorch."""
    from bridge_b200 import _C

    lib, fn = _lib()
    for rows, H, seed in ((300, 2560, 1), (57, 4096, 2)):
        dy, x, w, rstd = _case(rows, H, seed)
        rc, dx, dw = _call(fn, dy, x, w, rstd)
        assert rc == 0, lib.bb_noalloc_last_error()
        reg_dx, reg_dw = _C.rmsnorm_bwd(dy, x, w, rstd)
        torch.cuda.synchronize()
        assert (dx.float() - reg_dx.float()).abs().max().item() <= 3e-2 + 2e-2 * reg_dx.float().abs().max().item()
        assert (dw - reg_dw.float()).abs().max().item() <= 1e-2 + 1e-2 * reg_dw.float().abs().max().item()
        _check(dx, dw, *_fp32_reference(dy, x, w, rstd))


@pytest.mark.parametrize("rows,H", [(2048, 32768), (1000, 16384)])
def test_noalloc_wide_rows(rows, H):
    """H = 32768 caps the grid at 32 blocks (the scratch holds 32 partial rows) and needs 128 KB of
    shared memory; H = 16384 also needs the shared-memory attribute (64 KB)."""
    lib, fn = _lib()
    dy, x, w, rstd = _case(rows, H, 3)
    rc, dx, dw = _call(fn, dy, x, w, rstd)
    assert rc == 0, lib.bb_noalloc_last_error()
    torch.cuda.synchronize()
    _check(dx, dw, *_fp32_reference(dy, x, w, rstd))


def test_noalloc_rejects_bad_hidden_and_handles_empty():
    lib, fn = _lib()
    x = torch.zeros(2, 8, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    for bad_h in (40000, 4100, 4):
        rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, bad_h, s)
        assert rc != 0
        assert b"H must be" in lib.bb_noalloc_last_error()
    dw = torch.full((64,), float("nan"), device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), dw.data_ptr(), 0, 64, s)
    assert rc == 0, lib.bb_noalloc_last_error()
    torch.cuda.synchronize()
    assert bool((dw == 0).all())

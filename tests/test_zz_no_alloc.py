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


def test_noalloc_matches_regular_entry_point_twice():
    from bridge_b200 import _C

    lib, fn = _lib()
    for rows, H, seed in ((300, 2560, 1), (57, 4096, 2)):   # two calls in a row, different shapes
        dy, x, w, rstd = _case(rows, H, seed)
        rc, dx, dw = _call(fn, dy, x, w, rstd)
        assert rc == 0, lib.bb_noalloc_last_error()
        ref_dx, ref_dw = _C.rmsnorm_bwd(dy, x, w, rstd)
        torch.cuda.synchronize()
        assert (dx.float() - ref_dx.float()).abs().max().item() <= 3e-2 + 2e-2 * ref_dx.float().abs().max().item()
        assert (dw - ref_dw).abs().max().item() <= 1e-1 + 2e-2 * ref_dw.abs().max().item()


def test_noalloc_rejects_oversized_hidden():
    lib, fn = _lib()
    x = torch.zeros(2, 8, device="cuda", dtype=torch.bfloat16)
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 2, 40000,
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"H must be" in lib.bb_noalloc_last_error()

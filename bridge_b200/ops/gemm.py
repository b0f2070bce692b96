"""Linear layers on the tcgen05 GEMM: ``y = x @ W^T`` (bf16, FP32 accumulate).

All three GEMMs of a linear layer run in the persistent tcgen05 kernel of
``csrc/gemm_sm100.cu`` without transpose copies: forward ``x W^T`` (both
operands K-major), data gradient ``dy W`` (W consumed MN-major) and weight
gradient ``dy^T x`` (both consumed MN-major).  When a parameter carries an FP32
``main_grad`` buffer the weight gradient is accumulated straight into it by the
GEMM epilogue (read-add-write), so no bf16 weight gradient is materialised and
no separate accumulation pass runs.

``BRIDGE_B200_GEMM=cublas`` selects ``torch.matmul`` (the library baseline).
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import Tensor

from ._ext import ext, on_gpu


def _native() -> bool:
    if os.environ.get("BRIDGE_B200_GEMM", "tcgen05") != "tcgen05":
        return False
    m = ext()
    return m is not None and hasattr(m, "gemm")


def _aligned(*ts: Tensor) -> bool:
    return all(t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(-1) == 1 and t.stride(0) % 8 == 0
               and t.data_ptr() % 16 == 0 for t in ts)


def gemm(a: Tensor, b: Tensor, *, a_mn: bool = False, b_mn: bool = False, out: Tensor | None = None,
         accumulate: bool = False) -> Tensor:
    """``op(a) @ op(b)^T`` with ``op(a)=[M,K]`` (``a`` is ``[K,M]`` when ``a_mn``) and ``op(b)=[N,K]``."""
    if on_gpu(a) and _native() and _aligned(a, b):
        return ext().gemm(a, b, a_mn, b_mn, out, accumulate)
    A = a.t() if a_mn else a
    B = b if b_mn else b.t()
    r = torch.matmul(A, B)
    if out is None:
        return r
    if accumulate:
        out.add_(r.to(out.dtype))
    else:
        out.copy_(r)
    return out


def mm_nt(a: Tensor, b: Tensor, out: Tensor | None = None, *, accumulate: bool = False) -> Tensor:
    return gemm(a, b, out=out, accumulate=accumulate)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = gemm(x2, w)
        ctx.save_for_backward(x2, w)
        ctx.shape = shape
        return y.view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, w, b_mn=True).view(ctx.shape)                 # dy [T,out] @ W [out,in]
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                gemm(dy2, x2, a_mn=True, b_mn=True, out=main, accumulate=True)   # main += dy^T x
            else:
                dw = gemm(dy2, x2, a_mn=True, b_mn=True)
        return dx, dw


def linear(x: Tensor, weight: Tensor) -> Tensor:
    if on_gpu(x) and _native() and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16:
        return _LinearFn.apply(x, weight)
    return F.linear(x, weight)

"""Linear layers: ``y = x @ W^T`` for bf16 activations and weights.

On CUDA the forward (``x @ W^T``), data-gradient (``dy @ W``) and
weight-gradient (``dy^T @ x``) GEMMs are the tcgen05/TMEM kernel of
``csrc/gemm_sm100.cu`` (TMA-fed, warp-specialised, FP32 accumulation in
TMEM) whenever the shapes meet its tiling constraints (K and N multiples of
64/16); other shapes, and the ``BRIDGE_B200_GEMM=cublas`` baseline, use cuBLAS
through ``torch.matmul``.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import Tensor

from ._ext import ext, on_gpu

_MODE = os.environ.get("BRIDGE_B200_GEMM", "tcgen05")


def _native_ok(*ts: Tensor) -> bool:
    if _MODE != "tcgen05":
        return False
    m = ext()
    if m is None or not hasattr(m, "gemm_nt"):
        return False
    return all(t.dtype == torch.bfloat16 for t in ts)


def mm_nt(a: Tensor, b: Tensor, out: Tensor | None = None, *, accumulate: bool = False) -> Tensor:
    """``a [M, K] @ b[N, K]^T -> [M, N]`` (bf16 out, FP32 accumulate)."""
    if on_gpu(a) and _native_ok(a, b) and a.shape[1] % 64 == 0 and b.shape[0] % 16 == 0:
        return ext().gemm_nt(a.contiguous(), b.contiguous(), out, accumulate)
    r = torch.matmul(a, b.t())
    if out is None:
        return r
    if accumulate:
        out.add_(r)
    else:
        out.copy_(r)
    return out


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y = mm_nt(x2, w)
        ctx.save_for_backward(x2, w)
        ctx.shape = shape
        return y.view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0]).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            # dx = dy @ W  ==  dy [M,N] x (W^T)[K,N]^T
            dx = mm_nt(dy2, w.t().contiguous()).view(ctx.shape)
        if ctx.needs_input_grad[1]:
            # dW = dy^T @ x == (dy^T)[N,M] x (x^T)[K,M]^T
            dw = mm_nt(dy2.t().contiguous(), x2.t().contiguous())
        return dx, dw


def linear(x: Tensor, weight: Tensor) -> Tensor:
    if on_gpu(x) and _native_ok(x, weight):
        return _LinearFn.apply(x, weight)
    return F.linear(x, weight)

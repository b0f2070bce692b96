"""SwiGLU on a fused ``[gate | up]`` FC1 output: ``silu(gate) * up``.

CUDA kernel (``csrc/elementwise.cu``) reads the packed ``[T, 2F]`` FC1 output
once and writes ``[T, F]``; the backward reads gate/up and ``dy`` and writes
the packed ``[T, 2F]`` gradient in one pass.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from ._ext import kernels, on_gpu


def swiglu_reference(gate_up: Tensor) -> Tensor:
    g, u = gate_up.chunk(2, dim=-1)
    return (F.silu(g.float()) * u.float()).to(gate_up.dtype)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return kernels().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dy):
        (gu,) = ctx.saved_tensors
        return kernels().swiglu_bwd(dy.contiguous(), gu)


def swiglu(gate_up: Tensor) -> Tensor:
    if on_gpu(gate_up):
        return _SwiGLUFn.apply(gate_up)
    return swiglu_reference(gate_up)

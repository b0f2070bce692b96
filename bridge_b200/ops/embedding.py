"""Vocab-parallel embedding lookup with a scatter-add backward.

Forward: ``out[t] = W[ids[t] - start]`` for ids inside this rank's rows ``[start, start + rows)``,
zero rows otherwise (the TP all-reduce that follows assembles the full lookup).  Backward: the
gradient rows are added straight into the weight's FP32 ``main_grad`` (the engine's gradient arena)
-- no dense ``[vocab, hidden]`` bf16 gradient is built per call -- or, without one, into a fresh FP32
buffer.  Repeated ids add with FP32 atomics (summation order not fixed).

Parity: the Megatron ``VocabParallelEmbedding`` the reference model uses (masked local lookup +
TP all-reduce).
"""

from __future__ import annotations

import torch
from torch import Tensor

from ._ext import kernels, on_gpu


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, start):
        ids = ids.contiguous()
        ctx.save_for_backward(ids)
        ctx.start, ctx.weight = start, weight
        return kernels().embedding_fwd(ids, weight, start)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        w = ctx.weight
        main = getattr(w, "main_grad", None)
        dy = dy.contiguous()
        if main is not None and main.dtype == torch.float32 and main.is_contiguous():
            kernels().embedding_bwd_acc(ids, dy, main.view(w.shape), ctx.start)
            return None, None, None
        g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        kernels().embedding_bwd_acc(ids, dy, g, ctx.start)
        return None, g.to(w.dtype), None


def embedding(ids: Tensor, weight: Tensor, start: int = 0) -> Tensor:
    """Rows of ``weight`` for ``ids - start`` (zero for ids outside ``[start, start + len(weight))``)."""
    if on_gpu(weight) and weight.dtype == torch.bfloat16 and weight.shape[1] % 8 == 0 and ids.dim() == 1:
        return _EmbeddingFn.apply(ids.long(), weight, int(start))
    local = ids - start
    outside = (local < 0) | (local >= weight.shape[0])
    out = torch.nn.functional.embedding(local.clamp(0, weight.shape[0] - 1), weight)
    return out.masked_fill(outside[..., None], 0.0)

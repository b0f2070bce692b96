"""Tensor-parallel building blocks (Megatron-style column/row/vocab sharding).

* column-parallel linear: weight rows sharded, input replicated (identity
  forward, all-reduce of dX backward via :func:`copy_to_tp`);
* row-parallel linear: weight columns sharded, partial outputs all-reduced
  (:func:`reduce_from_tp`) -- or reduce-scattered over tokens under sequence
  parallelism (:func:`reduce_scatter_to_sp`), with the matching all-gather
  (:func:`gather_from_sp`) in front of the next column-parallel GEMM;
* vocab-parallel embedding: out-of-shard ids produce zeros, then all-reduce.

The process group is any ``torch.distributed`` group (NCCL on B200, gloo on
CPU).  ``group=None`` or size 1 makes every helper an identity.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn
from torch import Tensor

from ..ops.gemm import linear


def tp_size(group) -> int:
    return 1 if group is None else dist.get_world_size(group)


def tp_rank(group) -> int:
    return 0 if group is None else dist.get_rank(group)


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherFromSP(torch.autograd.Function):
    """All-gather along tokens (dim 0); backward reduce-scatters."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        out = x.new_empty((x.shape[0] * n, *x.shape[1:]))
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = dist.get_world_size(ctx.group)
        out = g.new_empty((g.shape[0] // n, *g.shape[1:]))
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


class _ReduceScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        out = x.new_empty((x.shape[0] // n, *x.shape[1:]))
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = dist.get_world_size(ctx.group)
        out = g.new_empty((g.shape[0] * n, *g.shape[1:]))
        dist.all_gather_into_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


def copy_to_tp(x: Tensor, group) -> Tensor:
    return x if tp_size(group) == 1 else _CopyToTP.apply(x, group)


def reduce_from_tp(x: Tensor, group) -> Tensor:
    return x if tp_size(group) == 1 else _ReduceFromTP.apply(x, group)


def gather_from_sp(x: Tensor, group) -> Tensor:
    return x if tp_size(group) == 1 else _GatherFromSP.apply(x, group)


def reduce_scatter_to_sp(x: Tensor, group) -> Tensor:
    return x if tp_size(group) == 1 else _ReduceScatterToSP.apply(x, group)


def _init(weight: Tensor, std: float, seed_offset: int) -> None:
    with torch.no_grad():
        weight.normal_(0.0, std)


class ColumnParallelLinear(nn.Module):
    """``out_features`` sharded over the TP group; ``sequence_parallel`` all-gathers tokens first."""

    def __init__(self, in_features: int, out_features: int, *, group=None, sequence_parallel: bool = False,
                 std: float = 0.02, dtype=torch.bfloat16, device=None) -> None:
        super().__init__()
        n = tp_size(group)
        if out_features % n:
            raise ValueError(f"out_features {out_features} not divisible by TP size {n}")
        self.group, self.sp = group, sequence_parallel
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features // n, in_features, dtype=dtype, device=device))
        _init(self.weight, std, 0)
        self.weight.tp_split_dim = 0  # type: ignore[attr-defined]

    def forward(self, x: Tensor) -> Tensor:
        if self.sp and x.dim() == 2:
            from .tp_fused import ag_linear, fused_comm

            comm = fused_comm(self.group, x)
            if comm is not None:
                return ag_linear(x, self.weight, comm)      # all-gather fused into the GEMM
        x = gather_from_sp(x, self.group) if self.sp else copy_to_tp(x, self.group)
        return linear(x, self.weight)


class RowParallelLinear(nn.Module):
    """``in_features`` sharded; output all-reduced (or reduce-scattered under SP)."""

    def __init__(self, in_features: int, out_features: int, *, group=None, sequence_parallel: bool = False,
                 std: float = 0.02, dtype=torch.bfloat16, device=None) -> None:
        super().__init__()
        n = tp_size(group)
        if in_features % n:
            raise ValueError(f"in_features {in_features} not divisible by TP size {n}")
        self.group, self.sp = group, sequence_parallel
        self.weight = nn.Parameter(torch.empty(out_features, in_features // n, dtype=dtype, device=device))
        _init(self.weight, std, 1)
        self.weight.tp_split_dim = 1  # type: ignore[attr-defined]

    def forward(self, x: Tensor) -> Tensor:
        if self.sp and x.dim() == 2:
            from .tp_fused import fused_comm, linear_rs

            comm = fused_comm(self.group, x)
            if comm is not None:
                return linear_rs(x, self.weight, comm)      # reduce-scatter fused into the GEMM epilogue
        y = linear(x, self.weight)
        return reduce_scatter_to_sp(y, self.group) if self.sp else reduce_from_tp(y, self.group)


class VocabParallelEmbedding(nn.Module):
    def __init__(self, vocab: int, dim: int, *, group=None, std: float = 0.02, dtype=torch.bfloat16,
                 device=None) -> None:
        super().__init__()
        n = tp_size(group)
        if vocab % n:
            raise ValueError(f"vocab {vocab} not divisible by TP size {n}")
        self.group = group
        self.vocab, self.per_rank = vocab, vocab // n
        self.start = tp_rank(group) * self.per_rank
        self.weight = nn.Parameter(torch.empty(self.per_rank, dim, dtype=dtype, device=device))
        _init(self.weight, std, 2)
        self.weight.tp_split_dim = 0  # type: ignore[attr-defined]

    def forward(self, ids: Tensor, *, reduce: bool = True) -> Tensor:
        """Rows of out-of-shard ids are zero; ``reduce=False`` returns these per-rank partials (the
        sequence-parallel caller reduce-scatters them instead of all-reducing)."""
        from ..ops.embedding import embedding

        out = embedding(ids, self.weight, self.start)
        return out if (tp_size(self.group) == 1 or not reduce) else reduce_from_tp(out, self.group)


def scaled_init_std(std: float, num_layers: int) -> float:
    return std / math.sqrt(2.0 * num_layers)

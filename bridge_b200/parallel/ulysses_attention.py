"""Ulysses context parallelism: sequence->head all-to-all, full-sequence attention
on local heads, head->sequence all-to-all back.

With contiguous shards, after the seq->head exchange rank r holds the whole
(padded) segment for heads ``[r*H/cp, (r+1)*H/cp)``; the prefix blocks go
through the same exchange (padding stripped), so the attention is plain tree
attention over ``prefix + causal self``.  Requires ``Hq`` and ``Hkv`` divisible
by the CP size.

Parity: verl/models/mcore/tpr/parallel/ulysses_attention.py:47-415.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops.attention import masked_attention, tree_attention
from ..ops._ext import on_gpu
from ..tpr.shard import PrefixShard, SequenceShard, physical_sequence_shard
from .execution_context import CPAttentionBackendBase, LocalKVBlock, prefix_blocks


def _a2a(x: Tensor, group) -> Tensor:
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)  # contiguous, unlike empty_like of a view
    dist.all_to_all_single(out, x, group=group)
    return out


class _SeqToHead(torch.autograd.Function):
    """``[L_local, H, D]`` (contiguous shard) -> ``[cp*L_local, H/cp, D]`` (global order)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        l, h, d = x.shape
        send = x.view(l, n, h // n, d).transpose(0, 1).contiguous()      # [n, l, h/n, d]
        return _a2a(send, group).view(n * l, h // n, d)

    @staticmethod
    def backward(ctx, g):
        return _HeadToSeq.apply(g, ctx.group), None


class _HeadToSeq(torch.autograd.Function):
    """Inverse of :class:`_SeqToHead`."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        lp, hl, d = x.shape
        recv = _a2a(x.view(n, lp // n, hl, d), group)                    # [n(src head chunk), l, hl, d]
        return recv.transpose(0, 1).reshape(lp // n, n * hl, d)

    @staticmethod
    def backward(ctx, g):
        return _SeqToHead.apply(g, ctx.group), None


def sequence_to_head(x: Tensor, group) -> Tensor:
    return _SeqToHead.apply(x, group)


def head_to_sequence(x: Tensor, group) -> Tensor:
    return _HeadToSeq.apply(x, group)


def ulysses_cp_rectangular_attention(query: Tensor, key: Tensor, value: Tensor, *,
                                     prefix_blocks: tuple[LocalKVBlock, ...], current_shard: SequenceShard,
                                     cp_group, softmax_scale: float | None) -> Tensor:
    n = dist.get_world_size(cp_group)
    if query.shape[1] % n or key.shape[1] % n:
        raise ValueError(f"Ulysses CP needs query and KV heads divisible by CP={n}")
    if not isinstance(physical_sequence_shard(current_shard), PrefixShard):
        raise TypeError("Ulysses CP requires contiguous shards")
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
    pk, pv = [], []
    for b in prefix_blocks:
        pk.append(sequence_to_head(b.key, cp_group)[: b.shard.global_length])
        pv.append(sequence_to_head(b.value, cp_group)[: b.shard.global_length])
    qh = sequence_to_head(query, cp_group)
    kh = sequence_to_head(key, cp_group)
    vh = sequence_to_head(value, cp_group)
    P = sum(b.shard.global_length for b in prefix_blocks)
    L, Lp = current_shard.global_length, qh.shape[0]
    if on_gpu(query):
        from ..tpr.context import SegmentBatchLayout

        lay = SegmentBatchLayout.build((Lp,), ((0, P),), device=query.device)
        oh = tree_attention(qh, kh, vh, torch.cat(pk) if pk else None, torch.cat(pv) if pv else None, lay,
                            softmax_scale=scale)
    else:
        dev = query.device
        keys = torch.cat(pk + [kh]) if pk else kh
        vals = torch.cat(pv + [vh]) if pv else vh
        k_valid = torch.arange(keys.shape[0], device=dev) < P + L
        oh = masked_attention(qh, keys, vals, torch.arange(P, P + Lp, device=dev),
                              torch.arange(keys.shape[0], device=dev), k_valid=k_valid, softmax_scale=scale)
    o = head_to_sequence(oh, cp_group)
    valid = current_shard.physical_global_indices(device=o.device) < L
    return o * valid[:, None, None].to(o.dtype)


class UlyssesCPAttentionBackend(CPAttentionBackendBase):
    def attention(self, layer_number: int, query: Tensor, key: Tensor, value: Tensor, *,
                  softmax_scale: float | None = None) -> Tensor:
        return ulysses_cp_rectangular_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                                current_shard=self.current_shard, cp_group=self.cp_group,
                                                softmax_scale=softmax_scale)


def make_ulysses_cp_backend(kv_stack, *, expected_layer_numbers, current_shard, cp_group, past_anchors=None):
    blocks = prefix_blocks(kv_stack, expected_layer_numbers, past_anchors)
    prefix = sum(e.state.shard.global_length for e in kv_stack.entries())
    return UlyssesCPAttentionBackend(blocks_by_layer=blocks, current_shard=current_shard, cp_group=cp_group,
                                     global_prefix_length=prefix)

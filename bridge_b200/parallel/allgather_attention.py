"""All-gather context parallelism: gather every prefix block and the current K/V,
then attend the local (contiguous) query shard.

Differentiable sequence all-gather: forward ``all_gather_into_tensor`` along
tokens, backward ``reduce_scatter_tensor`` (SUM) back to the owner.  After
gathering, padding rows of each segment are dropped so the prefix bank holds
exactly ``P`` valid tokens.  The local queries ``[r*c, (r+1)*c)`` of the
current segment see the gathered prefix, the current keys before their shard
(fully) and their own shard causally -- which is exactly the tree-attention
kernel's ``prefix span + causal self`` structure, so no mask tensor is built.

Parity: verl/models/mcore/tpr/parallel/allgather_attention.py:55-382.
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


class _AllGatherSequence(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        out = x.new_empty((n * x.shape[0], *x.shape[1:]))
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = dist.get_world_size(ctx.group)
        out = g.new_empty((g.shape[0] // n, *g.shape[1:]))
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


def all_gather_sequence(x: Tensor, group) -> Tensor:
    """Differentiable all-gather along dim 0 (rank order)."""
    return _AllGatherSequence.apply(x, group)


def _gather_global(block_k: Tensor, block_v: Tensor, shard: SequenceShard, group) -> tuple[Tensor, Tensor]:
    """Gather a contiguous-shard segment's K/V in global order, padding removed."""
    if not isinstance(physical_sequence_shard(shard), PrefixShard):
        raise TypeError("AllGather CP prefix blocks must use contiguous shards")
    kk = all_gather_sequence(block_k, group)
    vv = all_gather_sequence(block_v, group)
    return kk[: shard.global_length], vv[: shard.global_length]


def allgather_cp_rectangular_attention(query: Tensor, key: Tensor, value: Tensor, *,
                                       prefix_blocks: tuple[LocalKVBlock, ...], current_shard: SequenceShard,
                                       cp_group, softmax_scale: float | None) -> Tensor:
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
    phys = physical_sequence_shard(current_shard)
    if not isinstance(phys, PrefixShard):
        raise TypeError("AllGather CP requires contiguous physical sequence placement")
    pk, pv = [], []
    for b in prefix_blocks:
        k, v = _gather_global(b.key, b.value, b.shard, cp_group)
        pk.append(k)
        pv.append(v)
    ck = all_gather_sequence(key, cp_group)
    cv = all_gather_sequence(value, cp_group)
    start = phys.local_start
    P = sum(b.shard.global_length for b in prefix_blocks)
    n_local = query.shape[0]
    valid_q = current_shard.physical_global_indices() < current_shard.global_length
    if on_gpu(query):
        from ..tpr.context import SegmentBatchLayout

        # Always route the gathered current K/V into the graph (an empty bank on rank 0 of a root
        # segment): its backward is a reduce-scatter every CP rank must enter, or the peers hang.
        bank_k = torch.cat(pk + [ck[:start]])
        bank_v = torch.cat(pv + [cv[:start]])
        plen = P + start
        lay = SegmentBatchLayout.build((n_local,), ((0, plen),), device=query.device)
        o = tree_attention(query, key, value, bank_k, bank_v, lay, softmax_scale=scale)
    else:
        keys = torch.cat(pk + [ck]) if pk else ck
        vals = torch.cat(pv + [cv]) if pv else cv
        dev = query.device
        q_pos = P + phys.global_indices(device=dev)
        k_pos = torch.arange(keys.shape[0], device=dev)
        k_valid = torch.ones(keys.shape[0], dtype=torch.bool, device=dev)
        k_valid[P + current_shard.global_length:] = False
        o = masked_attention(query, keys, vals, q_pos, k_pos, k_valid=k_valid, softmax_scale=scale)
    if not bool(valid_q.all()):
        o = o * valid_q.to(o.device)[:, None, None].to(o.dtype)
    return o


class AllGatherCPAttentionBackend(CPAttentionBackendBase):
    def attention(self, layer_number: int, query: Tensor, key: Tensor, value: Tensor, *,
                  softmax_scale: float | None = None) -> Tensor:
        from .cp_p2p import cp_comm, p2p_cp_attention

        comm = cp_comm(self.cp_group, query)
        if comm is not None:     # NVLink P2P gather + tcgen05 attention + P2P dK/dV owner reduction
            scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
            return p2p_cp_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                    current_shard=self.current_shard, comm=comm, softmax_scale=scale)
        return allgather_cp_rectangular_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                                  current_shard=self.current_shard, cp_group=self.cp_group,
                                                  softmax_scale=softmax_scale)


def make_allgather_cp_backend(kv_stack, *, expected_layer_numbers, current_shard, cp_group, past_anchors=None):
    blocks = prefix_blocks(kv_stack, expected_layer_numbers, past_anchors)
    prefix = sum(e.state.shard.global_length for e in kv_stack.entries())
    return AllGatherCPAttentionBackend(blocks_by_layer=blocks, current_shard=current_shard, cp_group=cp_group,
                                       global_prefix_length=prefix)

"""Context-parallel prefix blocks: the local KV shards of the ancestors of a segment.

Under CP every pushed segment keeps only its rank-local K/V shard.  A forward
of segment ``s`` receives, per attention layer, the ordered list of its
ancestors' local blocks (root first) -- cached graph-free tensors during Push,
``requires_grad`` anchors during Pop/VisitLeaf -- and each backend turns them
into full prefix attention with its own communication pattern.

Parity: verl/models/mcore/tpr/parallel/execution_context.py:36-232.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from ..tpr.kv_stack import KVStack
from ..tpr.prefix_state import KVPrefixAnchors
from ..tpr.shard import SequenceShard


def resolve_cp_group(cp_group) -> tuple[int, int]:
    if cp_group is None:
        return 1, 0
    return dist.get_world_size(cp_group), dist.get_rank(cp_group)


@dataclass(frozen=True, slots=True)
class LocalKVBlock:
    """One ancestor segment's rank-local K/V shard for one layer."""

    segment_id: int
    shard: SequenceShard
    key: Tensor
    value: Tensor


RingLocalKVBlock = LocalKVBlock
HybridLocalKVBlock = LocalKVBlock


@dataclass(frozen=True, slots=True)
class ShardedPastKVAnchors:
    entries: tuple[KVPrefixAnchors, ...]
    shards: tuple[SequenceShard, ...]
    stack_signature: tuple[int, ...]

    @property
    def global_prefix_length(self) -> int:
        return sum(s.global_length for s in self.shards)


def build_sharded_past_anchors(kv_stack: KVStack) -> ShardedPastKVAnchors:
    entries, shards = [], []
    for e in kv_stack.entries():
        entries.append(e.state.make_anchors())
        shards.append(e.state.shard)
    return ShardedPastKVAnchors(tuple(entries), tuple(shards), kv_stack.segment_ids)


def accumulate_sharded_past_anchor_gradients(kv_stack: KVStack, anchors: ShardedPastKVAnchors | None) -> None:
    if anchors is None:
        return
    if anchors.stack_signature != kv_stack.segment_ids:
        raise RuntimeError(f"sharded past KV anchors are stale: built for {anchors.stack_signature}, "
                           f"stack is {kv_stack.segment_ids}")
    for a in anchors.entries:
        kv_stack.get(a.segment_id).state.accumulate_anchor_gradients(a)


def prefix_blocks(kv_stack: KVStack, layers: Sequence[int],
                  anchors: ShardedPastKVAnchors | None) -> dict[int, tuple[LocalKVBlock, ...]]:
    """Per-layer ordered ancestor blocks (anchors when given, cached KV otherwise)."""
    out: dict[int, list[LocalKVBlock]] = {layer: [] for layer in layers}
    if anchors is not None:
        if anchors.stack_signature != kv_stack.segment_ids:
            raise RuntimeError("sharded past KV anchors do not match the KV stack")
        for a, shard in zip(anchors.entries, anchors.shards):
            for layer in layers:
                k, v = a.key_values[layer]
                out[layer].append(LocalKVBlock(a.segment_id, shard, k, v))
    else:
        for e in kv_stack.entries():
            for layer in layers:
                k, v = e.state.key_values[layer]
                out[layer].append(LocalKVBlock(e.segment.segment_id, e.state.shard, k, v))
    return {k: tuple(v) for k, v in out.items()}


class CPAttentionBackendBase:
    """Common per-forward state of every CP attention backend."""

    def __init__(self, *, blocks_by_layer: Mapping[int, Sequence[LocalKVBlock]], current_shard: SequenceShard,
                 cp_group, global_prefix_length: int) -> None:
        size, rank = resolve_cp_group(cp_group)
        if (current_shard.cp_size, current_shard.cp_rank) != (size, rank):
            raise ValueError(f"current shard metadata must match the CP group: expected rank {rank}/{size}, got "
                             f"{current_shard.cp_rank}/{current_shard.cp_size}")
        sig = None
        for layer, blocks in blocks_by_layer.items():
            s = tuple(b.segment_id for b in blocks)
            if sig is None:
                sig = s
            elif s != sig:
                raise ValueError("prefix path differs across layers")
            if sum(b.shard.global_length for b in blocks) != global_prefix_length:
                raise ValueError(f"layer {layer} prefix blocks do not cover {global_prefix_length} tokens")
        self.blocks_by_layer = dict(blocks_by_layer)
        self.current_shard = current_shard
        self.cp_group = cp_group
        self._prefix = global_prefix_length
        self._size = size

    @property
    def global_prefix_length(self) -> int:
        return self._prefix

    @property
    def global_suffix_length(self) -> int:
        return self.current_shard.global_length

    @property
    def local_suffix_length(self) -> int:
        return self.current_shard.local_length

    @property
    def parallel_size(self) -> int:
        return self._size

    @property
    def layer_numbers(self) -> tuple[int, ...]:
        return tuple(sorted(self.blocks_by_layer))

    def blocks(self, layer_number: int) -> tuple[LocalKVBlock, ...]:
        try:
            return tuple(self.blocks_by_layer[layer_number])
        except KeyError as exc:
            raise KeyError(f"CP context has no layer {layer_number}") from exc

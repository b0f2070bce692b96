"""Hybrid (Ulysses x Ring) context parallelism.

``cp = U * R`` with ``cp_rank = ring_rank * U + ulysses_rank``.  A segment is
zigzag-sharded over the R ring ranks (padded to ``lcm(cp, 2R)``) and each
ring rank's two chunks are cut into U contiguous pieces, one per Ulysses rank.
Attention: seq->head all-to-all inside the Ulysses group (every member then
holds its ring rank's whole zigzag shard for ``H/U`` heads), ring attention
over the R ring ranks, head->seq all-to-all back.  On a single-node CUDA ring
group the ring leg is the NVLink transport of the ring backend (P2P KV row
gathers, the tcgen05 tree-attention kernel, P2P owner reduction of dK/dV);
elsewhere the NCCL / gloo ring.

Parity: verl/models/mcore/tpr/parallel/hybrid_attention.py:42-495
(HybridCPTopology, rank layout, shard, A2A -> ring -> A2A).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist
from torch import Tensor

from ..tpr.shard import (PaddedSequenceShard, RangeSequenceShard, SequenceShard, hybrid_alignment,
                         make_hybrid_sequence_shard, round_up_sequence_length)
from .execution_context import CPAttentionBackendBase, LocalKVBlock, prefix_blocks
from .ring_attention import ring_cp_attention
from .ulysses_attention import head_to_sequence, sequence_to_head


@dataclass(frozen=True)
class HybridCPTopology:
    cp_size: int
    ulysses_size: int
    cp_rank: int
    ulysses_group: object = None
    ring_group: object = None

    def __post_init__(self) -> None:
        if self.ulysses_size <= 1 or self.cp_size % self.ulysses_size or self.cp_size // self.ulysses_size <= 1:
            raise ValueError("hybrid CP needs U > 1 and R = cp/U > 1")

    @property
    def ring_size(self) -> int:
        return self.cp_size // self.ulysses_size

    @property
    def ring_rank(self) -> int:
        return self.cp_rank // self.ulysses_size

    @property
    def ulysses_rank(self) -> int:
        return self.cp_rank % self.ulysses_size

    def ulysses_members(self, ring_rank: int) -> tuple[int, ...]:
        return tuple(ring_rank * self.ulysses_size + u for u in range(self.ulysses_size))

    def ring_members(self, ulysses_rank: int) -> tuple[int, ...]:
        return tuple(r * self.ulysses_size + ulysses_rank for r in range(self.ring_size))


def resolve_mindspeed_hybrid_topology(cp_group, ulysses_size: int) -> HybridCPTopology:
    """Create the Ulysses and ring sub-groups of ``cp_group`` (every rank of the world must call this)."""
    n, r = dist.get_world_size(cp_group), dist.get_rank(cp_group)
    base = HybridCPTopology(n, ulysses_size, r)
    glob = [dist.get_global_rank(cp_group, i) for i in range(n)]
    ug = rg = None
    for rr in range(base.ring_size):
        g = dist.new_group([glob[i] for i in base.ulysses_members(rr)])
        if rr == base.ring_rank:
            ug = g
    for u in range(ulysses_size):
        g = dist.new_group([glob[i] for i in base.ring_members(u)])
        if u == base.ulysses_rank:
            rg = g
    return HybridCPTopology(n, ulysses_size, r, ug, rg)


def _ring_view(shard: SequenceShard, topo: HybridCPTopology) -> SequenceShard:
    """The ring-level zigzag shard a Ulysses group jointly holds after seq->head."""
    R = topo.ring_size
    padded = round_up_sequence_length(shard.global_length, hybrid_alignment(topo.cp_size, topo.ulysses_size))
    c = padded // (2 * R)
    rr = topo.ring_rank
    phys = RangeSequenceShard(padded, ((rr * c, (rr + 1) * c), ((2 * R - 1 - rr) * c, (2 * R - rr) * c)), rr, R)
    return phys if padded == shard.global_length else PaddedSequenceShard(shard.global_length, phys)


def hybrid_cp_rectangular_attention(query: Tensor, key: Tensor, value: Tensor, *,
                                    prefix_blocks: tuple[LocalKVBlock, ...], current_shard: SequenceShard,
                                    topology: HybridCPTopology, softmax_scale: float | None) -> Tensor:
    ug = topology.ulysses_group
    qh, kh, vh = (sequence_to_head(t, ug) for t in (query, key, value))
    ring_prefix = tuple(
        LocalKVBlock(b.segment_id, _ring_view(b.shard, topology), sequence_to_head(b.key, ug),
                     sequence_to_head(b.value, ug))
        for b in prefix_blocks
    )
    ring_shard = _ring_view(current_shard, topology)
    from .cp_p2p import cp_comm, p2p_cp_attention

    comm = cp_comm(topology.ring_group, qh)
    if comm is not None:        # CUDA, one node: P2P KV rows + tcgen05 tree attention + P2P owner reduction
        scale = softmax_scale if softmax_scale is not None else qh.shape[-1] ** -0.5
        oh = p2p_cp_attention(qh, kh, vh, prefix_blocks=ring_prefix, current_shard=ring_shard, comm=comm,
                              softmax_scale=scale)
    else:                       # NCCL / gloo ring (baseline and CPU path)
        oh = ring_cp_attention(qh, kh, vh, prefix_blocks=ring_prefix, current_shard=ring_shard,
                               cp_group=topology.ring_group, softmax_scale=softmax_scale)
    return head_to_sequence(oh, ug)


class HybridCPAttentionBackend(CPAttentionBackendBase):
    def __init__(self, *, topology: HybridCPTopology, **kw) -> None:
        super().__init__(**kw)
        self.topology = topology

    def attention(self, layer_number: int, query: Tensor, key: Tensor, value: Tensor, *,
                  softmax_scale: float | None = None) -> Tensor:
        return hybrid_cp_rectangular_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                               current_shard=self.current_shard, topology=self.topology,
                                               softmax_scale=softmax_scale)


def make_hybrid_cp_backend(kv_stack, *, expected_layer_numbers, current_shard, cp_group, topology,
                           past_anchors=None):
    blocks = prefix_blocks(kv_stack, expected_layer_numbers, past_anchors)
    prefix = sum(e.state.shard.global_length for e in kv_stack.entries())
    return HybridCPAttentionBackend(topology=topology, blocks_by_layer=blocks, current_shard=current_shard,
                                    cp_group=cp_group, global_prefix_length=prefix)


__all__ = ["HybridCPTopology", "resolve_mindspeed_hybrid_topology", "make_hybrid_sequence_shard",
           "hybrid_cp_rectangular_attention", "HybridCPAttentionBackend", "make_hybrid_cp_backend"]

"""Context-parallel backend policies and their resolver.

A policy owns sequence placement (``make_sequence_shard``) and builds the
per-forward attention backend from the KV stack (cached ancestor shards during
Push, anchors during Pop/VisitLeaf).  Names accept both this framework's short
names and the MindSpeed algorithm names; unknown names fail (no silent
fallback).

Parity: verl/models/mcore/tpr/parallel/backend.py:54-376.
"""

from __future__ import annotations

from typing import Any, Protocol, runtime_checkable

from ..tpr.shard import (PrefixShard, RangeSequenceShard, SequenceShard, make_hybrid_sequence_shard,
                         make_ring_sequence_shard, maybe_pad_sequence_shard, physical_sequence_shard,
                         round_up_sequence_length)
from .execution_context import resolve_cp_group

ALLGATHER_CP_BACKEND = "allgather"
MINDSPEED_ALLGATHER_CP_ALGO = "kvallgather_cp_algo"
ULYSSES_CP_BACKEND = "ulysses"
MINDSPEED_ULYSSES_CP_ALGO = "ulysses_cp_algo"
RING_CP_BACKEND = "ring"
MINDSPEED_RING_CP_ALGO = "megatron_cp_algo"
HYBRID_CP_BACKEND = "hybrid"
MINDSPEED_HYBRID_CP_ALGO = "hybrid_cp_algo"


@runtime_checkable
class TPRCPBackend(Protocol):
    @property
    def backend_name(self) -> str: ...
    @property
    def parallel_size(self) -> int: ...
    @property
    def parallel_rank(self) -> int: ...
    def validate_segment_length(self, global_length: int) -> None: ...
    def make_sequence_shard(self, global_length: int) -> SequenceShard: ...
    def make_attention_backend(self, kv_stack, *, expected_layer_numbers, current_shard, past_anchors): ...


class AllGatherCPBackend:
    backend_name = ALLGATHER_CP_BACKEND

    def __init__(self, cp_group: Any, *, parallel_size: int | None = None, parallel_rank: int | None = None) -> None:
        if (parallel_size is None) != (parallel_rank is None):
            raise ValueError("parallel_size and parallel_rank must be provided together")
        if parallel_size is None:
            parallel_size, parallel_rank = resolve_cp_group(cp_group)
        if parallel_size <= 1:
            raise ValueError(f"{self.backend_name} CP requires more than one rank, got {parallel_size}")
        if not 0 <= parallel_rank < parallel_size:
            raise ValueError(f"parallel_rank must be in [0, {parallel_size}), got {parallel_rank}")
        self._group, self._size, self._rank = cp_group, parallel_size, parallel_rank

    @property
    def parallel_size(self) -> int:
        return self._size

    @property
    def parallel_rank(self) -> int:
        return self._rank

    @property
    def cp_group(self):
        return self._group

    def validate_segment_length(self, global_length: int) -> None:
        if not isinstance(global_length, int) or isinstance(global_length, bool) or global_length <= 0:
            raise ValueError(f"length must be a positive integer, got {global_length!r}")

    def make_sequence_shard(self, global_length: int) -> SequenceShard:
        self.validate_segment_length(global_length)
        padded = round_up_sequence_length(global_length, self._size)
        return maybe_pad_sequence_shard(global_length, PrefixShard.contiguous(padded, cp_rank=self._rank,
                                                                              cp_size=self._size))

    def _require(self, shard, kind) -> None:
        if not isinstance(physical_sequence_shard(shard), kind):
            raise TypeError(f"{self.backend_name} CP requires a {kind.__name__}, got {type(shard).__name__}")

    def make_attention_backend(self, kv_stack, *, expected_layer_numbers, current_shard, past_anchors=None):
        from .allgather_attention import make_allgather_cp_backend

        self._require(current_shard, PrefixShard)
        return make_allgather_cp_backend(kv_stack, expected_layer_numbers=expected_layer_numbers,
                                         current_shard=current_shard, cp_group=self._group,
                                         past_anchors=past_anchors)


class UlyssesCPBackend(AllGatherCPBackend):
    backend_name = ULYSSES_CP_BACKEND

    def make_attention_backend(self, kv_stack, *, expected_layer_numbers, current_shard, past_anchors=None):
        from .ulysses_attention import make_ulysses_cp_backend

        self._require(current_shard, PrefixShard)
        return make_ulysses_cp_backend(kv_stack, expected_layer_numbers=expected_layer_numbers,
                                       current_shard=current_shard, cp_group=self._group, past_anchors=past_anchors)


class RingCPBackend(AllGatherCPBackend):
    backend_name = RING_CP_BACKEND

    def validate_segment_length(self, global_length: int) -> None:
        make_ring_sequence_shard(global_length, cp_rank=self._rank, cp_size=self._size)

    def make_sequence_shard(self, global_length: int) -> SequenceShard:
        return make_ring_sequence_shard(global_length, cp_rank=self._rank, cp_size=self._size)

    def make_attention_backend(self, kv_stack, *, expected_layer_numbers, current_shard, past_anchors=None):
        from .ring_attention import make_ring_cp_backend

        self._require(current_shard, RangeSequenceShard)
        return make_ring_cp_backend(kv_stack, expected_layer_numbers=expected_layer_numbers,
                                    current_shard=current_shard, cp_group=self._group, past_anchors=past_anchors)


class HybridCPBackend(AllGatherCPBackend):
    backend_name = HYBRID_CP_BACKEND

    def __init__(self, cp_group: Any, *, ulysses_size: int | None = None, topology=None,
                 parallel_size: int | None = None, parallel_rank: int | None = None) -> None:
        super().__init__(cp_group, parallel_size=parallel_size, parallel_rank=parallel_rank)
        if topology is None:
            from .hybrid_attention import resolve_mindspeed_hybrid_topology

            u = ulysses_size if ulysses_size is not None else 2
            topology = resolve_mindspeed_hybrid_topology(cp_group, u)
        self.topology = topology

    def validate_segment_length(self, global_length: int) -> None:
        make_hybrid_sequence_shard(global_length, cp_rank=self._rank, cp_size=self._size,
                                   ulysses_size=self.topology.ulysses_size)

    def make_sequence_shard(self, global_length: int) -> SequenceShard:
        return make_hybrid_sequence_shard(global_length, cp_rank=self._rank, cp_size=self._size,
                                          ulysses_size=self.topology.ulysses_size)

    def make_attention_backend(self, kv_stack, *, expected_layer_numbers, current_shard, past_anchors=None):
        from .hybrid_attention import make_hybrid_cp_backend

        return make_hybrid_cp_backend(kv_stack, expected_layer_numbers=expected_layer_numbers,
                                      current_shard=current_shard, cp_group=self._group, topology=self.topology,
                                      past_anchors=past_anchors)


_NAMES = {
    ALLGATHER_CP_BACKEND: AllGatherCPBackend, MINDSPEED_ALLGATHER_CP_ALGO: AllGatherCPBackend,
    ULYSSES_CP_BACKEND: UlyssesCPBackend, MINDSPEED_ULYSSES_CP_ALGO: UlyssesCPBackend,
    RING_CP_BACKEND: RingCPBackend, MINDSPEED_RING_CP_ALGO: RingCPBackend,
    HYBRID_CP_BACKEND: HybridCPBackend, MINDSPEED_HYBRID_CP_ALGO: HybridCPBackend,
}


def resolve_tpr_cp_backend(backend, *, cp_group, parallel_size: int, parallel_rank: int, **kw):
    """Return a backend policy for a name, or validate and return a policy object."""
    if backend is None:
        backend = ALLGATHER_CP_BACKEND
    if isinstance(backend, str):
        cls = _NAMES.get(backend)
        if cls is None:
            raise ValueError(f"unknown TPR CP backend {backend!r}; known: {sorted(_NAMES)}")
        return cls(cp_group, parallel_size=parallel_size, parallel_rank=parallel_rank, **kw)
    missing = [n for n in ("backend_name", "parallel_size", "parallel_rank", "validate_segment_length",
                           "make_sequence_shard", "make_attention_backend") if not hasattr(backend, n)]
    if missing:
        raise TypeError(f"custom CP backend is missing {missing}")
    if (backend.parallel_size, backend.parallel_rank) != (parallel_size, parallel_rank):
        raise ValueError("custom CP backend size/rank do not match the CP group")
    return backend

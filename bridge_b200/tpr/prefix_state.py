"""Graph-free prefix state of pushed segments and its delayed gradients.

A pushed segment leaves two kinds of continuation state for its descendants:

* **KV** -- post-RoPE K and raw V of every attention layer (``[L, Hkv, D]``
  packed token-major; under CP the rank-local shard);
* **GDN** -- the causal-conv tail ``[B, C, W]`` and the recurrent state
  ``[B, H, K, V]`` (FP32) of every Gated-DeltaNet layer.

Both are handled by one generic :class:`_LayerTupleState`: per layer a tuple
of detached compact tensors, per-layer FP32-or-native gradient accumulators,
autograd *anchors* (fresh ``requires_grad`` leaves over the same storage) and
a generation counter that makes anchors from an earlier consume/release stale.

Parity: verl/models/mcore/tpr/prefix_state.py:42-708 (PrefixState protocol,
GDNLayerState, GDNPrefixState, KVPrefixState, PrefixStateStack).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Protocol, runtime_checkable

import torch
from torch import Tensor

from .segment_plan import SegmentId, SegmentSpec, check_nonneg_int
from .shard import PrefixShard, SequenceShard

KVPair = tuple[Tensor, Tensor]


def _check_layer(layer: int) -> None:
    if not isinstance(layer, int) or isinstance(layer, bool) or layer <= 0:
        raise ValueError(f"layer_number must be a positive integer, got {layer!r}")


def _compact(t: Tensor) -> Tensor:
    t = t.detach()
    return t if t.is_contiguous() and t.storage_offset() == 0 and t.untyped_storage().nbytes() == t.nbytes \
        else t.clone(memory_format=torch.contiguous_format)


@runtime_checkable
class PrefixState(Protocol):
    state_kind: str

    @property
    def segment_id(self) -> SegmentId: ...
    @property
    def layer_numbers(self) -> tuple[int, ...]: ...
    @property
    def released(self) -> bool: ...
    def validate(self) -> None: ...
    def make_anchors(self) -> Any: ...
    def accumulate_anchor_gradients(self, anchors: Any) -> None: ...
    def consume_gradients(self) -> Any: ...
    def release(self) -> None: ...


@dataclass(frozen=True, slots=True)
class GDNLayerState:
    """Causal-conv ``[B, C, W]`` and recurrent ``[B, H, K, V]`` continuation of one GDN layer."""

    conv_state: Tensor
    recurrent_state: Tensor

    def __post_init__(self) -> None:
        c, r = self.conv_state, self.recurrent_state
        if not isinstance(c, Tensor) or not isinstance(r, Tensor):
            raise TypeError("GDN conv_state and recurrent_state must be torch tensors")
        if c.ndim != 3:
            raise ValueError(f"GDN conv_state must have shape [batch, channels, history], got {tuple(c.shape)}")
        if r.ndim != 4:
            raise ValueError(
                f"GDN recurrent_state must have shape [batch, heads, key_dim, value_dim], got {tuple(r.shape)}"
            )
        if min(c.shape) <= 0 or min(r.shape) <= 0:
            raise ValueError("GDN state dimensions must be positive")
        if c.shape[0] != r.shape[0]:
            raise ValueError("GDN continuation states must have the same batch size")
        if c.device != r.device:
            raise ValueError("GDN continuation states must be on the same device")
        if not c.is_floating_point() or not r.is_floating_point():
            raise ValueError("GDN conv_state and recurrent_state must be floating-point tensors")

    def as_tuple(self) -> tuple[Tensor, Tensor]:
        return (self.conv_state, self.recurrent_state)


@dataclass(frozen=True, slots=True)
class GDNPrefixAnchors:
    segment_id: SegmentId
    generation: int
    layer_states: Mapping[int, GDNLayerState]


@dataclass(frozen=True, slots=True)
class KVPrefixAnchors:
    segment_id: SegmentId
    generation: int
    key_values: Mapping[int, KVPair]


class _LayerTupleState:
    """Per-layer tuples of graph-free tensors plus accumulated gradients."""

    state_kind = "?"

    def __init__(self, segment_id: SegmentId, layers: Mapping[int, tuple[Tensor, ...]]) -> None:
        check_nonneg_int(segment_id, "segment_id")
        if not isinstance(layers, Mapping) or not layers:
            raise ValueError(f"{self.state_kind} layer states must be a non-empty mapping")
        self._segment_id = segment_id
        self._layers: dict[int, tuple[Tensor, ...]] = {}
        for layer in sorted(layers):
            _check_layer(layer)
            tensors = tuple(layers[layer])
            for t in tensors:
                if t.requires_grad or t.grad_fn is not None:
                    raise ValueError(f"layer {layer} cached {self.state_kind} state must be detached and graph-free")
            self._layers[layer] = tuple(_compact(t) for t in tensors)
        self._grads: dict[int, list[Tensor]] = {}
        self._generation = 0
        self._released = False

    # -- protocol
    @property
    def segment_id(self) -> SegmentId:
        return self._segment_id

    @property
    def layer_numbers(self) -> tuple[int, ...]:
        return tuple(self._layers)

    @property
    def released(self) -> bool:
        return self._released

    @property
    def generation(self) -> int:
        return self._generation

    def _live(self) -> None:
        if self._released:
            raise RuntimeError(f"{self.state_kind} prefix state for segment {self._segment_id} has been released")

    def validate(self) -> None:
        self._live()
        for layer, tensors in self._layers.items():
            for t in tensors:
                if t.requires_grad or t.grad_fn is not None:
                    raise RuntimeError(f"segment {self._segment_id} layer {layer} state gained a graph")

    def _anchor_tuples(self) -> dict[int, tuple[Tensor, ...]]:
        self._live()
        return {layer: tuple(t.detach().requires_grad_(True) for t in ts) for layer, ts in self._layers.items()}

    def _accumulate(self, layer: int, grads: tuple[Tensor | None, ...]) -> None:
        self._live()
        _check_layer(layer)
        saved = self._layers.get(layer)
        if saved is None:
            raise KeyError(f"segment {self._segment_id} has no {self.state_kind} state for layer {layer}")
        if len(grads) != len(saved):
            raise ValueError("gradient tuple arity mismatch")
        for g, s in zip(grads, saved):
            if g is not None and (g.shape != s.shape or g.device != s.device):
                raise ValueError(
                    f"segment {self._segment_id} layer {layer} gradient shape/device mismatch: "
                    f"expected {tuple(s.shape)}, got {tuple(g.shape)}"
                )
        acc = self._grads.get(layer)
        if acc is None:
            self._grads[layer] = [
                torch.zeros_like(s) if g is None else g.detach().to(s.dtype).clone(memory_format=torch.contiguous_format)
                for g, s in zip(grads, saved)
            ]
        else:
            for a, g in zip(acc, grads):
                if g is not None:
                    a.add_(g.detach())

    def _consume(self) -> dict[int, tuple[Tensor, ...]]:
        self._live()
        if self._grads and tuple(sorted(self._grads)) != self.layer_numbers:
            raise RuntimeError(
                f"segment {self._segment_id} gradient layers must be {self.layer_numbers}, got {tuple(self._grads)}"
            )
        out = {layer: tuple(g) for layer, g in sorted(self._grads.items())}
        self._grads = {}
        self._generation += 1
        return out

    def release(self) -> None:
        if self._released:
            return
        self._layers.clear()
        self._grads.clear()
        self._released = True
        self._generation += 1

    def _check_anchor_owner(self, segment_id: SegmentId, generation: int) -> None:
        self._live()
        if segment_id != self._segment_id or generation != self._generation:
            raise RuntimeError(f"{self.state_kind} prefix anchors for segment {segment_id} are stale")


class GDNPrefixState(_LayerTupleState):
    """GDN continuation states of one pushed segment and their relayed gradients."""

    state_kind = "gdn"

    def __init__(self, segment_id: SegmentId, sequence_length: int, layer_states: Mapping[int, GDNLayerState]) -> None:
        if not isinstance(sequence_length, int) or isinstance(sequence_length, bool) or sequence_length <= 0:
            raise ValueError(f"sequence_length must be positive, got {sequence_length!r}")
        for layer, st in layer_states.items():
            if not isinstance(st, GDNLayerState):
                raise TypeError(f"layer {layer} state must be GDNLayerState, got {type(st).__name__}")
        devices = {st.conv_state.device for st in layer_states.values()}
        batches = {st.conv_state.shape[0] for st in layer_states.values()}
        if len(devices) > 1 or len(batches) > 1:
            raise ValueError("all GDN layers in a prefix state must use the same device and batch size")
        super().__init__(segment_id, {k: v.as_tuple() for k, v in layer_states.items()})
        self._sequence_length = sequence_length

    @classmethod
    def save(cls, segment_id: SegmentId, sequence_length: int,
             layer_states: Mapping[int, GDNLayerState]) -> "GDNPrefixState":
        """Detach + compact the states a Push produced."""
        return cls(segment_id, sequence_length, {
            k: GDNLayerState(v.conv_state.detach().clone(memory_format=torch.contiguous_format),
                             v.recurrent_state.detach().clone(memory_format=torch.contiguous_format))
            for k, v in layer_states.items()
        })

    @property
    def sequence_length(self) -> int:
        return self._sequence_length

    @property
    def layer_states(self) -> Mapping[int, GDNLayerState]:
        self._live()
        return MappingProxyType({k: GDNLayerState(*v) for k, v in self._layers.items()})

    @property
    def gradients(self) -> Mapping[int, GDNLayerState]:
        return MappingProxyType({k: GDNLayerState(*v) for k, v in self._grads.items()})

    def restore(self, layer_number: int) -> GDNLayerState:
        self._live()
        try:
            return GDNLayerState(*self._layers[layer_number])
        except KeyError as exc:
            raise KeyError(f"segment {self._segment_id} has no GDN state for layer {layer_number}") from exc

    def make_anchors(self) -> GDNPrefixAnchors:
        return GDNPrefixAnchors(self._segment_id, self._generation,
                                MappingProxyType({k: GDNLayerState(*v) for k, v in self._anchor_tuples().items()}))

    def accumulate_layer_gradients(self, layer_number: int, conv_grad: Tensor, recurrent_grad: Tensor) -> None:
        self._accumulate(layer_number, (conv_grad, recurrent_grad))

    def accumulate_anchor_gradients(self, anchors: GDNPrefixAnchors) -> None:
        if not isinstance(anchors, GDNPrefixAnchors):
            raise TypeError(f"anchors must be GDNPrefixAnchors, got {type(anchors).__name__}")
        self._check_anchor_owner(anchors.segment_id, anchors.generation)
        if tuple(anchors.layer_states) != self.layer_numbers:
            raise RuntimeError(f"GDN prefix anchor layers must be {self.layer_numbers}")
        for layer, st in anchors.layer_states.items():
            if st.conv_state.grad is None and st.recurrent_state.grad is None:
                raise RuntimeError(f"layer {layer} GDN prefix anchor gradient is missing")
            self._accumulate(layer, (st.conv_state.grad, st.recurrent_state.grad))

    def consume_gradients(self) -> Mapping[int, GDNLayerState]:
        return MappingProxyType({k: GDNLayerState(*v) for k, v in self._consume().items()})


class KVPrefixState(_LayerTupleState):
    """Compact K/V of one pushed segment (rank-local under CP) and relayed dK/dV."""

    state_kind = "kv"

    def __init__(self, segment_id: SegmentId, sequence_length: int, key_values: Mapping[int, KVPair], *,
                 shard: SequenceShard | None = None) -> None:
        if not isinstance(sequence_length, int) or isinstance(sequence_length, bool) or sequence_length <= 0:
            raise ValueError(f"sequence_length must be positive, got {sequence_length!r}")
        shard = PrefixShard.full(sequence_length) if shard is None else shard
        if shard.global_length != sequence_length:
            raise ValueError("KV shard global length must equal the segment length")
        ref = None
        for layer, pair in key_values.items():
            if not isinstance(pair, tuple) or len(pair) != 2:
                raise TypeError(f"layer {layer} KV must be a (key, value) tuple")
            k, v = pair
            if k.ndim != 3 or v.ndim != 3 or k.shape[:2] != v.shape[:2]:
                raise ValueError(f"layer {layer} KV must be [tokens, heads, head_dim] with matching K/V")
            if k.shape[0] != shard.local_length:
                raise ValueError(f"layer {layer} KV length {k.shape[0]} != local shard length {shard.local_length}")
            sig = (k.shape[1:], k.device, k.dtype)
            if ref is None:
                ref = sig
            elif sig != ref:
                raise ValueError("all KV layers of a segment must share head shape, device and dtype")
        super().__init__(segment_id, key_values)
        self._sequence_length = sequence_length
        self._shard = shard

    @property
    def shard(self) -> SequenceShard:
        return self._shard

    @property
    def sequence_length(self) -> int:
        return self._sequence_length

    @property
    def global_length(self) -> int:
        return self._sequence_length

    @property
    def local_length(self) -> int:
        return self._shard.local_length

    @property
    def key_values(self) -> Mapping[int, KVPair]:
        self._live()
        return MappingProxyType({k: (v[0], v[1]) for k, v in self._layers.items()})

    @property
    def gradients(self) -> Mapping[int, KVPair]:
        return MappingProxyType({k: (v[0], v[1]) for k, v in self._grads.items()})

    def make_anchors(self) -> KVPrefixAnchors:
        return KVPrefixAnchors(self._segment_id, self._generation,
                               MappingProxyType({k: (v[0], v[1]) for k, v in self._anchor_tuples().items()}))

    def accumulate_layer_gradients(self, layer_number: int, key_grad: Tensor, value_grad: Tensor) -> None:
        self._accumulate(layer_number, (key_grad, value_grad))

    def accumulate_anchor_gradients(self, anchors: KVPrefixAnchors) -> None:
        if not isinstance(anchors, KVPrefixAnchors):
            raise TypeError(f"anchors must be KVPrefixAnchors, got {type(anchors).__name__}")
        self._check_anchor_owner(anchors.segment_id, anchors.generation)
        for layer, (k, v) in anchors.key_values.items():
            if k.grad is None and v.grad is None:
                raise RuntimeError(f"layer {layer} KV prefix anchor gradient is missing")
            self._accumulate(layer, (k.grad, v.grad))

    def consume_gradients(self) -> Mapping[int, KVPair]:
        return MappingProxyType({k: (v[0], v[1]) for k, v in self._consume().items()})


SegmentKV = KVPrefixState


class PrefixStateEntry:
    """One segment on the active root-to-leaf path with its state."""

    __slots__ = ("segment", "state")

    def __init__(self, segment: SegmentSpec, state) -> None:
        self.segment = segment
        self.state = state


class PrefixStateStack:
    """The active DFS path: entries pushed in root->leaf order."""

    label = "prefix-state stack"      # how error messages name this stack

    def __init__(self) -> None:
        self._entries: list[PrefixStateEntry] = []

    def __len__(self) -> int:
        return len(self._entries)

    @property
    def segment_ids(self) -> tuple[SegmentId, ...]:
        return tuple(e.segment.segment_id for e in self._entries)

    @property
    def prefix_length(self) -> int:
        return self._entries[-1].segment.position_end if self._entries else 0

    def entries(self) -> tuple[PrefixStateEntry, ...]:
        return tuple(self._entries)

    def top(self) -> PrefixStateEntry:
        if not self._entries:
            raise RuntimeError(f"{self.label} is empty")
        return self._entries[-1]

    def get(self, segment_id: SegmentId) -> PrefixStateEntry:
        for e in self._entries:
            if e.segment.segment_id == segment_id:
                return e
        raise KeyError(f"segment {segment_id} is not on the {self.label}")

    def push_state(self, segment: SegmentSpec, state, *, entry_type=PrefixStateEntry) -> PrefixStateEntry:
        if not isinstance(segment, SegmentSpec):
            raise TypeError("segment must be a SegmentSpec")
        if state.segment_id != segment.segment_id:
            raise ValueError("state segment_id must match the pushed segment")
        parent = self._entries[-1].segment.segment_id if self._entries else None
        if segment.parent_id != parent:
            raise ValueError(f"cannot push segment {segment.segment_id}: parent on stack is {parent}, "
                             f"segment parent is {segment.parent_id}")
        if segment.prefix_length != self.prefix_length:
            raise ValueError(f"segment {segment.segment_id} prefix_length {segment.prefix_length} does not match "
                             f"stack prefix length {self.prefix_length}")
        entry = entry_type(segment, state)
        self._entries.append(entry)
        return entry

    def pop_state(self, segment_id: SegmentId) -> PrefixStateEntry:
        if not self._entries or self._entries[-1].segment.segment_id != segment_id:
            raise RuntimeError(f"cannot pop segment {segment_id}: {self.label} is {list(self.segment_ids)}")
        return self._entries.pop()

    def assert_empty(self) -> None:
        if self._entries:
            raise RuntimeError(f"{self.label} is not empty: {list(self.segment_ids)}")

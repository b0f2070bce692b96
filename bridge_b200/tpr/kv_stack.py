"""KV-specialised prefix stack: ancestor KV bank, anchors and gradient split-back.

``build_past_key_values`` concatenates the ancestors' compact K/V along tokens
(root first) into one bank per layer; ``build_past_anchors`` wraps that bank in
fresh ``requires_grad`` leaves and records each ancestor's slice, and
``accumulate_anchor_gradients`` cuts the leaf gradients back into each
ancestor's dK/dV accumulator.

Parity: verl/models/mcore/tpr/kv_stack.py:36-212.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from types import MappingProxyType

import torch
from torch import Tensor

from .prefix_state import KVPair, KVPrefixState, PrefixStateEntry, PrefixStateStack
from .segment_plan import SegmentId, SegmentSpec
from .shard import SequenceShard


@dataclass(frozen=True, slots=True)
class PastKVSlice:
    segment_id: SegmentId
    start: int
    end: int


@dataclass(frozen=True, slots=True)
class PastKVAnchors:
    key_values: Mapping[int, KVPair]
    slices: tuple[PastKVSlice, ...]
    stack_signature: tuple[SegmentId, ...]

    @property
    def prefix_length(self) -> int:
        return self.slices[-1].end if self.slices else 0


class KVStackEntry(PrefixStateEntry):
    __slots__ = ()

    @property
    def kv(self) -> KVPrefixState:
        if not isinstance(self.state, KVPrefixState):
            raise TypeError(f"KVStackEntry requires KVPrefixState, got {type(self.state).__name__}")
        return self.state

    @property
    def gradients(self) -> Mapping[int, KVPair]:
        return self.kv.gradients

    def accumulate(self, layer_number: int, key_grad: Tensor, value_grad: Tensor) -> None:
        self.kv.accumulate_layer_gradients(layer_number, key_grad, value_grad)


class KVStack(PrefixStateStack):
    """Graph-free KV and relayed dK/dV of the active DFS path."""

    def top(self) -> KVStackEntry:
        return super().top()  # type: ignore[return-value]

    def get(self, segment_id: SegmentId) -> KVStackEntry:
        try:
            return super().get(segment_id)  # type: ignore[return-value]
        except KeyError as exc:
            raise KeyError(f"segment {segment_id} is not on the KV stack") from exc

    def push(self, segment: SegmentSpec, key_values: Mapping[int, KVPair], *,
             shard: SequenceShard | None = None) -> KVStackEntry:
        kv = KVPrefixState(segment.segment_id, segment.length, key_values, shard=shard)
        if self._entries:
            first = self._entries[0].state
            if kv.layer_numbers != first.layer_numbers:
                raise ValueError(f"segment {segment.segment_id} KV layers must be {first.layer_numbers}, "
                                 f"got {kv.layer_numbers}")
            prev = self._entries[-1].state
            for layer in kv.layer_numbers:
                a, b = prev.key_values[layer][0], kv.key_values[layer][0]
                if a.shape[1:] != b.shape[1:] or a.device != b.device or a.dtype != b.dtype:
                    raise ValueError(f"layer {layer} KV head shape, device or dtype differs across segments")
        return self.push_state(segment, kv, entry_type=KVStackEntry)  # type: ignore[return-value]

    def pop(self, segment_id: SegmentId) -> KVStackEntry:
        try:
            return self.pop_state(segment_id)  # type: ignore[return-value]
        except RuntimeError as exc:
            raise RuntimeError(str(exc).replace("prefix-state stack", "KV stack")) from exc

    def build_past_key_values(self) -> Mapping[int, KVPair]:
        if not self._entries:
            return MappingProxyType({})
        if any(e.state.shard.cp_size != 1 for e in self._entries):
            raise RuntimeError("sharded KV must be consumed through a context-parallel attention backend")
        out = {}
        for layer in self._entries[0].state.layer_numbers:
            ks = [e.state.key_values[layer][0] for e in self._entries]
            vs = [e.state.key_values[layer][1] for e in self._entries]
            out[layer] = (ks[0], vs[0]) if len(ks) == 1 else (torch.cat(ks), torch.cat(vs))
        return MappingProxyType(out)

    def build_past_anchors(self) -> PastKVAnchors:
        bank = self.build_past_key_values()
        leaves = {layer: (k.detach().requires_grad_(True), v.detach().requires_grad_(True))
                  for layer, (k, v) in bank.items()}
        slices, off = [], 0
        for e in self._entries:
            slices.append(PastKVSlice(e.segment.segment_id, off, off + e.segment.length))
            off += e.segment.length
        return PastKVAnchors(MappingProxyType(leaves), tuple(slices), self.segment_ids)

    def accumulate_anchor_gradients(self, anchors: PastKVAnchors) -> None:
        if not isinstance(anchors, PastKVAnchors):
            raise TypeError(f"anchors must be PastKVAnchors, got {type(anchors).__name__}")
        if anchors.stack_signature != self.segment_ids:
            raise RuntimeError(f"past KV anchors are stale: built for {anchors.stack_signature}, "
                               f"current stack is {self.segment_ids}")
        if not self._entries:
            if anchors.key_values or anchors.slices:
                raise RuntimeError("empty stack received non-empty past KV anchors")
            return
        want = self._entries[0].state.layer_numbers
        if tuple(anchors.key_values) != want:
            raise RuntimeError(f"past KV anchor layers must be {want}, got {tuple(anchors.key_values)}")
        for layer, (ka, va) in anchors.key_values.items():
            if ka.grad is None or va.grad is None:
                raise RuntimeError(f"layer {layer} past KV anchor gradient is missing")
            for sl in anchors.slices:
                self.get(sl.segment_id).accumulate(layer, ka.grad[sl.start:sl.end], va.grad[sl.start:sl.end])

    def get_new_kv_gradients(self, segment_id: SegmentId) -> Mapping[int, KVPair]:
        return self.get(segment_id).gradients

    def assert_empty(self) -> None:
        try:
            super().assert_empty()
        except RuntimeError as exc:
            raise RuntimeError(str(exc).replace("prefix-state stack", "KV stack")) from exc

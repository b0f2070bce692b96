"""The KV flavour of the prefix-state stack used by the per-segment executor.

While a segment runs, every attention layer needs the K/V of the whole ancestor path as one
token-major bank ``[P, Hkv, D]`` (root first).  For a graph-free push that bank is just the
concatenation of the ancestors' compact K/V.  For a pop or a leaf visit the bank has to be
differentiable on its own, so :meth:`KVStack.build_past_anchors` materialises it once per layer as
a fresh leaf tensor and remembers how its rows divide among the ancestors; after the backward,
:meth:`KVStack.accumulate_anchor_gradients` splits each leaf's gradient along those row counts
and adds the pieces to the ancestors' dK/dV accumulators.

Anchors are tied to the exact stack they were built from (``stack_signature``), so gradients of a
bank built before a push or pop can never be credited to the wrong segments.

Parity: the KV stack of verl/models/mcore/tpr/kv_stack.py:36-212 (same public types and methods);
the implementation is this framework's own.
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
    """Rows ``[start, end)`` of an anchor bank belong to ``segment_id``."""

    segment_id: SegmentId
    start: int
    end: int


@dataclass(frozen=True, slots=True)
class PastKVAnchors:
    """Differentiable per-layer prefix banks plus their row ownership."""

    key_values: Mapping[int, KVPair]
    slices: tuple[PastKVSlice, ...]
    stack_signature: tuple[SegmentId, ...]

    @property
    def prefix_length(self) -> int:
        return self.slices[-1].end if self.slices else 0


class KVStackEntry(PrefixStateEntry):
    """A stack entry whose prefix state is a :class:`KVPrefixState`."""

    __slots__ = ()

    @property
    def kv(self) -> KVPrefixState:
        st = self.state
        if isinstance(st, KVPrefixState):
            return st
        raise TypeError(f"a KV stack entry holds KVPrefixState, found {type(st).__name__}")

    @property
    def gradients(self) -> Mapping[int, KVPair]:
        return self.kv.gradients

    def accumulate(self, layer_number: int, key_grad: Tensor, value_grad: Tensor) -> None:
        self.kv.accumulate_layer_gradients(layer_number, key_grad, value_grad)


def _kv_signature(state: KVPrefixState) -> tuple:
    """Everything two stacked segments must agree on: layers and per-layer (heads, dim, dtype, device)."""
    return tuple((layer, tuple(k.shape[1:]), k.dtype, k.device) for layer, (k, _) in state.key_values.items())


class KVStack(PrefixStateStack):
    """Graph-free K/V of the active DFS path and the dK/dV relayed to each ancestor."""

    label = "KV stack"

    def top(self) -> KVStackEntry:
        return super().top()  # type: ignore[return-value]

    def get(self, segment_id: SegmentId) -> KVStackEntry:
        return super().get(segment_id)  # type: ignore[return-value]

    def push(self, segment: SegmentSpec, key_values: Mapping[int, KVPair], *,
             shard: SequenceShard | None = None) -> KVStackEntry:
        state = KVPrefixState(segment.segment_id, segment.length, key_values, shard=shard)
        if self._entries:
            have, got = _kv_signature(self._entries[-1].state), _kv_signature(state)
            if have != got:
                raise ValueError(f"segment {segment.segment_id} cannot extend the KV path: its per-layer K/V "
                                 f"layout {got} differs from the ancestors' {have}")
        return self.push_state(segment, state, entry_type=KVStackEntry)  # type: ignore[return-value]

    def pop(self, segment_id: SegmentId) -> KVStackEntry:
        return self.pop_state(segment_id)  # type: ignore[return-value]

    # ------------------------------------------------------------------ banks
    def _layer_banks(self) -> dict[int, KVPair]:
        states = [e.state for e in self._entries]
        if any(st.shard.cp_size != 1 for st in states):
            raise RuntimeError("this path holds context-parallel shards; read it through the CP attention backend")
        banks = {}
        for layer in states[0].layer_numbers:
            pairs = [st.key_values[layer] for st in states]
            if len(pairs) == 1:
                banks[layer] = pairs[0]
            else:
                banks[layer] = (torch.cat([k for k, _ in pairs]), torch.cat([v for _, v in pairs]))
        return banks

    def build_past_key_values(self) -> Mapping[int, KVPair]:
        """Graph-free ancestor banks (views of the stored K/V when the path has one segment)."""
        return MappingProxyType(self._layer_banks() if self._entries else {})

    def build_past_anchors(self) -> PastKVAnchors:
        """Fresh ``requires_grad`` leaf banks for one differentiable forward."""
        if not self._entries:
            return PastKVAnchors(MappingProxyType({}), (), ())
        leaves = {layer: tuple(t.detach().requires_grad_(True) for t in pair)
                  for layer, pair in self._layer_banks().items()}
        ends = torch.tensor([e.segment.length for e in self._entries]).cumsum(0).tolist()
        slices = tuple(PastKVSlice(e.segment.segment_id, end - e.segment.length, end)
                       for e, end in zip(self._entries, ends))
        return PastKVAnchors(MappingProxyType(leaves), slices, self.segment_ids)

    def accumulate_anchor_gradients(self, anchors: PastKVAnchors) -> None:
        """Split every anchor gradient by ancestor and add it to that ancestor's dK/dV."""
        if not isinstance(anchors, PastKVAnchors):
            raise TypeError(f"expected PastKVAnchors, got {type(anchors).__name__}")
        if anchors.stack_signature != self.segment_ids:
            raise RuntimeError(f"anchors describe the path {anchors.stack_signature} but the KV stack now holds "
                               f"{self.segment_ids}")
        if not self._entries:
            if anchors.key_values or anchors.slices:
                raise RuntimeError("anchors carry prefix rows although the KV stack is empty")
            return
        layers = self._entries[0].state.layer_numbers
        if tuple(anchors.key_values) != tuple(layers):
            raise RuntimeError(f"anchor layers {tuple(anchors.key_values)} do not match the stack's {tuple(layers)}")
        sizes = [sl.end - sl.start for sl in anchors.slices]
        owners = [self.get(sl.segment_id) for sl in anchors.slices]
        for layer, (ka, va) in anchors.key_values.items():
            if ka.grad is None or va.grad is None:
                raise RuntimeError(f"layer {layer}: the backward left no gradient on the prefix anchors")
            for owner, dk, dv in zip(owners, ka.grad.split(sizes), va.grad.split(sizes)):
                owner.accumulate(layer, dk, dv)

    def get_new_kv_gradients(self, segment_id: SegmentId) -> Mapping[int, KVPair]:
        return self.get(segment_id).gradients

"""Segment trees and the Push/Pop event protocol the TPR executors follow.

A :class:`SegmentPlan` is host-side metadata: a rooted tree whose nodes are contiguous token
segments.  A child begins at the absolute position where its parent ends, so the external prefix of
any segment is the concatenation of its ancestors.  Executing a plan means walking it with two
kinds of events -- *push* (forward a segment and keep its prefix state for the descendants) and
*pop* (backward it with the gradients its descendants relayed, then drop it).  Any order is legal
as long as it is a depth-first walk: a segment is pushed while its parent is the open segment on
top, and popped only after all of its children were popped.

Internally the plan keeps the tree as a parent map plus ordered child tuples; the canonical walk
(:meth:`SegmentPlan.dfs_events`) is derived from the preorder with depths, and
:meth:`SegmentPlan.validate_events` replays a caller's stream against the open path.

Parity: the public types of verl/models/mcore/tpr/segment_plan.py:36-313 (SegmentLossTerm,
SegmentSpec, SegmentEvent(Kind), Push/PopSegment, SegmentPlan with dfs_events /
validate_events); the implementation and messages are this framework's own.
"""

from __future__ import annotations

import math
from collections.abc import Iterable, Iterator, Mapping, Sequence
from dataclasses import dataclass, field
from enum import Enum
from types import MappingProxyType

import torch
from torch import Tensor

SegmentId = int


def _is_int(value) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


def check_nonneg_int(value, name: str) -> int:
    """``value`` if it is a plain non-negative int (bools rejected), else ``ValueError``."""
    if _is_int(value) and value >= 0:
        return value
    raise ValueError(f"{name}: expected an int >= 0, got {value!r}")


def _finite_number(value) -> bool:
    return isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)


@dataclass(frozen=True, slots=True)
class SegmentLossTerm:
    """A weighted next-token CE term predicted by one query row of a segment.

    Several terms may share a ``query_offset``: the last row of a branching segment predicts the
    first token of each child.
    """

    query_offset: int
    target_token_id: int
    weight: float = 1.0
    sample_id: int | None = None

    def __post_init__(self) -> None:
        check_nonneg_int(self.query_offset, "query_offset")
        check_nonneg_int(self.target_token_id, "target_token_id")
        if not _finite_number(self.weight) or self.weight < 0:
            raise ValueError(f"weight: expected a finite number >= 0, got {self.weight!r}")
        if self.sample_id is not None:
            check_nonneg_int(self.sample_id, "sample_id")


@dataclass(frozen=True, slots=True)
class SegmentSpec:
    """One non-empty contiguous token segment (CPU ``int64`` token ids, privately copied)."""

    segment_id: SegmentId
    parent_id: SegmentId | None
    token_ids: Tensor
    position_start: int
    prefix_length: int
    loss_terms: tuple[SegmentLossTerm, ...] = field(default_factory=tuple)

    def __post_init__(self) -> None:
        for name in ("segment_id", "position_start", "prefix_length"):
            check_nonneg_int(getattr(self, name), name)
        if self.parent_id is not None and check_nonneg_int(self.parent_id, "parent_id") == self.segment_id:
            raise ValueError(f"segment {self.segment_id} names itself as parent")
        tok = self.token_ids
        if not isinstance(tok, Tensor):
            raise TypeError(f"token_ids: expected a torch.Tensor, got {type(tok).__name__}")
        problems = []
        if tok.ndim != 1:
            problems.append(f"{tok.ndim} dims")
        if tok.dtype != torch.long:
            problems.append(f"dtype {tok.dtype}")
        if tok.device.type != "cpu":
            problems.append(f"device {tok.device}")
        if problems:
            raise ValueError("token_ids: expected a 1-D int64 CPU tensor, got " + ", ".join(problems))
        n = int(tok.numel())
        if n == 0:
            raise ValueError(f"segment {self.segment_id} has no tokens")
        if int(tok.min()) < 0:
            raise ValueError(f"segment {self.segment_id} contains a negative token id")
        terms = tuple(self.loss_terms)
        bad = [t for t in terms if not isinstance(t, SegmentLossTerm)]
        if bad:
            raise TypeError(f"loss_terms: expected SegmentLossTerm items, got {type(bad[0]).__name__}")
        late = [t.query_offset for t in terms if t.query_offset >= n]
        if late:
            raise ValueError(f"segment {self.segment_id}: loss term query offset {late[0]} is past its {n} rows")
        object.__setattr__(self, "loss_terms", terms)
        object.__setattr__(self, "token_ids", tok.detach().clone())   # caller mutations cannot leak in

    @property
    def length(self) -> int:
        return int(self.token_ids.numel())

    @property
    def position_end(self) -> int:
        return self.position_start + self.length


class SegmentEventKind(str, Enum):
    PUSH = "push"
    POP = "pop"


@dataclass(frozen=True, slots=True)
class SegmentEvent:
    kind: SegmentEventKind
    segment_id: SegmentId

    def __post_init__(self) -> None:
        if not isinstance(self.kind, SegmentEventKind):
            raise TypeError(f"kind: expected a SegmentEventKind, got {type(self.kind).__name__}")
        check_nonneg_int(self.segment_id, "segment_id")


def PushSegment(segment_id: SegmentId) -> SegmentEvent:  # noqa: N802 (public API name)
    """Event: forward a segment and keep its prefix state for descendants."""
    return SegmentEvent(SegmentEventKind.PUSH, segment_id)


def PopSegment(segment_id: SegmentId) -> SegmentEvent:  # noqa: N802 (public API name)
    """Event: backward a segment (with relayed prefix gradients) and release it."""
    return SegmentEvent(SegmentEventKind.POP, segment_id)


def _index_specs(segments) -> dict[SegmentId, SegmentSpec]:
    items = segments.values() if isinstance(segments, Mapping) else segments
    by_id: dict[SegmentId, SegmentSpec] = {}
    for spec in items:
        if not isinstance(spec, SegmentSpec):
            raise TypeError(f"segments: expected SegmentSpec items, got {type(spec).__name__}")
        if by_id.setdefault(spec.segment_id, spec) is not spec:
            raise ValueError(f"segment id {spec.segment_id} appears twice")
    if not by_id:
        raise ValueError("a segment plan needs at least one segment")
    return by_id


def _check_geometry(by_id: dict[SegmentId, SegmentSpec], root_id: SegmentId) -> None:
    """The root starts at position 0; every other segment starts exactly where its parent ends."""
    for spec in by_id.values():
        if spec.parent_id is None:
            if spec.segment_id != root_id:
                raise ValueError(f"segment {spec.segment_id} has no parent but the root is {root_id}")
            if (spec.prefix_length, spec.position_start) != (0, 0):
                raise ValueError(f"root segment {root_id} must start at position 0 with no prefix, got "
                                 f"position_start={spec.position_start}, prefix_length={spec.prefix_length}")
            continue
        parent = by_id.get(spec.parent_id)
        if parent is None:
            raise ValueError(f"segment {spec.segment_id} refers to parent {spec.parent_id}, which is not in the plan")
        end = parent.position_end
        if spec.position_start != end or spec.prefix_length != end:
            raise ValueError(f"segment {spec.segment_id} starts at position {spec.position_start} with prefix "
                             f"{spec.prefix_length}; its parent {parent.segment_id} ends at {end}")


def _preorder(root_id: SegmentId, children: Mapping[SegmentId, tuple[SegmentId, ...]]) -> list[tuple[SegmentId, int]]:
    """``(segment, depth)`` in preorder (child insertion order), iterative."""
    out: list[tuple[SegmentId, int]] = []
    todo = [(root_id, 0)]
    while todo:
        sid, depth = todo.pop()
        out.append((sid, depth))
        todo.extend((c, depth + 1) for c in reversed(children[sid]))
    return out


@dataclass(frozen=True, slots=True)
class SegmentPlan:
    """Validated rooted segment tree, host metadata only.

    ``topology_only`` plans carry no CE terms: an external objective (PPO) owns the loss and its
    normaliser.
    """

    segments: Mapping[SegmentId, SegmentSpec] | Sequence[SegmentSpec]
    root_id: SegmentId
    total_loss_weight: float | None = None
    topology_only: bool = False
    _children: Mapping[SegmentId, tuple[SegmentId, ...]] = field(init=False, repr=False)

    def __post_init__(self) -> None:
        check_nonneg_int(self.root_id, "root_id")
        by_id = _index_specs(self.segments)
        if self.root_id not in by_id:
            raise ValueError(f"root_id {self.root_id} is not one of the plan's segments")
        _check_geometry(by_id, self.root_id)
        kids: dict[SegmentId, list[SegmentId]] = {sid: [] for sid in by_id}
        for spec in by_id.values():
            if spec.parent_id is not None:
                kids[spec.parent_id].append(spec.segment_id)
        children = {sid: tuple(v) for sid, v in kids.items()}
        # Every segment has one parent and positions grow along edges, so a segment missing from the
        # root's preorder sits in a cycle detached from the root.
        reached = {sid for sid, _ in _preorder(self.root_id, children)}
        if reached != set(by_id):
            raise ValueError(f"segments {sorted(set(by_id) - reached)} cannot be reached from root {self.root_id}")
        has_terms = any(spec.loss_terms for spec in by_id.values())
        if self.topology_only:
            if has_terms or self.total_loss_weight is not None:
                raise ValueError("a topology_only plan describes structure only: it takes no loss terms and no "
                                 "total_loss_weight")
            total = None
        else:
            total = self.total_loss_weight
            if total is None:
                total = sum(t.weight for spec in by_id.values() for t in spec.loss_terms)
            if not _finite_number(total) or total <= 0:
                raise ValueError(f"total_loss_weight: expected a finite number > 0, got {total!r}")
            total = float(total)
        object.__setattr__(self, "segments", MappingProxyType(by_id))
        object.__setattr__(self, "_children", MappingProxyType(children))
        object.__setattr__(self, "total_loss_weight", total)

    # ------------------------------------------------------------------ queries
    def get(self, segment_id: SegmentId) -> SegmentSpec:
        spec = self.segments.get(segment_id)
        if spec is None:
            raise KeyError(f"segment {segment_id} is not in this plan")
        return spec

    def parent_of(self, segment_id: SegmentId) -> SegmentSpec | None:
        pid = self.get(segment_id).parent_id
        return None if pid is None else self.segments[pid]

    def child_ids(self, segment_id: SegmentId) -> tuple[SegmentId, ...]:
        self.get(segment_id)
        return self._children[segment_id]

    def children_of(self, segment_id: SegmentId) -> tuple[SegmentSpec, ...]:
        return tuple(self.segments[c] for c in self.child_ids(segment_id))

    def path_to(self, segment_id: SegmentId) -> tuple[SegmentSpec, ...]:
        """Root-to-``segment_id`` specs."""
        chain = [self.get(segment_id)]
        while chain[-1].parent_id is not None:
            chain.append(self.segments[chain[-1].parent_id])
        chain.reverse()
        return tuple(chain)

    def depth_of(self, segment_id: SegmentId) -> int:
        return len(self.path_to(segment_id)) - 1

    @property
    def total_tokens(self) -> int:
        return sum(s.length for s in self.segments.values())

    # ------------------------------------------------------------------ events
    def dfs_events(self) -> Iterator[SegmentEvent]:
        """Canonical depth-first walk in child insertion order.

        From the preorder with depths: before entering a segment at depth ``d`` every open segment
        at depth ``>= d`` is closed (popped), and the walk ends by closing the remaining path."""
        open_path: list[SegmentId] = []
        for sid, depth in _preorder(self.root_id, self._children):
            while len(open_path) > depth:
                yield PopSegment(open_path.pop())
            yield PushSegment(sid)
            open_path.append(sid)
        while open_path:
            yield PopSegment(open_path.pop())

    def validate_events(self, events: Iterable[SegmentEvent]) -> tuple[SegmentEvent, ...]:
        """Replay ``events`` against the open path; return them as a tuple if they form a complete
        depth-first walk of this plan (every segment pushed and popped exactly once)."""
        seq = tuple(events)
        open_path: list[SegmentId] = []
        state: dict[SegmentId, str] = {}                                 # "open" | "closed"
        unfinished = {sid: len(c) for sid, c in self._children.items()}  # children not yet closed
        for i, ev in enumerate(seq):
            if not isinstance(ev, SegmentEvent):
                raise TypeError(f"event {i}: expected a SegmentEvent, got {type(ev).__name__}")
            spec = self.get(ev.segment_id)
            sid = ev.segment_id
            if ev.kind is SegmentEventKind.PUSH:
                if sid in state:
                    raise ValueError(f"event {i}: segment {sid} was already pushed")
                on_top = open_path[-1] if open_path else None
                if on_top != spec.parent_id:
                    raise ValueError(f"event {i}: push of segment {sid} needs its parent {spec.parent_id} on top "
                                     f"of the open path, found {on_top}")
                open_path.append(sid)
                state[sid] = "open"
                continue
            if not open_path or open_path[-1] != sid:
                raise ValueError(f"event {i}: pop of segment {sid} while the open path is {open_path}")
            if unfinished[sid]:
                raise ValueError(f"event {i}: segment {sid} still has {unfinished[sid]} child(ren) to pop")
            open_path.pop()
            state[sid] = "closed"
            if spec.parent_id is not None:
                unfinished[spec.parent_id] -= 1
        missing = sorted(sid for sid in self.segments if state.get(sid) != "closed")
        if open_path or missing:
            raise ValueError(f"the event stream ends early: open path {open_path}, segments not completed "
                             f"{missing}")
        return seq

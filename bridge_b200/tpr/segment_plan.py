"""Immutable segment topology and its Push/Pop event protocol.

A :class:`SegmentPlan` is a rooted tree of token segments kept entirely on the
host. Every child starts exactly where its parent ends, so a segment's absolute
positions are ``[prefix_length, prefix_length + length)`` and its external
prefix is the concatenation of its ancestors. The plan yields a deterministic
DFS Push/Pop stream and validates arbitrary streams against stack discipline.

Parity: verl/models/mcore/tpr/segment_plan.py:36-313 (SegmentLossTerm,
SegmentSpec, SegmentEvent, SegmentPlan.dfs_events / validate_events).
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
    if not _is_int(value) or value < 0:
        raise ValueError(f"{name} must be a non-negative integer, got {value!r}")
    return value


@dataclass(frozen=True, slots=True)
class SegmentLossTerm:
    """A weighted next-token CE term predicted by one query row of a segment.

    Several terms may share a ``query_offset``: the last row of a branching
    segment predicts the first token of each child.
    """

    query_offset: int
    target_token_id: int
    weight: float = 1.0
    sample_id: int | None = None

    def __post_init__(self) -> None:
        check_nonneg_int(self.query_offset, "query_offset")
        check_nonneg_int(self.target_token_id, "target_token_id")
        if isinstance(self.weight, bool) or not isinstance(self.weight, (int, float)):
            raise ValueError(f"weight must be a finite number, got {self.weight!r}")
        if not math.isfinite(self.weight) or self.weight < 0:
            raise ValueError(f"weight must be finite and non-negative, got {self.weight!r}")
        if self.sample_id is not None:
            check_nonneg_int(self.sample_id, "sample_id")


@dataclass(frozen=True, slots=True)
class SegmentSpec:
    """One non-empty contiguous token segment (CPU ``int64`` token ids)."""

    segment_id: SegmentId
    parent_id: SegmentId | None
    token_ids: Tensor
    position_start: int
    prefix_length: int
    loss_terms: tuple[SegmentLossTerm, ...] = field(default_factory=tuple)

    def __post_init__(self) -> None:
        check_nonneg_int(self.segment_id, "segment_id")
        if self.parent_id is not None:
            check_nonneg_int(self.parent_id, "parent_id")
            if self.parent_id == self.segment_id:
                raise ValueError(f"segment {self.segment_id} cannot be its own parent")
        tok = self.token_ids
        if not isinstance(tok, Tensor):
            raise TypeError("token_ids must be a torch.Tensor")
        if tok.device.type != "cpu" or tok.dtype != torch.long or tok.ndim != 1:
            raise ValueError(
                "token_ids must be a 1-D CPU torch.long tensor, got "
                f"shape={tuple(tok.shape)} dtype={tok.dtype} device={tok.device}"
            )
        if tok.numel() == 0:
            raise ValueError("token_ids must contain at least one token")
        if bool((tok < 0).any()):
            raise ValueError("token_ids must be non-negative")
        check_nonneg_int(self.position_start, "position_start")
        check_nonneg_int(self.prefix_length, "prefix_length")
        terms = tuple(self.loss_terms)
        for term in terms:
            if not isinstance(term, SegmentLossTerm):
                raise TypeError(f"loss_terms must hold SegmentLossTerm, got {type(term).__name__}")
            if term.query_offset >= tok.numel():
                raise ValueError(
                    f"segment {self.segment_id} loss query_offset {term.query_offset} "
                    f"is outside length {tok.numel()}"
                )
        object.__setattr__(self, "loss_terms", terms)
        # The plan owns a private copy: later caller mutation cannot leak in.
        object.__setattr__(self, "token_ids", tok.detach().clone())

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
            raise TypeError(f"kind must be SegmentEventKind, got {type(self.kind).__name__}")
        check_nonneg_int(self.segment_id, "segment_id")


def PushSegment(segment_id: SegmentId) -> SegmentEvent:  # noqa: N802 (public API name)
    """Event: forward a segment and keep its prefix state for descendants."""
    return SegmentEvent(SegmentEventKind.PUSH, segment_id)


def PopSegment(segment_id: SegmentId) -> SegmentEvent:  # noqa: N802 (public API name)
    """Event: backward a segment (with relayed prefix gradients) and release it."""
    return SegmentEvent(SegmentEventKind.POP, segment_id)


@dataclass(frozen=True, slots=True)
class SegmentPlan:
    """Validated rooted segment tree, host metadata only.

    ``topology_only`` plans carry no CE terms: an external objective (PPO)
    owns the loss and its normaliser.
    """

    segments: Mapping[SegmentId, SegmentSpec] | Sequence[SegmentSpec]
    root_id: SegmentId
    total_loss_weight: float | None = None
    topology_only: bool = False
    _children: Mapping[SegmentId, tuple[SegmentId, ...]] = field(init=False, repr=False)

    def __post_init__(self) -> None:
        check_nonneg_int(self.root_id, "root_id")
        items = self.segments.values() if isinstance(self.segments, Mapping) else self.segments
        by_id: dict[SegmentId, SegmentSpec] = {}
        for spec in items:
            if not isinstance(spec, SegmentSpec):
                raise TypeError(f"segments must hold SegmentSpec, got {type(spec).__name__}")
            if spec.segment_id in by_id:
                raise ValueError(f"duplicate segment_id {spec.segment_id}")
            by_id[spec.segment_id] = spec
        if not by_id:
            raise ValueError("segments must not be empty")
        if self.root_id not in by_id:
            raise ValueError(f"root_id {self.root_id} does not exist")
        roots = sorted(s.segment_id for s in by_id.values() if s.parent_id is None)
        if roots != [self.root_id]:
            raise ValueError(f"plan must have exactly root {self.root_id}, got roots={roots}")

        children: dict[SegmentId, list[SegmentId]] = {sid: [] for sid in by_id}
        for spec in by_id.values():
            if spec.parent_id is None:
                if spec.prefix_length != 0 or spec.position_start != 0:
                    raise ValueError("root segment must have prefix_length=0 and position_start=0")
                continue
            parent = by_id.get(spec.parent_id)
            if parent is None:
                raise ValueError(f"segment {spec.segment_id} has missing parent {spec.parent_id}")
            if spec.prefix_length != parent.position_end or spec.position_start != parent.position_end:
                raise ValueError(
                    f"segment {spec.segment_id} must start at parent {parent.segment_id} end "
                    f"{parent.position_end}, got prefix_length={spec.prefix_length}, "
                    f"position_start={spec.position_start}"
                )
            children[spec.parent_id].append(spec.segment_id)

        # Reachability (the position rule already excludes cycles through the root,
        # but a detached cycle of non-root segments must still be rejected).
        seen: set[SegmentId] = set()
        stack = [self.root_id]
        while stack:
            sid = stack.pop()
            if sid in seen:
                raise ValueError(f"cycle detected at segment {sid}")
            seen.add(sid)
            stack.extend(children[sid])
        if seen != set(by_id):
            raise ValueError(f"segments are not reachable from root: {sorted(set(by_id) - seen)}")

        inferred = sum(t.weight for s in by_id.values() for t in s.loss_terms)
        if self.topology_only:
            if any(s.loss_terms for s in by_id.values()) or self.total_loss_weight is not None:
                raise ValueError("topology_only plans must not carry CE loss terms or total_loss_weight")
            total = None
        else:
            total = inferred if self.total_loss_weight is None else self.total_loss_weight
            if (
                isinstance(total, bool)
                or not isinstance(total, (int, float))
                or not math.isfinite(total)
                or total <= 0
            ):
                raise ValueError(f"total_loss_weight must be finite and positive, got {total!r}")
            total = float(total)
        object.__setattr__(self, "segments", MappingProxyType(by_id))
        object.__setattr__(self, "_children", MappingProxyType({k: tuple(v) for k, v in children.items()}))
        object.__setattr__(self, "total_loss_weight", total)

    # ------------------------------------------------------------------ queries
    def get(self, segment_id: SegmentId) -> SegmentSpec:
        try:
            return self.segments[segment_id]
        except KeyError as exc:
            raise KeyError(f"unknown segment_id {segment_id}") from exc

    def parent_of(self, segment_id: SegmentId) -> SegmentSpec | None:
        spec = self.get(segment_id)
        return None if spec.parent_id is None else self.segments[spec.parent_id]

    def children_of(self, segment_id: SegmentId) -> tuple[SegmentSpec, ...]:
        self.get(segment_id)
        return tuple(self.segments[c] for c in self._children[segment_id])

    def child_ids(self, segment_id: SegmentId) -> tuple[SegmentId, ...]:
        self.get(segment_id)
        return self._children[segment_id]

    def path_to(self, segment_id: SegmentId) -> tuple[SegmentSpec, ...]:
        path = []
        spec: SegmentSpec | None = self.get(segment_id)
        while spec is not None:
            path.append(spec)
            spec = None if spec.parent_id is None else self.segments[spec.parent_id]
        return tuple(reversed(path))

    def depth_of(self, segment_id: SegmentId) -> int:
        return len(self.path_to(segment_id)) - 1

    @property
    def total_tokens(self) -> int:
        return sum(s.length for s in self.segments.values())

    # ------------------------------------------------------------------ events
    def dfs_events(self) -> Iterator[SegmentEvent]:
        """Deterministic DFS in child insertion order (iterative, no recursion limit)."""
        stack: list[tuple[SegmentId, bool]] = [(self.root_id, False)]
        while stack:
            sid, done = stack.pop()
            if done:
                yield PopSegment(sid)
                continue
            yield PushSegment(sid)
            stack.append((sid, True))
            for child in reversed(self._children[sid]):
                stack.append((child, False))

    def validate_events(self, events: Iterable[SegmentEvent]) -> tuple[SegmentEvent, ...]:
        """Check stack discipline and that every segment is pushed and popped once."""
        seq = tuple(events)
        stack: list[SegmentId] = []
        pushed: set[SegmentId] = set()
        popped: set[SegmentId] = set()
        for ev in seq:
            if not isinstance(ev, SegmentEvent):
                raise TypeError(f"events must hold SegmentEvent, got {type(ev).__name__}")
            spec = self.get(ev.segment_id)
            if ev.kind is SegmentEventKind.PUSH:
                if ev.segment_id in pushed:
                    raise ValueError(f"segment {ev.segment_id} is pushed more than once")
                top = stack[-1] if stack else None
                if spec.parent_id != top:
                    raise ValueError(
                        f"cannot push segment {ev.segment_id}: expected parent on stack "
                        f"{spec.parent_id}, got {top}"
                    )
                stack.append(ev.segment_id)
                pushed.add(ev.segment_id)
            else:
                if not stack or stack[-1] != ev.segment_id:
                    raise ValueError(f"cannot pop segment {ev.segment_id}: current stack is {stack}")
                if any(c not in popped for c in self._children[ev.segment_id]):
                    raise ValueError(f"cannot pop segment {ev.segment_id} before all children")
                stack.pop()
                popped.add(ev.segment_id)
        every = set(self.segments)
        if stack or pushed != every or popped != every:
            raise ValueError(
                f"incomplete event stream: stack={stack}, unpushed={sorted(every - pushed)}, "
                f"unpopped={sorted(every - popped)}"
            )
        return seq

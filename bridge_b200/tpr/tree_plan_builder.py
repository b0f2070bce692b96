"""Lower trajectory tries to executable plans plus logical PPO token references.

``response_mask`` is right-aligned with ``input_ids`` (prompt + response).  The
token at absolute position ``t`` is predicted by the query row ``t - 1``, which
may sit in the *parent* segment when ``t`` is the first token of a child.  Every
supervised logical token maps to exactly one :class:`SegmentObjectiveRef`;
duplicate trajectories keep separate refs.

Parity: verl/models/mcore/tpr/tree_plan_builder.py:21-212.
"""

from __future__ import annotations

from bisect import bisect_right
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from .segment_plan import SegmentPlan, SegmentSpec
from .trajectory_tree import TrajectoryTree, build_trajectory_trees


@dataclass(frozen=True, slots=True)
class SegmentObjectiveRef:
    segment_id: int
    query_offset: int
    target_token_id: int
    sample_row: int
    response_offset: int


class ObjectiveRefs(Sequence):
    """Immutable sequence of :class:`SegmentObjectiveRef` stored as int64 columns ``[n, 5]``
    ``(segment_id, query_offset, target_token_id, sample_row, response_offset)``; ref objects are
    built only when indexed or iterated, and ``columns`` feeds the vectorised consumers directly."""

    __slots__ = ("columns",)

    def __init__(self, columns: np.ndarray) -> None:
        cols = np.ascontiguousarray(columns, dtype=np.int64).reshape(-1, 5)
        cols.setflags(write=False)
        self.columns = cols

    def __len__(self) -> int:
        return self.columns.shape[0]

    def __getitem__(self, i):
        if isinstance(i, slice):
            return ObjectiveRefs(self.columns[i])
        a = self.columns[i]
        return SegmentObjectiveRef(int(a[0]), int(a[1]), int(a[2]), int(a[3]), int(a[4]))

    def __iter__(self):
        for a in self.columns.tolist():
            yield SegmentObjectiveRef(*a)

    def __eq__(self, other) -> bool:
        if isinstance(other, ObjectiveRefs):
            return bool(np.array_equal(self.columns, other.columns))
        return tuple(self) == tuple(other)

    def __hash__(self) -> int:
        return hash(self.columns.tobytes())

    def __repr__(self) -> str:
        return f"ObjectiveRefs(n={len(self)})"


@dataclass(frozen=True, slots=True)
class TreeExecutionPlan:
    tree: TrajectoryTree
    segment_plan: SegmentPlan
    objective_refs: tuple[SegmentObjectiveRef, ...]

    def refs_for_segment(self, segment_id: int) -> tuple[SegmentObjectiveRef, ...]:
        self.segment_plan.get(segment_id)
        cols = getattr(self.objective_refs, "columns", None)
        if cols is not None:
            return tuple(ObjectiveRefs(cols[cols[:, 0] == segment_id]))
        return tuple(r for r in self.objective_refs if r.segment_id == segment_id)

    @property
    def logical_loss_tokens(self) -> int:
        return len(self.objective_refs)


@dataclass(frozen=True, slots=True)
class ForestExecutionPlan:
    trees: tuple[TreeExecutionPlan, ...]
    logical_loss_tokens: int

    def __post_init__(self) -> None:
        if sum(t.logical_loss_tokens for t in self.trees) != self.logical_loss_tokens:
            raise ValueError("forest logical_loss_tokens disagrees with objective refs")

    @property
    def segment_count(self) -> int:
        return sum(len(t.segment_plan.segments) for t in self.trees)

    @property
    def unique_tokens(self) -> int:
        return sum(t.segment_plan.total_tokens for t in self.trees)


def _tensor_rows(batch: Any, key: str) -> list[torch.Tensor]:
    try:
        value = batch[key]
    except (KeyError, TypeError) as exc:
        raise ValueError(f"batch is missing {key!r}") from exc
    rows = list(value) if isinstance(value, (list, tuple)) else list(value.unbind())
    if not all(isinstance(r, torch.Tensor) and r.ndim == 1 for r in rows):
        raise ValueError(f"{key!r} must contain one-dimensional tensor rows")
    return rows


def _has(batch: Any, key: str) -> bool:
    try:
        return key in batch
    except TypeError:
        return False


def build_tree_execution_plans(
    keys,
    batch: Any,
    *,
    trees: tuple[TrajectoryTree, ...] | None = None,
    require_loss_mask_alignment: bool = False,
    tree_policy: str = "exact",
    turn_min_segment_tokens: int = 128,
) -> ForestExecutionPlan:
    """Build topology-only SegmentPlans and PPO ownership refs for a mini-batch."""
    if tree_policy not in ("exact", "qwen_turn"):
        raise ValueError(f"unknown TPR tree_policy: {tree_policy!r}")
    keys = list(keys)
    if trees is None:
        if tree_policy == "qwen_turn":
            from .trajectory_tree_turn import build_trajectory_trees_turn

            trees = build_trajectory_trees_turn(keys, batch, min_segment_tokens=turn_min_segment_tokens)
        else:
            trees = build_trajectory_trees(keys, batch)
    inputs = _tensor_rows(batch, "input_ids")
    masks = _tensor_rows(batch, "response_mask")
    if len(keys) != len(inputs) or len(keys) != len(masks):
        raise ValueError("keys, input_ids and response_mask must have identical row counts")
    responses = _tensor_rows(batch, "responses") if _has(batch, "responses") else None

    supervised: list[np.ndarray] = []
    expected = 0
    for row, (tokens, mask) in enumerate(zip(inputs, masks)):
        if mask.numel() > tokens.numel():
            raise ValueError(f"response_mask[{row}] is longer than input_ids[{row}]")
        if responses is not None:
            resp = responses[row]
            if resp.numel() != mask.numel():
                raise ValueError(f"responses/response_mask length mismatch on row {row}")
            if not torch.equal(tokens[tokens.numel() - resp.numel():].cpu(), resp.cpu()):
                raise ValueError(f"response is not an input_ids suffix on row {row}")
        offs = np.flatnonzero(mask.detach().to(torch.bool).cpu().numpy()).astype(np.int64)
        if offs.size and tokens.numel() - mask.numel() + int(offs[0]) == 0:
            raise ValueError(f"row {row} has no preceding query token for first supervised token")
        supervised.append(offs)
        expected += int(offs.size)

    if require_loss_mask_alignment:
        loss_masks = _tensor_rows(batch, "loss_mask")
        if len(loss_masks) != len(keys):
            raise ValueError("loss_mask rows do not match keys")
        for row, (lm, rm) in enumerate(zip(loss_masks, masks)):
            if lm.numel() == rm.numel():
                aligned = lm
            elif lm.numel() == inputs[row].numel():
                aligned = lm[lm.numel() - rm.numel():]
                if bool(lm[: lm.numel() - rm.numel()].to(torch.bool).any()):
                    raise ValueError(f"row {row} loss_mask includes prompt tokens")
            else:
                raise ValueError(f"row {row} loss_mask shape is incompatible with response_mask")
            if not torch.equal(aligned.to(torch.bool).cpu(), rm.to(torch.bool).cpu()):
                raise ValueError(f"row {row} response_mask and loss_mask disagree")

    consumed: set[int] = set()
    plans: list[TreeExecutionPlan] = []
    for tree in trees:
        specs = []
        for node in tree.nodes.values():
            ref = node.segment
            ids = inputs[ref.row][ref.start:ref.end].detach().to("cpu", torch.long)
            specs.append(SegmentSpec(segment_id=node.node_id, parent_id=node.parent_id, token_ids=ids,
                                     position_start=ref.start, prefix_length=ref.start))
        plan = SegmentPlan(specs, root_id=tree.root_id, topology_only=True)

        # Root-to-terminal path of every member row.
        path_of: dict[int, tuple[int, ...]] = {}
        stack = [(tree.root_id, ())]
        while stack:
            nid, path = stack.pop()
            node = tree.get(nid)
            here = (*path, nid)
            for row in node.terminal_rows:
                if row in path_of:
                    raise ValueError(f"trajectory row {row} has multiple terminal nodes")
                path_of[row] = here
            stack.extend((c, here) for c in node.children)
        if set(path_of) != set(tree.member_rows):
            raise ValueError(f"tree {tree.key} terminal rows do not cover members")

        # ownership search, vectorised per row: token t (response offset `off`) is predicted by query
        # q = t - 1, owned by the first node on the row's root-to-terminal path whose end exceeds q
        parts: list[np.ndarray] = []
        for row in tree.member_rows:
            if row in consumed:
                raise ValueError(f"row {row} appears in more than one tree")
            consumed.add(row)
            off = supervised[row]
            if not off.size:
                continue
            ids = inputs[row]
            resp_start = ids.numel() - masks[row].numel()
            path = np.asarray(path_of[row], dtype=np.int64)
            segs = [tree.get(int(n)).segment for n in path]
            ends = np.asarray([sg.end for sg in segs], dtype=np.int64)
            starts = np.asarray([sg.start for sg in segs], dtype=np.int64)
            t = resp_start + off
            q = t - 1
            k = np.searchsorted(ends, q, side="right")
            if bool((k >= len(path)).any()):
                raise ValueError(f"row {row} query position {int(q[k >= len(path)][0])} is outside tree")
            if not bool(((starts[k] <= q) & (q < ends[k])).all()):
                raise ValueError(f"row {row} has uncovered query positions")
            targets = ids.detach().cpu().numpy().astype(np.int64)[t]
            parts.append(np.stack([path[k], q - starts[k], targets, np.full_like(off, row), off], axis=1))
        refs = ObjectiveRefs(np.concatenate(parts) if parts else np.zeros((0, 5), dtype=np.int64))
        plans.append(TreeExecutionPlan(tree=tree, segment_plan=plan, objective_refs=refs))

    if consumed != set(range(len(keys))):
        raise ValueError(f"forest does not cover all input rows: {sorted(set(range(len(keys))) - consumed)}")
    return ForestExecutionPlan(tuple(plans), logical_loss_tokens=expected)

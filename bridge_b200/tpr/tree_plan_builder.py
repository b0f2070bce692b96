"""Lower trajectory tries to executable plans plus logical PPO token references.

``response_mask`` is right-aligned with ``input_ids`` (prompt + response).  The
token at absolute position ``t`` is predicted by the query row ``t - 1``, which
may sit in the *parent* segment when ``t`` is the first token of a child.  Every
supervised logical token maps to exactly one :class:`SegmentObjectiveRef`;
duplicate trajectories keep separate refs.

Lowering runs in three stages: per-row supervised offsets (with the optional loss-mask check),
one topology-only :class:`SegmentPlan` per trie, and a vectorised ownership search per row over
the row's root-to-terminal node chain (found by walking parent links up from the terminal node).

Parity: the data contract of verl/models/mcore/tpr/tree_plan_builder.py:21-212 (same public types,
same batch fields and the same ownership rule); the implementation is this framework's own.
"""

from __future__ import annotations

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
    """Rows of ``batch[key]`` as 1-D tensors (a list/tuple of rows or a tensor split along dim 0)."""
    try:
        value = batch[key]
    except (KeyError, TypeError) as exc:
        raise ValueError(f"the mini-batch has no {key!r} field") from exc
    rows = list(value) if isinstance(value, (list, tuple)) else list(value.unbind())
    odd = next((i for i, r in enumerate(rows) if not (isinstance(r, torch.Tensor) and r.ndim == 1)), None)
    if odd is not None:
        raise ValueError(f"{key}[{odd}] is not a 1-D tensor")
    return rows


def _has(batch: Any, key: str) -> bool:
    try:
        return key in batch
    except TypeError:
        return False


def _supervised_offsets(inputs, masks, responses) -> list[np.ndarray]:
    """Per row: response offsets whose mask is set (the tokens that carry a PPO term)."""
    out = []
    for row, (tokens, mask) in enumerate(zip(inputs, masks)):
        n_tok, n_resp = tokens.numel(), mask.numel()
        if n_resp > n_tok:
            raise ValueError(f"row {row}: response_mask has {n_resp} entries for only {n_tok} input tokens")
        if responses is not None:
            resp = responses[row]
            if resp.numel() != n_resp:
                raise ValueError(f"row {row}: responses has {resp.numel()} tokens, response_mask {n_resp}")
            if not torch.equal(tokens[n_tok - n_resp:].cpu(), resp.cpu()):
                raise ValueError(f"row {row}: responses differ from the tail of input_ids")
        offs = np.flatnonzero(mask.detach().to(torch.bool).cpu().numpy()).astype(np.int64)
        if offs.size and n_tok - n_resp + int(offs[0]) == 0:
            raise ValueError(f"row {row}: token 0 is supervised, but no earlier token can predict it")
        out.append(offs)
    return out


def _check_loss_mask(batch, inputs, masks) -> None:
    """``loss_mask`` (response-aligned or full-length) must select exactly the response-mask tokens."""
    lms = _tensor_rows(batch, "loss_mask")
    if len(lms) != len(masks):
        raise ValueError(f"loss_mask has {len(lms)} rows, response_mask {len(masks)}")
    for row, (lm, rm) in enumerate(zip(lms, masks)):
        lm, rm = lm.to(torch.bool).cpu(), rm.to(torch.bool).cpu()
        n_prompt = inputs[row].numel() - rm.numel()
        if lm.numel() == inputs[row].numel() and lm.numel() != rm.numel():
            if bool(lm[:n_prompt].any()):
                raise ValueError(f"row {row}: loss_mask selects prompt tokens")
            lm = lm[n_prompt:]
        if lm.numel() != rm.numel():
            raise ValueError(f"row {row}: loss_mask length {lm.numel()} fits neither the response "
                             f"({rm.numel()}) nor the whole row ({inputs[row].numel()})")
        if not torch.equal(lm, rm):
            raise ValueError(f"row {row}: loss_mask and response_mask select different tokens")


def _tree_segment_plan(tree: TrajectoryTree, inputs) -> SegmentPlan:
    specs = []
    for node in tree.nodes.values():
        ref = node.segment
        ids = inputs[ref.row][ref.start:ref.end].detach().to("cpu", torch.long)
        specs.append(SegmentSpec(segment_id=node.node_id, parent_id=node.parent_id, token_ids=ids,
                                 position_start=ref.start, prefix_length=ref.start))
    return SegmentPlan(specs, root_id=tree.root_id, topology_only=True)


def _row_chains(tree: TrajectoryTree) -> dict[int, tuple[np.ndarray, np.ndarray]]:
    """Member row -> (node ids from the root down to the node where the row ends, their [start, end)
    token spans); rows ending at the same node share both arrays."""
    chains: dict[int, tuple[np.ndarray, np.ndarray]] = {}
    for node in tree.nodes.values():
        if not node.terminal_rows:
            continue
        up = [node.node_id]
        while tree.get(up[-1]).parent_id is not None:
            up.append(tree.get(up[-1]).parent_id)
        ids = up[::-1]
        chain = np.asarray(ids, dtype=np.int64)
        spans = np.asarray([(tree.get(n).segment.start, tree.get(n).segment.end) for n in ids],
                           dtype=np.int64).reshape(-1, 2)
        for row in node.terminal_rows:
            if row in chains:
                raise ValueError(f"tree {tree.key}: row {row} ends at two different nodes")
            chains[row] = (chain, spans)
    if set(chains) != set(tree.member_rows):
        raise ValueError(f"tree {tree.key}: rows {sorted(set(tree.member_rows) - set(chains))} end at no node")
    return chains


def _row_refs(tree: TrajectoryTree, chain_spans: tuple[np.ndarray, np.ndarray], row: int, tokens, n_resp: int,
              off: np.ndarray) -> np.ndarray:
    """Ref columns of one row: the token at response offset ``off`` (absolute position ``t``) is
    predicted by query ``t - 1``, owned by the first node of the chain whose span contains it."""
    chain, spans = chain_spans
    t = tokens.numel() - n_resp + off
    q = t - 1
    k = np.searchsorted(spans[:, 1], q, side="right")
    outside = k >= len(chain)
    if bool(outside.any()):
        raise ValueError(f"row {row}: query position {int(q[outside][0])} lies past the row's last node")
    kk = np.minimum(k, len(chain) - 1)
    if not bool((spans[kk, 0] <= q).all()):
        raise ValueError(f"row {row}: a query position falls between node spans")
    targets = tokens.detach().cpu().numpy()[t].astype(np.int64, copy=False)
    out = np.empty((off.size, 5), dtype=np.int64)
    out[:, 0] = chain[k]
    out[:, 1] = q - spans[k, 0]
    out[:, 2] = targets
    out[:, 3] = row
    out[:, 4] = off
    return out


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
    if not len(keys) == len(inputs) == len(masks):
        raise ValueError(f"row counts differ: {len(keys)} keys, {len(inputs)} input_ids, {len(masks)} response_mask")
    responses = _tensor_rows(batch, "responses") if _has(batch, "responses") else None
    supervised = _supervised_offsets(inputs, masks, responses)
    if require_loss_mask_alignment:
        _check_loss_mask(batch, inputs, masks)

    owner_tree: dict[int, int] = {}
    plans: list[TreeExecutionPlan] = []
    for ti, tree in enumerate(trees):
        chains = _row_chains(tree)
        parts = []
        for row in tree.member_rows:
            if owner_tree.setdefault(row, ti) != ti:
                raise ValueError(f"row {row} belongs to trees {owner_tree[row]} and {ti}")
            if supervised[row].size:
                parts.append(_row_refs(tree, chains[row], row, inputs[row], masks[row].numel(), supervised[row]))
        refs = ObjectiveRefs(np.concatenate(parts) if parts else np.zeros((0, 5), dtype=np.int64))
        plans.append(TreeExecutionPlan(tree=tree, segment_plan=_tree_segment_plan(tree, inputs), objective_refs=refs))
    orphans = sorted(set(range(len(keys))) - set(owner_tree))
    if orphans:
        raise ValueError(f"rows {orphans} are in no tree")
    return ForestExecutionPlan(tuple(plans), logical_loss_tokens=sum(int(o.size) for o in supervised))

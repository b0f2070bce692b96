"""Token-exact compressed tries over the rows of one training batch.

Rows are grouped by the ``uid`` part of their trajectory key
(``"<uid>_<x>_<index>"``, split from the right).  Within a group the rows form
a radix tree built by longest-common-prefix partitioning: a node spans the
tokens every member shares, rows that end there are *terminal*, and the
remaining rows are split by their next token (first-appearance order).  Each
first-token branch becomes its own executable :class:`TrajectoryTree` whose
root starts at absolute position 0.  Nodes keep zero-copy ``(row, start, end)``
references into the batch.

Parity: verl/models/mcore/tpr/trajectory_tree.py:26-301 (SegmentRef,
TrajectoryNode, TrajectoryTree, build_trajectory_trees; the key format and the
node-id numbering -- pre-order, children in first-appearance order -- are kept
identical so plans digest the same on both sides).
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Mapping

import numpy as np
import torch

from .segment_plan import _is_int


def _need(ok: bool, message: str) -> None:
    if not ok:
        raise ValueError(message)


@dataclass(frozen=True, slots=True)
class SegmentRef:
    """Zero-copy reference ``input_ids[row][start:end]`` (``end > start``)."""

    row: int
    start: int
    end: int

    def __post_init__(self) -> None:
        for name in ("row", "start", "end"):
            v = getattr(self, name)
            _need(_is_int(v) and v >= 0, f"SegmentRef.{name}: expected an int >= 0, got {v!r}")
        _need(self.end > self.start, f"SegmentRef [{self.start}, {self.end}) is empty")

    @property
    def length(self) -> int:
        return self.end - self.start


@dataclass(frozen=True, slots=True)
class TrajectoryNode:
    """One trie node: the token span its member rows share, the rows that end here, its children."""

    node_id: int
    parent_id: int | None
    segment: SegmentRef
    member_rows: tuple[int, ...]
    terminal_rows: tuple[int, ...]
    children: tuple[int, ...]

    def __post_init__(self) -> None:
        nid = self.node_id
        _need(_is_int(nid) and nid >= 0, f"node_id: expected an int >= 0, got {nid!r}")
        if self.parent_id is not None:
            _need(_is_int(self.parent_id) and self.parent_id >= 0 and self.parent_id != nid,
                  f"trie node {nid}: parent_id {self.parent_id!r} is not another node's id")
        members = set(self.member_rows)
        _need(len(members) == len(self.member_rows) > 0,
              f"trie node {nid}: member_rows must be distinct and non-empty, got {self.member_rows}")
        _need(members.issuperset(self.terminal_rows),
              f"trie node {nid}: terminal rows {sorted(set(self.terminal_rows) - members)} are not members")


@dataclass(frozen=True, slots=True)
class TrajectoryTree:
    """One executable compressed trie whose root starts at position 0."""

    uid: str
    tree_index: int
    root_id: int
    member_rows: tuple[int, ...]
    nodes: Mapping[int, TrajectoryNode]

    def __post_init__(self) -> None:
        table = dict(self.nodes)
        _need(all(k == n.node_id for k, n in table.items()), "trie nodes must be keyed by their node_id")
        root = table.get(self.root_id)
        _need(root is not None, f"trie root {self.root_id} is not among the nodes")
        _need(root.parent_id is None and root.segment.start == 0,
              f"trie root {self.root_id} must be parentless and begin at token 0")
        _need(tuple(root.member_rows) == tuple(self.member_rows),
              f"tree rows {self.member_rows} differ from its root's rows {root.member_rows}")
        # Edges must agree from both ends, and each child continues where its parent stops.
        for nid, node in table.items():
            _need(node.parent_id is None or node.parent_id in table,
                  f"trie node {nid} points at parent {node.parent_id}, which is not in the tree")
            for cid in node.children:
                child = table.get(cid)
                _need(child is not None and child.parent_id == nid,
                      f"trie node {nid} lists child {cid}, which does not name {nid} as its parent")
                _need(child.segment.start == node.segment.end,
                      f"trie node {cid} begins at token {child.segment.start}, not where its parent {nid} "
                      f"ends ({node.segment.end})")
        object.__setattr__(self, "nodes", MappingProxyType(table))

    @property
    def key(self) -> str:
        return f"{self.uid}:{self.tree_index}"

    def get(self, node_id: int) -> TrajectoryNode:
        node = self.nodes.get(node_id)
        if node is None:
            raise KeyError(f"trie {self.key} has no node {node_id}")
        return node

    @property
    def unique_tokens(self) -> int:
        return sum(n.segment.length for n in self.nodes.values())


# --------------------------------------------------------------------------- batch access
def batch_rows(batch: Any, name: str) -> list[Any]:
    """Row-wise view of ``batch[name]`` (list/tuple, or anything with ``unbind``)."""
    try:
        value = batch[name]
    except Exception as exc:  # TensorDict raises KeyError, dict KeyError, others vary
        raise ValueError(f"training batch is missing required field {name!r}") from exc
    if isinstance(value, (list, tuple)):
        return list(value)
    unbind = getattr(value, "unbind", None)
    if callable(unbind):
        return list(unbind())
    raise TypeError(f"field {name!r} does not expose row-wise values: {type(value)!r}")


def as_token_row(value: Any, *, row: int) -> torch.Tensor:
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"input_ids[{row}] must be a torch.Tensor, got {type(value)!r}")
    if value.ndim != 1:
        raise ValueError(f"input_ids[{row}] must be 1-D, got shape={tuple(value.shape)}")
    if value.numel() == 0:
        raise ValueError(f"input_ids[{row}] must not be empty")
    if value.dtype == torch.bool or torch.is_floating_point(value) or torch.is_complex(value):
        raise ValueError(f"input_ids[{row}] must use an integer dtype, got {value.dtype}")
    if bool((value < 0).any()):
        raise ValueError(f"input_ids[{row}] must contain non-negative token ids")
    return value


def parse_trajectory_key(key: str) -> tuple[str, str, int]:
    """Split ``"<uid>_<x>_<index>"`` from the right into ``(uid, x, index)``."""
    if not isinstance(key, str):
        raise TypeError(f"trajectory key must be str, got {type(key)!r}")
    parts = key.rsplit("_", 2)
    if len(parts) != 3 or not parts[0] or not parts[1]:
        raise ValueError(f"unexpected trajectory key format: {key!r}")
    try:
        index = int(parts[2])
    except ValueError as exc:
        raise ValueError(f"trajectory key has non-integer index: {key!r}") from exc
    return parts[0], parts[1], index


def group_rows_by_uid(keys) -> dict[str, list[int]]:
    seen: set[str] = set()
    groups: dict[str, list[int]] = {}
    for row, key in enumerate(keys):
        if key in seen:
            raise ValueError(f"duplicate trajectory key: {key!r}")
        seen.add(key)
        uid, _, _ = parse_trajectory_key(key)
        groups.setdefault(uid, []).append(row)
    return groups


# --------------------------------------------------------------------------- radix build
def _first_mismatch(a: np.ndarray, b: np.ndarray, start: int, end: int) -> int:
    if end <= start:
        return end
    diff = np.flatnonzero(a[start:end] != b[start:end])
    return start + int(diff[0]) if diff.size else end


def _radix_nodes(seqs: list[np.ndarray], rows: list[int]) -> list[dict]:
    """Compressed radix tree of ``rows`` (all sharing their first token).

    Returns node records in pre-order (node id == list index), children in the
    order their first member row appears in ``rows``.
    """
    out: list[dict] = []
    # Explicit stack of (rows, start, parent_id, slot) where slot is the index in
    # the parent's children list to fill -- keeps pre-order ids without recursion.
    work = [(rows, 0, None)]
    while work:
        members, start, parent = work.pop()
        lead = seqs[members[0]]
        end = min(len(seqs[r]) for r in members)
        for r in members[1:]:
            end = _first_mismatch(lead, seqs[r], start, end)
        node_id = len(out)
        terminal = [r for r in members if len(seqs[r]) == end]
        out.append(
            dict(node_id=node_id, parent_id=parent, start=start, end=end, rows=list(members),
                 terminal=terminal, children=[])
        )
        if parent is not None:
            out[parent]["children"].append(node_id)
        groups: dict[int, list[int]] = {}
        for r in members:
            if len(seqs[r]) > end:
                groups.setdefault(int(seqs[r][end]), []).append(r)
        # Push in reverse so the first group is expanded next (pre-order ids).
        for grp in reversed(list(groups.values())):
            work.append((grp, end, node_id))
    return out


def _records_to_tree(records: list[dict], *, uid: str, tree_index: int) -> TrajectoryTree:
    nodes = {
        r["node_id"]: TrajectoryNode(
            node_id=r["node_id"],
            parent_id=r["parent_id"],
            segment=SegmentRef(row=r["rows"][0], start=r["start"], end=r["end"]),
            member_rows=tuple(r["rows"]),
            terminal_rows=tuple(r["terminal"]),
            children=tuple(r["children"]),
        )
        for r in records
    }
    return TrajectoryTree(uid=uid, tree_index=tree_index, root_id=0,
                          member_rows=nodes[0].member_rows, nodes=nodes)


def build_trajectory_trees(keys, batch: Any) -> tuple[TrajectoryTree, ...]:
    """Build token-exact compressed tries for every uid group of ``batch``.

    ``uid`` only bounds which rows may share; topology is decided by exact token
    prefixes of the whole ``input_ids`` row (prompt/response boundaries do not
    matter).  A uid group whose rows start with different tokens yields one
    tree per first token.
    """
    keys = list(keys)
    if not keys:
        return ()
    inputs = batch_rows(batch, "input_ids")
    if len(keys) != len(inputs):
        raise ValueError(f"keys/batch row mismatch: keys={len(keys)} rows={len(inputs)}")
    groups = group_rows_by_uid(keys)
    seqs = [as_token_row(t, row=i).detach().cpu().numpy().astype(np.int64, copy=False)
            for i, t in enumerate(inputs)]
    trees: list[TrajectoryTree] = []
    for uid, rows in groups.items():
        by_first: dict[int, list[int]] = {}
        for r in rows:
            by_first.setdefault(int(seqs[r][0]), []).append(r)
        for tree_index, members in enumerate(by_first.values()):
            trees.append(_records_to_tree(_radix_nodes(seqs, members), uid=uid, tree_index=tree_index))
    return tuple(trees)


def build_prompt_sibling_trees(keys, batch: Any) -> tuple[TrajectoryTree, ...]:
    """Alias kept for callers of the older prompt->siblings builder name."""
    return build_trajectory_trees(keys, batch)

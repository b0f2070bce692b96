"""Turn-boundary tries: share only whole chat turns (Qwen ChatML ``<|im_end|>``).

A row is cut into *units* that end just after an ``<|im_end|>`` token, at the
prompt length (when ``prompts`` is present) and at the end of the row.  Units
shorter than ``min_segment_tokens`` are merged into the next one, except the
final tail which always stands.  Rows of one uid are then inserted unit by unit
(a unit matches only when its tokens are identical) and single-child chains with
unchanged membership are compressed.

Parity: verl/models/mcore/tpr/trajectory_tree_turn.py:33-186
(QWEN3_IM_END_TOKEN_ID, unit rule, compression rule and node numbering).
"""

from __future__ import annotations

from typing import Any

import torch

from .trajectory_tree import (
    SegmentRef,
    TrajectoryNode,
    TrajectoryTree,
    as_token_row,
    batch_rows,
    group_rows_by_uid,
)

QWEN3_IM_END_TOKEN_ID = 151645


def turn_units(tokens: list[int], *, prompt_length: int | None, min_segment_tokens: int,
               end_token_id: int) -> list[tuple[tuple[int, ...], int]]:
    """Split one row into ``(unit_tokens, absolute_end)`` pairs."""
    n = len(tokens)
    cuts = {i + 1 for i, t in enumerate(tokens) if t == end_token_id}
    if prompt_length is not None and 0 < prompt_length < n:
        cuts.add(prompt_length)
    cuts.add(n)
    units: list[tuple[tuple[int, ...], int]] = []
    prev = 0
    for end in sorted(cuts):
        if end < n and end - prev < min_segment_tokens:
            continue  # too short to be worth sharing: fold into the next unit
        units.append((tuple(tokens[prev:end]), end))
        prev = end
    assert prev == n and units, "turn units must cover the row"
    return units


class _Unit:
    __slots__ = ("end", "source_row", "rows", "terminal", "children")

    def __init__(self, end: int, source_row: int) -> None:
        self.end = end
        self.source_row = source_row
        self.rows: list[int] = []
        self.terminal: list[int] = []
        self.children: dict[tuple[int, ...], _Unit] = {}


def _emit(node: _Unit, start: int, parent: int | None, nodes: dict[int, TrajectoryNode]) -> int:
    last = node
    while not last.terminal and len(last.children) == 1:
        (nxt,) = last.children.values()
        if nxt.rows != last.rows:
            break
        last = nxt
    node_id = len(nodes)
    seg = SegmentRef(row=node.source_row, start=start, end=last.end)
    # Reserve the id (pre-order) before the children are numbered.
    nodes[node_id] = None  # type: ignore[assignment]
    kids = tuple(_emit(c, last.end, node_id, nodes) for c in last.children.values())
    nodes[node_id] = TrajectoryNode(node_id=node_id, parent_id=parent, segment=seg,
                                    member_rows=tuple(last.rows), terminal_rows=tuple(last.terminal),
                                    children=kids)
    return node_id


def build_trajectory_trees_turn(keys, batch: Any, *, min_segment_tokens: int = 128,
                                end_token_id: int = QWEN3_IM_END_TOKEN_ID) -> tuple[TrajectoryTree, ...]:
    """Build tries that share only completed turn units (Qwen ChatML policy)."""
    if not isinstance(min_segment_tokens, int) or isinstance(min_segment_tokens, bool) or min_segment_tokens < 1:
        raise ValueError("min_segment_tokens must be a positive integer")
    if not isinstance(end_token_id, int) or isinstance(end_token_id, bool) or end_token_id < 0:
        raise ValueError("end_token_id must be a non-negative integer")
    keys = list(keys)
    if not keys:
        return ()
    inputs = batch_rows(batch, "input_ids")
    if len(inputs) != len(keys):
        raise ValueError("turn builder input rows and trajectory keys disagree")
    try:
        prompts = batch_rows(batch, "prompts")
    except (ValueError, KeyError):
        prompts = None
    if prompts is not None and len(prompts) != len(keys):
        raise ValueError("turn builder prompt rows and trajectory keys disagree")
    groups = group_rows_by_uid(keys)
    units_by_row = []
    for row in range(len(keys)):
        ids = as_token_row(inputs[row], row=row)
        plen = None
        if prompts is not None:
            prompt = as_token_row(prompts[row], row=row)
            plen = int(prompt.numel())
            if plen > ids.numel() or not torch.equal(ids[:plen].cpu(), prompt.cpu()):
                raise ValueError(f"turn builder prompt is not an exact input prefix for row={row}")
        units_by_row.append(turn_units(ids.detach().cpu().tolist(), prompt_length=plen,
                                       min_segment_tokens=min_segment_tokens, end_token_id=end_token_id))
    forest: list[TrajectoryTree] = []
    for uid, rows in groups.items():
        top = _Unit(0, rows[0])
        for row in rows:
            cur = top
            for sig, end in units_by_row[row]:
                nxt = cur.children.get(sig)
                if nxt is None:
                    nxt = cur.children[sig] = _Unit(end, row)
                elif nxt.end != end:
                    raise AssertionError("identical turn tokens have different absolute ends")
                nxt.rows.append(row)
                cur = nxt
            cur.terminal.append(row)
        for tree_index, first in enumerate(top.children.values()):
            nodes: dict[int, TrajectoryNode] = {}
            root = _emit(first, 0, None, nodes)
            forest.append(TrajectoryTree(uid=uid, tree_index=tree_index, root_id=root,
                                         member_rows=nodes[root].member_rows, nodes=nodes))
    return tuple(forest)

"""Token tries, turn tries, plan lowering and SegmentPlan validation (CPU)."""

import pytest
import torch

from bridge_b200.tpr import (PopSegment, PushSegment, SegmentPlan, SegmentSpec, build_trajectory_trees,
                             build_trajectory_trees_turn, build_tree_execution_plans)
from bridge_b200.tpr.trajectory_tree_turn import QWEN3_IM_END_TOKEN_ID


def _batch(rows, resp_lens):
    ids = [torch.tensor(r) for r in rows]
    masks = [torch.ones(n, dtype=torch.bool) for n in resp_lens]
    return {"input_ids": ids, "response_mask": masks}


def test_exact_trie_shares_prefix_and_splits_first_token():
    rows = [[1, 2, 3, 4], [1, 2, 3, 5], [1, 2, 9], [7, 8], [1, 2, 3, 4]]
    keys = [f"u_a_{i}" for i in range(4)] + ["v_a_0"]
    trees = build_trajectory_trees(keys, _batch(rows, [1, 1, 1, 1, 1]))
    assert len(trees) == 3  # uid u: first tokens 1 and 7 -> two trees; uid v: one tree
    t0 = trees[0]
    root = t0.get(t0.root_id)
    assert (root.segment.start, root.segment.end) == (0, 2) and set(root.member_rows) == {0, 1, 2}
    kids = [t0.get(c) for c in root.children]
    assert [(k.segment.start, k.segment.end) for k in kids] == [(2, 3), (2, 3)]
    mid = kids[0]
    assert len(mid.children) == 2 and mid.terminal_rows == ()
    assert t0.unique_tokens == 2 + 1 + 1 + 1 + 1


def test_duplicate_rows_are_terminal_in_one_node():
    rows = [[4, 5, 6], [4, 5, 6], [4, 5]]
    trees = build_trajectory_trees(["x_y_0", "x_y_1", "x_y_2"], _batch(rows, [1, 1, 1]))
    (t,) = trees
    root = t.get(t.root_id)
    assert root.terminal_rows == (2,) and (root.segment.start, root.segment.end) == (0, 2)
    (leaf,) = [t.get(c) for c in root.children]
    assert leaf.terminal_rows == (0, 1)


def test_key_parsing_and_duplicates():
    with pytest.raises(ValueError):
        build_trajectory_trees(["bad"], _batch([[1]], [1]))
    with pytest.raises(ValueError):
        build_trajectory_trees(["a_b_0", "a_b_0"], _batch([[1], [1]], [1, 1]))


def test_turn_trie_shares_whole_turns_only():
    E = QWEN3_IM_END_TOKEN_ID
    common = [1, 2, E, 3, 4, E]
    rows = [common + [9, 9, 9], common + [8, 8], common[:4] + [5, 5]]
    trees = build_trajectory_trees_turn(["s_a_0", "s_a_1", "s_a_2"], _batch(rows, [3, 2, 2]), min_segment_tokens=2)
    (t,) = trees
    root = t.get(t.root_id)
    assert (root.segment.start, root.segment.end) == (0, 3)  # first complete turn only
    assert set(root.member_rows) == {0, 1, 2}


def test_plan_ownership_first_response_token_owned_by_parent():
    rows = [[10, 11, 12, 20, 21], [10, 11, 12, 30, 31]]
    batch = _batch(rows, [2, 2])
    forest = build_tree_execution_plans(["u_a_0", "u_a_1"], batch)
    (tree,) = forest.trees
    assert forest.logical_loss_tokens == 4
    root = tree.segment_plan.root_id
    owners = sorted((r.sample_row, r.response_offset, r.segment_id == root, r.query_offset) for r in tree.objective_refs)
    # response token at position 3 is predicted by query 2 (last root row); position 4 by the child's row 0
    assert owners[0] == (0, 0, True, 2) and owners[1][2] is False and owners[1][3] == 0


def test_plan_loss_mask_alignment_checks():
    batch = _batch([[1, 2, 3]], [1])
    batch["loss_mask"] = [torch.tensor([0, 1, 1])]
    with pytest.raises(ValueError):
        build_tree_execution_plans(["a_b_0"], batch, require_loss_mask_alignment=True)


def test_segment_plan_validation_and_events():
    s0 = SegmentSpec(0, None, torch.tensor([1, 2]), 0, 0)
    s1 = SegmentSpec(1, 0, torch.tensor([3]), 2, 2)
    s2 = SegmentSpec(2, 0, torch.tensor([4, 5]), 2, 2)
    plan = SegmentPlan([s0, s1, s2], root_id=0, topology_only=True)
    ev = tuple(plan.dfs_events())
    assert ev == (PushSegment(0), PushSegment(1), PopSegment(1), PushSegment(2), PopSegment(2), PopSegment(0))
    with pytest.raises(ValueError):
        plan.validate_events([PushSegment(0), PushSegment(1), PopSegment(0)])
    with pytest.raises(ValueError):
        SegmentPlan([s0, SegmentSpec(1, 0, torch.tensor([3]), 3, 3)], root_id=0, topology_only=True)
    with pytest.raises(ValueError):
        SegmentPlan([s0, s1], root_id=1, topology_only=True)

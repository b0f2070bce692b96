"""DP placement planner and TP plan agreement (gloo)."""

import itertools

import pytest
import torch

from bridge_b200.tpr.dp_placement import plan_dta_dfs, plan_tpr_dta_dp, plan_verl_uid, trie_token_cost
from tests.dist_utils import run_ranks


def _brute(seqs, dp):
    order = sorted(range(len(seqs)), key=lambda i: (seqs[i], i))
    best = None
    for cuts in itertools.combinations(range(1, len(seqs)), dp - 1):
        bounds = (0, *cuts, len(seqs))
        cost = max(trie_token_cost([seqs[order[i]] for i in range(a, b)]) for a, b in zip(bounds, bounds[1:]))
        best = cost if best is None else min(best, cost)
    return best


def test_dta_is_minimax_optimal_over_contiguous_partitions():
    g = torch.Generator().manual_seed(1)
    seqs = []
    for t in range(3):
        p = torch.randint(0, 5, (6,), generator=g).tolist()
        for s in range(3):
            seqs.append(tuple(p + torch.randint(0, 5, (int(torch.randint(1, 6, (1,), generator=g)),), generator=g).tolist()))
    plan = plan_dta_dfs(seqs, 3, enforce_equal_rows=False)
    assert plan.max_rank_tree_tokens == _brute(seqs, 3)
    assert sorted(i for p in plan.partitions for i in p) == list(range(len(seqs)))


def test_tpr_dta_respects_uid_and_equal_rows():
    seqs = [(1, 2, 3), (1, 2, 4), (1, 2, 3), (1, 2, 4)]
    keys = ["a_x_0", "a_x_1", "b_x_0", "b_x_1"]
    plan = plan_tpr_dta_dp(seqs, keys, 2)
    assert plan.equal_rows_per_rank and plan.global_tree_tokens == 8
    base = plan_verl_uid(seqs, ["a", "a", "b", "b"], 2)
    assert base.equal_rows_per_rank and len(base.partitions) == 2


def _tp_worker(rank, world, same):
    from bridge_b200.tpr.tp_validation import assert_tp_plan_agreement

    digest = ("ab" * 32) if (same or rank == 0) else ("cd" * 32)
    try:
        assert_tp_plan_agreement(digest, tp_size=world)
        return "ok"
    except RuntimeError as exc:
        return "mismatch" if "mismatch" in str(exc) else repr(exc)


def test_tp_plan_agreement_collective():
    assert run_ranks(2, _tp_worker, True) == ["ok", "ok"]
    assert run_ranks(2, _tp_worker, False) == ["mismatch", "mismatch"]


def test_forest_digest_is_deterministic():
    from bridge_b200.tpr import build_tree_execution_plans
    from bridge_b200.tpr.tp_validation import digest_forest_plan
    from tests.helpers import tree_batch

    b = tree_batch(n_trees=2, prefix=8, siblings=3, resp=4)
    keys = [f"{u}_x_{i}" for i, u in enumerate(b["uid"])]
    d1 = digest_forest_plan(build_tree_execution_plans(keys, b))
    d2 = digest_forest_plan(build_tree_execution_plans(keys, b))
    b["input_ids"][0] = b["input_ids"][0].clone()
    b["input_ids"][0][-1] += 1
    assert d1 == d2 != digest_forest_plan(build_tree_execution_plans(keys, b))


class _FakeBuffer:
    def __init__(self, nbytes):
        self.local = torch.zeros(nbytes, dtype=torch.uint8)
        self.ptrs = [0]

    def view(self, dtype, numel=None):
        t = self.local.view(dtype)
        return t if numel is None else t[:numel]


class _FakeHeap:
    def __init__(self, size, rank):
        self.size, self.rank = size, rank

    def alloc(self, nbytes):
        return _FakeBuffer((int(nbytes) + 255) // 256 * 256)


def test_sharded_arena_bucket_layout_round_trips():
    """Bucket-interleaved shards of the NVLink optimizer: every bucket is padded to 8 x N and split N ways;
    gathering all ranks' pieces and reordering gives the parameters back in order, and the inverse
    recovers each rank's piece."""
    from bridge_b200.engine.optim import _ShardedArena, bucket_groups
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model

    cfg = get_config("tiny", num_layers=3)
    n = 3
    pieces, ref = [], None
    for r in range(n):
        model = build_model(cfg, dtype=torch.float32, seed=0)
        groups = bucket_groups(model)
        assert [g[0] for g in groups] == ["embed", 0, 1, 2, "tail"]
        flat = torch.cat([p.detach().reshape(-1).clone() for _, g in groups for p in g])
        ref = flat if ref is None else ref
        a = _ShardedArena(groups, torch.float32, _FakeHeap(n, r))
        for _, off, padded, sub, lo in a.buckets:
            assert padded % (8 * n) == 0 and sub * n == padded and off % (8 * n) == 0
        assert a.master.numel() == a.shard == sum(b[3] for b in a.buckets)
        pieces.append(a.master.clone())
        assert torch.equal(a.from_param_order(flat, r), a.master)
    assert torch.equal(a.to_param_order(pieces), ref)

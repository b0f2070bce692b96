"""Prefix-aware data-parallel placement of trajectories (offline planner).

The cost of a set of rows is the number of *unique trie tokens* it needs: in
sorted order, ``len(first) + sum(len(row) - lcp(row, previous))`` (rows of
different uids never share).  ``plan_dta_dfs`` sorts rows by (uid, tokens) and
finds the contiguous partition into ``dp`` ranks that minimises the largest
per-rank cost (binary search on the bound + greedy feasibility), preferring an
equal-rows split when it achieves the same optimum.  ``plan_verl_uid`` is the
uid-balanced baseline (whole uid groups, equal group counts, longest-first
greedy on token length).

Parity: verl/models/mcore/tpr/dp_placement.py:25-327 (DPPlacementPlan,
plan_dta_dfs, plan_tpr_dta_dp, plan_verl_uid; the minimax contiguous-partition
objective is the DTA rule and is kept as specified).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

from .trajectory_tree import parse_trajectory_key

Policy = Literal["dta_dfs", "tpr_dta", "verl_uid"]


@dataclass(frozen=True, slots=True)
class DPPlacementPlan:
    partitions: tuple[tuple[int, ...], ...]
    tree_tokens_by_rank: tuple[int, ...]
    global_tree_tokens: int
    duplicated_tree_tokens: int
    equal_rows_per_rank: bool
    policy: Policy

    @property
    def max_rank_tree_tokens(self) -> int:
        return max(self.tree_tokens_by_rank)


def _as_tuples(seqs) -> tuple[tuple[int, ...], ...]:
    out = []
    for i, s in enumerate(seqs):
        t = tuple(s)
        if not t:
            raise ValueError(f"sequence {i} is empty; pass unpadded real tokens")
        if any(not isinstance(x, int) or isinstance(x, bool) or x < 0 for x in t):
            raise TypeError(f"sequence {i} must contain nonnegative Python int token IDs")
        out.append(t)
    return tuple(out)


def _lcp(a: tuple[int, ...], b: tuple[int, ...]) -> int:
    n = min(len(a), len(b))
    i = 0
    while i < n and a[i] == b[i]:
        i += 1
    return i


def trie_token_cost(seqs: Sequence[tuple[int, ...]], uids: Sequence[str] | None = None) -> int:
    """Unique trie tokens of ``seqs`` (shared only within a uid when ``uids`` is given)."""
    if not seqs:
        return 0
    idx = sorted(range(len(seqs)), key=(lambda i: seqs[i]) if uids is None else (lambda i: (uids[i], seqs[i])))
    total = len(seqs[idx[0]])
    for p, c in zip(idx, idx[1:]):
        same = uids is None or uids[p] == uids[c]
        total += len(seqs[c]) - (_lcp(seqs[p], seqs[c]) if same else 0)
    return total


def _finish(seqs, parts, policy, dp, enforce_equal, uids) -> DPPlacementPlan:
    if len(parts) != dp:
        raise ValueError(f"expected {dp} DP partitions, got {len(parts)}")
    if any(not p for p in parts):
        raise ValueError("each DP replica must receive at least one trajectory")
    if sorted(i for p in parts for i in p) != list(range(len(seqs))):
        raise ValueError("DP partitions must cover each input row exactly once")
    equal = len({len(p) for p in parts}) == 1
    if enforce_equal and not equal:
        raise ValueError("placement produced unequal per-DP row counts; the equal-count dispatch contract forbids it")

    def cost(ix):
        sub = [seqs[i] for i in ix]
        return trie_token_cost(sub, None if uids is None else [uids[i] for i in ix])

    costs = tuple(cost(p) for p in parts)
    glob = cost(range(len(seqs)))
    dup = sum(costs) - glob
    if dup < 0:
        raise AssertionError("partitions cannot need fewer unique tokens than the global forest")
    return DPPlacementPlan(tuple(tuple(p) for p in parts), costs, glob, dup, equal, policy)


def plan_dta_dfs(token_sequences, dp_size: int, *, enforce_equal_rows: bool = True,
                 uid_list: Sequence[str] | None = None) -> DPPlacementPlan:
    if type(dp_size) is not int or dp_size <= 0:
        raise ValueError("dp_size must be a positive integer")
    seqs = _as_tuples(token_sequences)
    n = len(seqs)
    if n < dp_size:
        raise ValueError("number of trajectories must be >= dp_size")
    if uid_list is not None and len(uid_list) != n:
        raise ValueError("uid_list and trajectories must have the same row count")
    order = sorted(range(n), key=(lambda i: (seqs[i], i)) if uid_list is None else (lambda i: (uid_list[i], seqs[i], i)))
    lens = [len(seqs[i]) for i in order]
    # prefix sums of the incremental trie cost of each sorted row (relative to its predecessor)
    inc = [0] * n
    for j in range(1, n):
        a, b = order[j - 1], order[j]
        shared = uid_list is None or uid_list[a] == uid_list[b]
        inc[j] = lens[j] - (_lcp(seqs[a], seqs[b]) if shared else 0)
    pre = [0]
    for x in inc:
        pre.append(pre[-1] + x)

    def seg_cost(s: int, e: int) -> int:  # rows order[s:e]
        return lens[s] + pre[e] - pre[s + 1]

    def greedy(bound: int) -> list[tuple[int, int]]:
        out, s = [], 0
        while s < n:
            lo, hi = s + 1, n
            while lo < hi:  # largest e with cost <= bound (cost is monotone in e)
                mid = (lo + hi + 1) // 2
                if seg_cost(s, mid) <= bound:
                    lo = mid
                else:
                    hi = mid - 1
            out.append((s, lo))
            s = lo
        return out

    lo = max(lens)
    hi = trie_token_cost(seqs, uid_list)
    while lo < hi:
        mid = (lo + hi) // 2
        if len(greedy(mid)) <= dp_size:
            hi = mid
        else:
            lo = mid + 1
    groups = greedy(lo)
    if enforce_equal_rows and n % dp_size == 0:
        k = n // dp_size
        eq = [(r * k, (r + 1) * k) for r in range(dp_size)]
        if all(seg_cost(s, e) <= lo for s, e in eq):
            groups = eq
    while len(groups) < dp_size:  # split (never increases the max) until every rank has rows
        j = max((i for i, (s, e) in enumerate(groups) if e - s > 1), default=None)
        if j is None:
            raise AssertionError("could not construct non-empty DP partitions")
        s, e = groups[j]
        groups[j:j + 1] = [(s, e - 1), (e - 1, e)]
    parts = [[order[i] for i in range(s, e)] for s, e in groups]
    return _finish(seqs, parts, "dta_dfs" if uid_list is None else "tpr_dta", dp_size, enforce_equal_rows, uid_list)


def plan_tpr_dta_dp(token_sequences, trajectory_keys: Sequence[str], dp_size: int, *,
                    enforce_equal_rows: bool = True) -> DPPlacementPlan:
    if len(trajectory_keys) != len(token_sequences):
        raise ValueError("trajectory_keys and token_sequences must have equal lengths")
    if len(set(trajectory_keys)) != len(trajectory_keys):
        raise ValueError("trajectory_keys must be unique")
    uids = tuple(parse_trajectory_key(k)[0] for k in trajectory_keys)
    return plan_dta_dfs(token_sequences, dp_size, enforce_equal_rows=enforce_equal_rows, uid_list=uids)


def plan_verl_uid(token_sequences, uid_list: Sequence[str], dp_size: int) -> DPPlacementPlan:
    """Whole-uid balanced placement (equal group count per rank, longest-first greedy on tokens)."""
    if type(dp_size) is not int or dp_size <= 0:
        raise ValueError("dp_size must be a positive integer")
    seqs = _as_tuples(token_sequences)
    if len(uid_list) != len(seqs):
        raise ValueError("uid_list and trajectories must have the same row count")
    if len(seqs) < dp_size:
        raise ValueError("number of trajectories must be >= dp_size")
    groups: dict[str, list[int]] = {}
    last = object()
    for i, u in enumerate(uid_list):
        if u != last and u in groups:
            raise ValueError("uid balancing requires contiguous rows for each uid")
        groups.setdefault(u, []).append(i)
        last = u
    glist = list(groups.values())
    if len(glist) % dp_size:
        raise ValueError("uid balancing needs a number of uid groups divisible by dp_size")
    cap = len(glist) // dp_size
    load = [0] * dp_size
    members: list[list[int]] = [[] for _ in range(dp_size)]
    counts = [0] * dp_size
    for g in sorted(glist, key=lambda g: -sum(len(seqs[i]) for i in g)):
        r = min((r for r in range(dp_size) if counts[r] < cap), key=lambda r: load[r])
        members[r].extend(g)
        load[r] += sum(len(seqs[i]) for i in g)
        counts[r] += 1
    return _finish(seqs, [sorted(m) for m in members], "verl_uid", dp_size, True, uid_list)

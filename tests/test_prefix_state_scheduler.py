"""Prefix state, KV stack relay, scheduler leaf fusion and failure semantics (CPU)."""

import pytest
import torch

from bridge_b200.tpr import (FixedTopologyScheduler, GDNLayerState, GDNPrefixState, KVStack, PhysicalExecutionKind,
                             SchedulerState, SegmentExecutor, SegmentPlan, SegmentSpec, TPRBatchRunner)


def _seg(i, parent, n, start):
    return SegmentSpec(i, parent, torch.arange(n) % 7, start, start)


def test_kv_stack_anchor_relay_split_back():
    st = KVStack()
    a, b = _seg(0, None, 3, 0), _seg(1, 0, 2, 3)
    st.push(a, {1: (torch.ones(3, 2, 4), torch.ones(3, 2, 4))})
    st.push(b, {1: (torch.zeros(2, 2, 4), torch.zeros(2, 2, 4))})
    anchors = st.build_past_anchors()
    k, v = anchors.key_values[1]
    assert k.shape[0] == 5 and anchors.prefix_length == 5
    (k.sum() * 2 + v.sum()).backward()
    st.accumulate_anchor_gradients(anchors)
    g0 = st.get(0).gradients[1]
    assert torch.all(g0[0] == 2) and g0[0].shape[0] == 3
    st.pop(1)
    with pytest.raises(RuntimeError):
        st.accumulate_anchor_gradients(anchors)  # stale: stack changed


def test_gdn_prefix_state_generation_guard():
    s = GDNPrefixState.save(0, 4, {2: GDNLayerState(torch.zeros(1, 3, 4), torch.zeros(1, 2, 2, 2))})
    anc = s.make_anchors()
    (anc.layer_states[2].conv_state.sum() + anc.layer_states[2].recurrent_state.sum()).backward()
    s.accumulate_anchor_gradients(anc)
    grads = s.consume_gradients()
    assert torch.all(grads[2].conv_state == 1)
    with pytest.raises(RuntimeError):
        s.accumulate_anchor_gradients(anc)  # generation advanced by consume


class _Toy(torch.nn.Module):
    """Minimal model honouring the TPR context (one attention layer, tied head)."""

    attention_layer_numbers = (1,)
    gdn_layer_numbers = ()

    def __init__(self, fail_at=None):
        super().__init__()
        from bridge_b200.models import get_config
        from bridge_b200.models.decoder import build_model

        self.inner = build_model(get_config("tiny", num_layers=1), dtype=torch.float32)
        self.fail_at = fail_at
        self.calls = 0
        self.vocab_size = 1024
        self.tp_group = None
        self.vocab_start = 0

    def forward(self, ids, pos, max_position=None):
        self.calls += 1
        if self.fail_at is not None and self.calls >= self.fail_at:
            raise RuntimeError("injected failure")
        return self.inner(ids, pos, max_position)

    def head_input(self, h):
        return h

    @property
    def head_weight(self):
        return self.inner.head_weight


def _ce_plan():
    from bridge_b200.tpr import SegmentLossTerm

    s0 = SegmentSpec(0, None, torch.arange(6), 0, 0, (SegmentLossTerm(5, 3),))
    s1 = SegmentSpec(1, 0, torch.arange(4) + 1, 6, 6, (SegmentLossTerm(0, 5), SegmentLossTerm(2, 8)))
    s2 = SegmentSpec(2, 0, torch.arange(3) + 2, 6, 6, (SegmentLossTerm(1, 9),))
    return SegmentPlan([s0, s1, s2], root_id=0)


def test_scheduler_fuses_leaves_and_completes():
    plan = _ce_plan()
    ex = SegmentExecutor(_Toy(), plan)
    sched = FixedTopologyScheduler(plan, ex)
    res = sched.run()
    kinds = [e.kind for e in res.execution_trace]
    assert kinds == [PhysicalExecutionKind.PUSH, PhysicalExecutionKind.VISIT_LEAF, PhysicalExecutionKind.VISIT_LEAF,
                     PhysicalExecutionKind.POP]
    assert sched.state is SchedulerState.COMPLETED and res.peak_path_tokens == 10
    with pytest.raises(RuntimeError):
        sched.run()


def test_failure_latch_and_runner_does_not_finalize():
    plan = _ce_plan()
    ex = SegmentExecutor(_Toy(fail_at=2), plan)
    sched = FixedTopologyScheduler(plan, ex)
    with pytest.raises(RuntimeError, match="injected"):
        sched.run()
    assert sched.state is SchedulerState.FAILED and ex.failed
    with pytest.raises(RuntimeError, match="failed"):
        ex.push(0)
    finalized = []

    def run_tree(tp):
        raise RuntimeError("tree failed")

    runner = TPRBatchRunner(run_tree=run_tree, finalize_gradients=lambda: finalized.append(1))
    from tests.helpers import tree_batch
    from bridge_b200.tpr import build_tree_execution_plans

    b = tree_batch(n_trees=1, prefix=4, siblings=2, resp=2)
    forest = build_tree_execution_plans([f"{u}_x_{i}" for i, u in enumerate(b["uid"])], b)
    with pytest.raises(RuntimeError, match="tree failed"):
        runner.run(forest)
    assert finalized == []
    with pytest.raises(RuntimeError, match="single-use"):
        runner.run(forest)


def test_ce_segment_executor_matches_flat_ce():
    torch.manual_seed(0)
    model = _Toy()
    plan = _ce_plan()
    res = FixedTopologyScheduler(plan, SegmentExecutor(model, plan)).run()
    g_tpr = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad()
    # flattened: root+leaf1 and root+leaf2 sequences, CE on the same terms
    seqs = [(torch.cat([torch.arange(6), torch.arange(4) + 1]), [(5, 3), (6, 5), (8, 8)]),
            (torch.cat([torch.arange(6), torch.arange(3) + 2]), [(7, 9)])]
    total = 0.0
    for ids, terms in seqs:
        h = model(ids, torch.arange(ids.numel()))
        logits = h @ model.head_weight.t()
        for q, t in terms:
            total = total + torch.nn.functional.cross_entropy(logits[q][None], torch.tensor([t]))
    # the root term (5 -> 3) is owned once by the root segment, so it appears in one flattened row only
    loss = total / plan.total_loss_weight
    loss.backward()
    assert abs(float(res.normalized_loss) - float(loss.detach())) < 1e-5
    for n, g in g_tpr.items():
        ref = dict(model.named_parameters())[n].grad
        assert float((g - ref).norm() / (ref.norm() + 1e-12)) < 1e-4, n

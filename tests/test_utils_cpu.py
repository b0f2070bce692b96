"""Profiler records and actor-update capture / replay (CPU)."""

import os

import pytest
import torch

from bridge_b200.engine import EngineConfig, TPREngine
from bridge_b200.models import get_config
from bridge_b200.models.decoder import build_model
from tests.helpers import set_old_log_probs, tree_batch


def _engine(**kw):
    cfg = get_config("tiny")
    return TPREngine(cfg, EngineConfig(**kw), device="cpu", model=build_model(cfg, dtype=torch.float32, seed=0))


@pytest.mark.parametrize("executor", ["forest", "segment"])
def test_exec_profile_records_every_event(executor):
    eng = _engine(exec_profile=True, executor=executor)
    batch = tree_batch(n_trees=2, prefix=32, siblings=3, resp=8, seed=1)
    set_old_log_probs(eng.model, batch)
    eng.forward_backward_batch(batch)
    prof = eng._tpr_segment_event_profiler
    recs = prof.materialize()
    kinds = {r["kind"] for r in recs}
    if executor == "forest":
        assert kinds == {"push_chunk", "visit_chunk", "pop_chunk"}
    else:
        assert "visit_leaf" in kinds and "push" in kinds and "pop" in kinds
    assert all(r["cpu_enqueue_ms"] >= 0 for r in recs)
    assert prof.summary()["events"] == len(recs)


def test_actor_capture_is_atomic_refuses_overwrite_and_replays(tmp_path, monkeypatch):
    from bridge_b200.utils.capture import capture_actor_update_minibatch, load_capture

    batch = tree_batch(n_trees=2, prefix=32, siblings=3, resp=8, seed=2)
    eng = _engine()
    set_old_log_probs(eng.model, batch)
    batch["global_steps"] = torch.full((len(batch["input_ids"]),), 7)
    path = capture_actor_update_minibatch(batch, batch_idx=0, rank=0, directory=str(tmp_path))
    assert os.path.basename(path) == "step00000007_rank00000_capture000000_batch0.pt"
    assert not [f for f in os.listdir(tmp_path) if f.startswith(".capture_")]
    with pytest.raises(FileExistsError):
        capture_actor_update_minibatch(batch, batch_idx=0, rank=0, directory=str(tmp_path))
    bad = dict(batch, global_steps=torch.tensor([1, 2] + [1] * (len(batch["input_ids"]) - 2)))
    with pytest.raises(ValueError):
        capture_actor_update_minibatch(bad, batch_idx=1, rank=0, directory=str(tmp_path))
    replay = load_capture(path)
    a = eng.forward_backward_batch(batch)["loss"][0]
    eng.zero_grad()
    b = eng.forward_backward_batch(replay)["loss"][0]
    assert abs(a - b) < 1e-6


def test_capture_env_hook_writes_once_per_minibatch(tmp_path, monkeypatch):
    monkeypatch.setenv("TPR_CAPTURE_DIR", str(tmp_path))
    batch = tree_batch(n_trees=1, prefix=16, siblings=2, resp=8, seed=3)
    eng = _engine()
    set_old_log_probs(eng.model, batch)
    batch["global_steps"] = 3
    eng.forward_backward_batch(batch)
    eng.forward_backward_batch(batch)
    files = sorted(os.listdir(tmp_path))
    assert files == ["step00000003_rank00000_capture000000_batch0.pt", "step00000003_rank00000_capture000001_batch1.pt"]


def test_gemm_mshape_tool_reports_split_drift():
    from bridge_b200.utils.gemm_mshape import mshape_drift

    r = mshape_drift(96, 256, 128, 32, device="cpu")
    assert r["torch"]["rel_l2"] < 1e-2 and r["torch"]["max_abs"] >= 0.0


def test_cp_drift_tool(tmp_path):
    from bridge_b200.utils.cp_drift import _flat, drift, main

    a = torch.randn(500) - 3
    b = a + 1e-3 * torch.randn(500)
    torch.save(a, tmp_path / "a.pt")
    torch.save({"log_probs": [b[:200], b[200:]]}, tmp_path / "b.pt")
    out = drift(_flat(torch.load(tmp_path / "a.pt")), _flat(torch.load(tmp_path / "b.pt", weights_only=False)))
    assert out["cosine"] > 0.999 and out["rel_l2"] < 1e-3
    main([str(tmp_path / "a.pt"), str(tmp_path / "b.pt")])


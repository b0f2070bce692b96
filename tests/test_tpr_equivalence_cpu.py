"""Config #1 gate (single rank): TPR logprobs, PPO loss and grads equal the flattened batch (FP32, CPU)."""

import pytest
import torch

from bridge_b200.engine import EngineConfig, TPREngine
from bridge_b200.models import get_config
from bridge_b200.models.decoder import build_model
from tests.helpers import flat_ppo_loss, grads_of, rel_err, set_old_log_probs, tree_batch


def _engine(executor, mode="retain", cfg="tiny", budget=8192):
    model = build_model(get_config(cfg), dtype=torch.float32, seed=0)
    ec = EngineConfig(executor=executor, forest_mode=mode, token_budget=budget)
    return TPREngine(get_config(cfg), ec, device="cpu", model=model)


def _oracle(cfg="tiny", batch=None):
    model = build_model(get_config(cfg), dtype=torch.float32, seed=0)
    loss, lps = flat_ppo_loss(model, batch)
    loss.backward()
    return model, loss.detach()


@pytest.mark.parametrize("executor,mode,budget", [
    ("forest", "retain", 8192), ("forest", "recompute", 8192), ("forest", "retain", 130), ("segment", "retain", 8192),
])
def test_tpr_matches_flattened(executor, mode, budget):
    ref_model = build_model(get_config("tiny"), dtype=torch.float32, seed=0)
    batch = tree_batch(n_trees=1, prefix=128, siblings=4, resp=64, seed=0)
    set_old_log_probs(ref_model, batch)
    oracle, ref_loss = _oracle(batch=batch)
    eng = _engine(executor, mode, budget=budget)
    out = eng.forward_backward_batch(batch)
    assert out["metrics"]["tpr/logical_loss_tokens"] == [256]
    assert out["metrics"]["tpr/unique_tree_tokens"] == [128 + 4 * 64]
    assert abs(out["loss"][0] - float(ref_loss)) < 1e-5 * max(1.0, abs(float(ref_loss)))
    g_tpr = {n: p.main_grad for n, p in eng.model.named_parameters()}
    g_ref = {n: p.grad for n, p in oracle.named_parameters()}
    for n in g_ref:
        assert rel_err(g_tpr[n], g_ref[n]) < 1e-4, n


def test_multi_tree_forest_and_masks():
    batch = tree_batch(n_trees=3, prefix=40, siblings=3, resp=24, seed=3, mask_prob=0.5, temperature=0.7)
    ref_model = build_model(get_config("tiny"), dtype=torch.float32, seed=0)
    set_old_log_probs(ref_model, batch)
    oracle, ref_loss = _oracle(batch=batch)
    eng = _engine("forest", budget=100)
    out = eng.forward_backward_batch(batch)
    assert abs(out["loss"][0] - float(ref_loss)) < 1e-5
    for n, p in oracle.named_parameters():
        assert rel_err(dict(eng.model.named_parameters())[n].main_grad, p.grad) < 1e-4, n

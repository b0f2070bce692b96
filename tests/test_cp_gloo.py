"""Config #1 gate: CP world_size 2 (gloo, FP32) -- TPR loss, log-probs and grads equal the flattened 4x192 batch,
for every context-parallel backend; hybrid (Ulysses x ring) at CP 4."""

import pytest
import torch

from tests.dist_utils import run_ranks


def _worker(rank, world, backend, n_layers, preset="tiny", prefix=128, resp=64):
    import torch

    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel.groups import build_parallel_state
    from tests.helpers import flat_ppo_loss, set_old_log_probs, tree_batch

    cfg = get_config(preset, num_layers=n_layers)
    batch = tree_batch(n_trees=1, prefix=prefix, siblings=4, resp=resp, seed=0)
    ref = build_model(cfg, dtype=torch.float32, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, lps = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    ps = build_parallel_state(tp=1, cp=world)
    model = build_model(cfg, dtype=torch.float32, seed=0)
    ec = EngineConfig(context_parallel_size=world, tpr_cp_backend=backend)
    eng = TPREngine(cfg, ec, device="cpu", model=model, parallel_state=ps)
    batch["tpr_capture_log_probs"] = True
    out = eng.forward_backward_batch(batch)
    errs = {}
    for n, p in eng.model.named_parameters():
        g_ref = dict(ref.named_parameters())[n].grad
        errs[n] = float((p.main_grad - g_ref).norm() / (g_ref.norm() + 1e-12))
    return {"loss": out["loss"][0], "loss_ref": float(loss_ref), "grad_rel": errs}


@pytest.mark.parametrize("backend", ["allgather", "ring", "ulysses"])
def test_cp2_matches_flattened(backend):
    res = run_ranks(2, _worker, backend, 2)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_hybrid_cp4_matches_flattened():
    res = run_ranks(4, _worker, "hybrid", 1)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


@pytest.mark.parametrize("prefix,resp", [(128, 64), (131, 63)])
def test_hybrid_gdn_cp2_ring_matches_flattened(prefix, resp):
    """GDN layers under ring CP: head-parallel exchange with un-zigzag (and padding), head-local state relay."""
    res = run_ranks(2, _worker, "ring", 4, "tiny_hybrid", prefix, resp)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def _tpcp_worker(rank, world, backend):
    import torch

    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel.groups import build_parallel_state
    from tests.helpers import flat_ppo_loss, set_old_log_probs, tree_batch

    cfg = get_config("tiny", num_layers=2)
    batch = tree_batch(n_trees=1, prefix=128, siblings=4, resp=64, seed=0)
    ref = build_model(cfg, dtype=torch.float32, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    from bridge_b200.models.checkpoint import hf_state_dict, load_hf_state_dict

    ps = build_parallel_state(tp=2, cp=2)
    model = build_model(cfg, dtype=torch.float32, seed=1, tp_group=ps.tp_group)
    load_hf_state_dict(model, hf_state_dict(ref))          # TP shards of the reference weights
    eng = TPREngine(cfg, EngineConfig(tensor_model_parallel_size=2, context_parallel_size=2, tpr_cp_backend=backend),
                    device="cpu", model=model, parallel_state=ps)
    out = eng.forward_backward_batch(batch)
    # expected TP-sharded gradients: the reference gradients sharded by the same HF -> Megatron loader
    import copy

    gm = copy.deepcopy(ref)
    with torch.no_grad():
        for (_, pg), (_, pr) in zip(gm.named_parameters(), ref.named_parameters()):
            pg.copy_(pr.grad)
    holder = build_model(cfg, dtype=torch.float32, seed=2, tp_group=ps.tp_group)
    load_hf_state_dict(holder, hf_state_dict(gm))
    expected = dict(holder.named_parameters())
    errs = {}
    for n, p in eng.model.named_parameters():
        g_ref = expected[n].detach()
        errs[n] = float((p.main_grad - g_ref).norm() / (g_ref.norm() + 1e-12))
    return {"loss": out["loss"][0], "loss_ref": float(loss_ref), "grad_rel": errs}


@pytest.mark.parametrize("backend", ["ring", "allgather"])
def test_tp2_cp2_matches_flattened(backend):
    """TP x CP together (the flagship layout's axes) against the flattened batch, FP32 on gloo."""
    res = run_ranks(4, _tpcp_worker, backend)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst

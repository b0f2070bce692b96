"""Hybrid GDN/attention and hybrid MoE models through TPR (GDN state relay) vs the flattened batch;
checkpoint round trip; activation offload scope (CPU, FP32)."""

import os

import pytest
import torch

from bridge_b200.engine import EngineConfig, TPREngine
from bridge_b200.models import get_config
from bridge_b200.models.decoder import build_model
from tests.helpers import flat_ppo_loss, rel_err, set_old_log_probs, tree_batch


@pytest.mark.parametrize("preset", ["tiny_hybrid", "tiny_moe"])
@pytest.mark.parametrize("executor,mode", [("forest", "retain"), ("forest", "recompute"), ("segment", "retain")])
def test_hybrid_models_tpr_match_flattened(preset, executor, mode):
    cfg = get_config(preset)
    batch = tree_batch(n_trees=2, prefix=48, siblings=3, resp=16, seed=7)
    ref = build_model(cfg, dtype=torch.float32, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    eng = TPREngine(cfg, EngineConfig(executor=executor, forest_mode=mode, token_budget=80), device="cpu",
                    model=build_model(cfg, dtype=torch.float32, seed=0))
    out = eng.forward_backward_batch(batch)
    assert abs(out["loss"][0] - float(loss_ref)) < 1e-5 * max(1, abs(float(loss_ref)))
    for n, p in eng.model.named_parameters():
        g = dict(ref.named_parameters())[n].grad
        if g is None:
            assert float(p.main_grad.abs().max()) == 0.0, n
            continue
        assert rel_err(p.main_grad, g) < 2e-4, n


def test_deep_session_tree_relays_through_three_levels():
    """A multi-turn session: prompt -> turn1 fork -> turn2 fork (depth 3), exact trie."""
    g = torch.Generator().manual_seed(11)
    p = torch.randint(0, 1024, (24,), generator=g)
    t1 = [torch.randint(0, 1024, (12,), generator=g) for _ in range(2)]
    rows, masks = [], []
    for a in range(2):
        for b in range(2):
            tail = torch.randint(0, 1024, (10,), generator=g)
            ids = torch.cat([p, t1[a], tail])
            rows.append(ids)
            m = torch.zeros(22, dtype=torch.bool)
            m[-10:] = True
            m[2:8] = True
            masks.append(m)
    batch = {"input_ids": rows, "response_mask": masks, "old_log_probs": [torch.zeros(22)] * 4,
             "advantages": [torch.randn(22, generator=g) for _ in range(4)], "uid": ["s"] * 4, "temperature": 1.0,
             "dp_size": 1}
    batch["batch_num_tokens"] = int(sum(int(m.sum()) for m in masks))
    for preset in ("tiny", "tiny_hybrid"):
        cfg = get_config(preset)
        ref = build_model(cfg, dtype=torch.float32, seed=0)
        set_old_log_probs(ref, batch)
        loss_ref, _ = flat_ppo_loss(ref, batch)
        loss_ref.backward()
        for budget in (1000, 30):
            eng = TPREngine(cfg, EngineConfig(token_budget=budget), device="cpu",
                            model=build_model(cfg, dtype=torch.float32, seed=0))
            out = eng.forward_backward_batch(batch)
            assert out["metrics"]["tpr/physical_segments"] == [7]
            assert abs(out["loss"][0] - float(loss_ref)) < 1e-5
            for n, prm in eng.model.named_parameters():
                gref = dict(ref.named_parameters())[n].grad
                assert rel_err(prm.main_grad, gref) < 2e-4, (preset, budget, n)


def test_checkpoint_round_trip(tmp_path):
    from bridge_b200.models.checkpoint import hf_state_dict, load_checkpoint, save_checkpoint

    for preset in ("tiny", "tiny_moe"):
        cfg = get_config(preset)
        eng = TPREngine(cfg, EngineConfig(), device="cpu", model=build_model(cfg, dtype=torch.float32, seed=1))
        d = os.path.join(tmp_path, preset)
        eng.optimizer.step_count = 7
        save_checkpoint(d, eng, step=7)
        eng2 = TPREngine(cfg, EngineConfig(), device="cpu", model=build_model(cfg, dtype=torch.float32, seed=2))
        assert load_checkpoint(d, eng2) == 7 and eng2.optimizer.step_count == 7
        a, b = hf_state_dict(eng.model), hf_state_dict(eng2.model)
        assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)
        if preset == "tiny":
            assert "model.layers.0.self_attn.q_proj.weight" in a and "model.layers.1.mlp.down_proj.weight" in a


def test_activation_offload_scope_preserves_gradients():
    from bridge_b200.tpr.activation_offload import OffloadConfig, offload_scope

    cfg = get_config("tiny")
    model = build_model(cfg, dtype=torch.float32, seed=0)
    ids = torch.randint(0, 1024, (40,))
    pos = torch.arange(40)
    model(ids, pos).pow(2).mean().backward()
    ref = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad()
    with offload_scope(model, OffloadConfig(enabled=True, min_bytes=1)) as off:
        model(ids, pos).pow(2).mean().backward()
        # restored tensors belong to the backward that consumed them, not to the offloader (only a
        # prefetched tensor that no backward node read is still held, until the scope releases)
        left = sum(s.restored.numel() * s.restored.element_size() for lst in off.by_layer.values() for s in lst
                   if s.restored is not None)
        assert left <= 0.02 * off.offloaded_bytes, (left, off.offloaded_bytes)
    assert off.offloaded_bytes > 0
    for n, p in model.named_parameters():
        assert torch.allclose(p.grad, ref[n], atol=1e-6), n


@pytest.mark.parametrize("mode", ["retain", "recompute"])
@pytest.mark.parametrize("preset", ["tiny", "tiny_hybrid"])
def test_forest_splits_segments_longer_than_the_budget(mode, preset):
    """A token budget shorter than the prompt (128 tokens) cuts long segments into prefix chains: same
    loss and gradients as a budget that holds every segment whole."""
    from bridge_b200.engine import EngineConfig, TPREngine
    from tests.helpers import nested_tree_batch

    cfg = get_config(preset)
    batch = nested_tree_batch(prefix=128, mid=40, resp=24)
    out, grads = {}, {}
    for budget in (4096, 48):
        eng = TPREngine(cfg, EngineConfig(forest_mode=mode, token_budget=budget), device="cpu",
                        model=build_model(cfg, dtype=torch.float32, seed=0))
        res = eng.forward_backward_batch(batch)
        out[budget] = float(res["loss"][0])
        grads[budget] = {n: p.main_grad.clone() for n, p in eng.model.named_parameters()}
    assert abs(out[48] - out[4096]) <= 1e-5 * abs(out[4096]) + 1e-7, out
    for n, g in grads[4096].items():
        assert torch.allclose(grads[48][n], g, rtol=1e-4, atol=1e-6), n


def test_offload_host_arena_reuses_slabs(monkeypatch):
    """Saved tensors of every size and dtype share pinned slabs; scopes of different chunk shapes reuse
    the slabs a released scope handed back instead of allocating new host memory."""
    from bridge_b200.tpr import activation_offload as ao

    monkeypatch.setenv("TPR_OFFLOAD_SLAB_BYTES", str(1 << 16))
    monkeypatch.setattr(ao, "_SLABS", ao._PinnedSlabs())
    for rows in (37, 53, 29, 61, 41):               # a different chunk shape per scope
        arena = ao._HostArena()
        got = []
        for dtype, cols in ((torch.float32, 64), (torch.bfloat16, 96), (torch.int64, 8), (torch.float32, 1)):
            src = torch.randn(rows, cols).to(dtype) if dtype != torch.int64 else torch.arange(rows * cols)
            h = arena.alloc(src.numel(), src.dtype)
            assert h.dtype == src.dtype and h.numel() == src.numel() and h.data_ptr() % 64 == 0
            h.copy_(src.reshape(-1))
            got.append((h, src))
        big = arena.alloc(3 << 15, torch.float32)     # larger than one slab: a slab of its own
        big.fill_(1.0)
        for h, src in got:                             # no two tensors overlap
            assert torch.equal(h.view(src.shape), src)
        arena.release()
    # two slabs at most were ever live at once, plus the big one
    assert len(ao._SLABS.free) <= 3, [s.numel() for s in ao._SLABS.free]


@pytest.mark.parametrize("mode", ["retain", "recompute"])
def test_forest_activation_offload_preserves_gradients(mode, monkeypatch):
    """EngineConfig.activation_offload reaches the forest executor: same loss and gradients, and the
    saved activations of leaf and retained push chunks go through the offloader."""
    from bridge_b200.engine import EngineConfig, TPREngine
    from tests.helpers import nested_tree_batch

    monkeypatch.setenv("TPR_OFFLOAD_MIN_BYTES", "4096")
    cfg = get_config("tiny")
    out, grads = {}, {}
    for off in (False, True):
        eng = TPREngine(cfg, EngineConfig(activation_offload=off, forest_mode=mode, token_budget=160), device="cpu",
                        model=build_model(cfg, dtype=torch.float32, seed=0))
        res = eng.forward_backward_batch(nested_tree_batch())
        out[off] = res["loss"][0]
        grads[off] = {n: p.main_grad.clone() for n, p in eng.model.named_parameters()}
        if off:
            assert res["metrics"]["tpr/offloaded_bytes"][0] > 0
    assert out[True] == out[False]
    for n in grads[False]:
        assert torch.equal(grads[True][n], grads[False][n]), n


def test_truncated_hybrid_config_keeps_layer_pattern():
    """``get_config(name, num_layers=n)`` on a hybrid preset keeps the first n entries of its layer pattern
    (bench.py --num-layers relies on it) and refuses more layers than the pattern defines."""
    full = get_config("qwen3_next_24l")
    cut = get_config("qwen3_next_24l", num_layers=8)
    assert cut.num_layers == 8 and cut.layer_types == full.layer_types[:8]
    assert cut.num_experts == full.num_experts and cut.attention_layer_numbers == (4, 8)
    with pytest.raises(ValueError):
        get_config("tiny_hybrid", num_layers=5)


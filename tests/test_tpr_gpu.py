"""On the GPU (bf16, sm_100a kernels): TPR log-probs / loss / grads vs the flattened non-TPR batch."""

import pytest
import torch

from tests.helpers import flat_ppo_loss, set_old_log_probs, tree_batch

pytestmark = pytest.mark.gpu


def _cfg():
    from bridge_b200.models import get_config

    return get_config("tiny", hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=1024,
                      num_layers=3)


def _cos(a, b):
    return float(torch.nn.functional.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0))


@pytest.mark.parametrize("mode", ["retain", "recompute"])
def test_tpr_vs_flat_bf16(mode):
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models.decoder import build_model

    dev = torch.device("cuda")
    batch = tree_batch(n_trees=2, prefix=200, siblings=4, resp=96, seed=5)
    ref = build_model(_cfg(), device=dev, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    eng = TPREngine(_cfg(), EngineConfig(forest_mode=mode, token_budget=1024), device=dev,
                    model=build_model(_cfg(), device=dev, seed=0))
    out = eng.forward_backward_batch(batch)
    assert abs(out["loss"][0] - float(loss_ref)) <= 2e-3 * abs(float(loss_ref)) + 1e-4
    gr = {n: p.grad for n, p in ref.named_parameters()}
    for n, p in eng.model.named_parameters():
        a, b = p.main_grad.float(), gr[n].float()
        rel = float((a - b).norm() / (b.norm() + 1e-12))
        assert rel < 3e-2 and _cos(a, b) > 0.999, (n, rel)


def test_bench_cli_small():
    import json
    import subprocess
    import sys

    out = subprocess.run([sys.executable, "bench.py", "--model", "tiny", "--steps", "2", "--warmup", "1",
                          "--trees-per-gpu", "2", "--prefix", "64", "--siblings", "3", "--resp", "32"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["value"] > 0 and line["gpu_launches"] > 0 and line["n_gpus"] == 1


@pytest.mark.parametrize("preset,head_dim", [("tiny_hybrid", 128), ("tiny_hybrid", 256), ("tiny_moe", 128)])
def test_hybrid_tpr_vs_flat_bf16(preset, head_dim):
    """Hybrid GDN/attention (and hybrid MoE) on the GPU kernels: conv + gated delta rule state relay."""
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model

    cfg = get_config(preset, hidden_size=512, num_heads=4, num_kv_heads=2, head_dim=head_dim, gdn_num_qk_heads=2,
                     gdn_num_v_heads=4, gdn_head_dim=64)
    dev = torch.device("cuda")
    batch = tree_batch(n_trees=2, prefix=150, siblings=3, resp=70, seed=9)
    ref = build_model(cfg, device=dev, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    eng = TPREngine(cfg, EngineConfig(token_budget=512), device=dev, model=build_model(cfg, device=dev, seed=0))
    out = eng.forward_backward_batch(batch)
    gr = {n: p.grad for n, p in ref.named_parameters()}
    # The PPO loss is a token mean of +-A * ratio terms that nearly cancel; the GDN kernels' bf16
    # tensor-core intermediates round differently when TPR moves the chunk boundaries, so the loss is
    # compared against the size of its terms (mean |A|), not its cancelled value.
    scale = float(torch.cat([a[m] for a, m in zip(batch["advantages"], batch["response_mask"])]).abs().mean())
    if cfg.is_moe:
        # bf16 rounding also flips near-tied top-k routes between the two layouts: compare in aggregate
        assert abs(out["loss"][0] - float(loss_ref)) <= 3e-3 * scale
        names = [n for n, _ in eng.model.named_parameters() if gr[n] is not None]
        a = torch.cat([dict(eng.model.named_parameters())[n].main_grad.float().flatten() for n in names])
        b = torch.cat([gr[n].float().flatten() for n in names])
        assert _cos(a, b) > 0.99
        return
    assert abs(out["loss"][0] - float(loss_ref)) <= 1e-3 * scale
    # Per-head scalars (A_log, dt_bias: a handful of values, each a long cancelling token sum) carry
    # far more bf16 noise than the matrices, in the flat path as much as in TPR.  They are judged
    # against an FP32 CPU run of the same weights: TPR may not be much noisier than the flat path.
    small = {n for n, p in eng.model.named_parameters() if p.numel() < 64 and gr[n] is not None}
    if small:
        ref32 = build_model(cfg, device="cpu", seed=0, dtype=torch.float32)
        ref32.load_state_dict({k: v.detach().float().cpu() for k, v in ref.state_dict().items()})
        loss32, _ = flat_ppo_loss(ref32, batch)
        loss32.backward()
        g32 = {n: p.grad for n, p in ref32.named_parameters()}
    for n, p in eng.model.named_parameters():
        b = gr[n]
        if b is None:
            continue
        a = p.main_grad.float()
        if n in small:
            e_tpr = float((a.cpu() - g32[n]).norm())
            e_flat = float((b.float().cpu() - g32[n]).norm())
            assert e_tpr <= 2 * e_flat + 0.05 * float(g32[n].norm()), (n, e_tpr, e_flat)
            continue
        rel = float((a - b.float()).norm() / (b.float().norm() + 1e-12))
        assert rel < 5e-2 and _cos(a, b) > 0.998, (n, rel)


@pytest.mark.parametrize("mode", ["retain", "recompute"])
def test_forest_activation_offload_gpu(mode, monkeypatch):
    """Activation offload through the engine on the GPU: same loss and gradients (within bf16 / atomic
    reordering), saved tensors really moved to pinned host memory, and a lower device peak.

    The forward of this model produces activations faster than PCIe drains them, so the device bytes
    whose host copy is still pending are capped well below the chunk's activations: without the cap a
    chunk that is forwarded and back-propagated at once (every leaf chunk, and every chunk in recompute
    mode) would hold all of them until the backward."""
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models.decoder import build_model

    from bridge_b200.models import get_config

    monkeypatch.setenv("TPR_OFFLOAD_INFLIGHT_BYTES", str(256 << 20))
    dev = torch.device("cuda")
    # deep and wide enough that the saved activations, not the weights or the LM head, set the peak
    cfg = get_config("tiny", hidden_size=1024, num_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=4096,
                     num_layers=8)
    batch = tree_batch(n_trees=2, prefix=2048, siblings=4, resp=1024, seed=9)
    res, peaks, grads = {}, {}, {}
    for off in (False, True):
        eng = TPREngine(cfg, EngineConfig(forest_mode=mode, token_budget=8192, activation_offload=off),
                        device=dev, model=build_model(cfg, device=dev, seed=0))
        set_old_log_probs(eng.model, batch)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        res[off] = eng.forward_backward_batch(batch)
        torch.cuda.synchronize()
        peaks[off] = torch.cuda.max_memory_allocated() - base
        grads[off] = {n: p.main_grad.clone() for n, p in eng.model.named_parameters()}
        del eng
    assert res[True]["metrics"]["tpr/offloaded_bytes"][0] > 0
    assert abs(res[True]["loss"][0] - res[False]["loss"][0]) <= 1e-5 * abs(res[False]["loss"][0]) + 1e-7
    # the attention backward reduces prefix dK/dV with FP32 atomics (bf16 rounding flips between runs), so
    # the offloaded run is held to the same oracle as the plain one: the flattened non-TPR computation
    ref = build_model(cfg, device=dev, seed=0)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    gr = {n: p.grad.float() for n, p in ref.named_parameters()}
    for off in (False, True):
        assert abs(res[off]["loss"][0] - float(loss_ref)) <= 2e-3 * abs(float(loss_ref)) + 1e-4
        for n, g in grads[off].items():
            rel = float((g - gr[n]).norm() / (gr[n].norm() + 1e-12))
            assert rel < 3e-2 and _cos(g, gr[n]) > 0.999, (off, n, rel)
    for n, g in grads[False].items():
        rel = float((grads[True][n] - g).norm() / (g.norm() + 1e-12))
        assert rel < 1e-2, (n, rel)
    assert peaks[True] < peaks[False], peaks

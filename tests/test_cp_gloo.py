"""Config #1 gate: CP world_size 2 (gloo, FP32) -- TPR loss, log-probs and grads equal the flattened 4x192 batch,
for every context-parallel backend; hybrid (Ulysses x ring) at CP 4."""

import pytest
import torch

from tests.dist_utils import run_ranks


def _worker(rank, world, backend, n_layers, preset="tiny", prefix=128, resp=64, gdn_cp_mode="head",
            executor="segment"):
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
    ec = EngineConfig(context_parallel_size=world, tpr_cp_backend=backend, gdn_cp_mode=gdn_cp_mode,
                      executor=executor)
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


@pytest.mark.parametrize("prefix,resp", [(128, 64), (131, 63)])
def test_hybrid_gdn_cp2_sequence_sharded_matches_flattened(prefix, resp):
    """GDN layers sequence-sharded under ring CP (zigzag pieces, padding): exchanged per-piece state maps
    and conv halos, full-head state relayed between segments."""
    res = run_ranks(2, _worker, "ring", 4, "tiny_hybrid", prefix, resp, "sequence")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def _seq_layer_worker(rank, world):
    """forward_gdn_cp_sequence on contiguous shards vs the whole segment on one rank (FP32)."""
    import torch

    from bridge_b200.models import get_config
    from bridge_b200.models.layers import TPRGatedDeltaNet
    from bridge_b200.parallel.gdn_state import forward_gdn_cp_sequence
    from bridge_b200.tpr.prefix_state import GDNLayerState

    cfg = get_config("tiny_hybrid")
    torch.manual_seed(0)
    layer = TPRGatedDeltaNet(cfg, 1).float()
    L = 48
    x = torch.randn(world * L, cfg.hidden_size)
    cc = 2 * layer.hk * layer.dk + layer.hv * layer.dv
    h_conv = torch.randn(1, cc, layer.w)
    h_conv[:, :, 0] = 0
    h_rec = 0.1 * torch.randn(1, layer.hv, layer.dk, layer.dv)
    # reference: whole segment, one process
    xr, hc_r, hr_r = (t.clone().requires_grad_() for t in (x, h_conv, h_rec))
    ref_layer = TPRGatedDeltaNet(cfg, 1).float()
    ref_layer.load_state_dict(layer.state_dict())
    out_r, fin_r = _whole_segment(ref_layer, xr, GDNLayerState(hc_r, hr_r))
    w_out = torch.randn_like(out_r)
    w_rec = torch.randn_like(fin_r.recurrent_state)
    w_conv = torch.randn_like(fin_r.conv_state)
    ((out_r * w_out).sum() + (fin_r.recurrent_state * w_rec).sum() + (fin_r.conv_state * w_conv).sum()).backward()
    # sequence-sharded
    xs = x[rank * L:(rank + 1) * L].clone().requires_grad_()
    hc, hr = h_conv.clone().requires_grad_(), h_rec.clone().requires_grad_()
    out, fin = forward_gdn_cp_sequence(layer, xs, GDNLayerState(hc, hr), _world(), capture_final_state=True)
    loss = (out * w_out[rank * L:(rank + 1) * L]).sum()
    # the final state is replicated: one rank's copy carries the state loss, as in the single-process run
    if rank == 0:
        loss = loss + (fin.recurrent_state * w_rec).sum() + (fin.conv_state * w_conv).sum()
    loss.backward()
    # dh0 partials: rank 1 never reads the initial conv state (its halo is rank 0's tail)
    d_hc = hc.grad if hc.grad is not None else torch.zeros_like(hc)
    d_hr = hr.grad if hr.grad is not None else torch.zeros_like(hr)
    torch.distributed.all_reduce(d_hc)
    torch.distributed.all_reduce(d_hr)
    rel = lambda a, b: float((a - b).norm() / (b.norm() + 1e-12))  # noqa: E731
    errs = {"out": rel(out.detach(), out_r.detach()[rank * L:(rank + 1) * L]),
            "rec": rel(fin.recurrent_state.detach(), fin_r.recurrent_state.detach()),
            "conv": rel(fin.conv_state.detach(), fin_r.conv_state.detach()),
            "dx": rel(xs.grad, xr.grad[rank * L:(rank + 1) * L]),
            "dh_conv": rel(d_hc, hc_r.grad), "dh_rec": rel(d_hr, hr_r.grad)}
    pg = {n: (p.grad if p.grad is not None else torch.zeros_like(p)).clone() for n, p in layer.named_parameters()}
    for t in pg.values():
        torch.distributed.all_reduce(t)
    for n, p in ref_layer.named_parameters():
        errs["param:" + n] = rel(pg[n], p.grad)
    return errs


def _world():
    import torch.distributed as dist

    return dist.group.WORLD


def _whole_segment(layer, x, state):
    """The layer's own single-process path with an explicit initial state (no TPR context)."""
    from bridge_b200.ops.gdn import (causal_conv1d, chunk_gated_delta_rule, gated_rmsnorm, gdn_gates,
                                     l2norm)
    from bridge_b200.tpr.prefix_state import GDNLayerState

    t = x.shape[0]
    kd, vd = layer.hk * layer.dk, layer.hv * layer.dv
    qkv, z, b, a = layer.in_proj(x).split((2 * kd + vd, vd, layer.hv, layer.hv), dim=-1)
    y, conv_final = causal_conv1d(qkv, layer.conv_weight, None, [0, t], None, state.conv_state, activation=True)
    q, k, v = y.split((kd, kd, vd), dim=-1)
    q = l2norm(q.reshape(t, layer.hk, layer.dk))
    k = l2norm(k.reshape(t, layer.hk, layer.dk))
    v = v.reshape(t, layer.hv, layer.dv)
    if layer.hv // layer.hk > 1:
        q, k = q.repeat_interleave(layer.hv // layer.hk, 1), k.repeat_interleave(layer.hv // layer.hk, 1)
    g, beta = gdn_gates(a, b, layer.A_log, layer.dt_bias)
    o, rec = chunk_gated_delta_rule(q, k, v, g, beta, [0, t], None, state.recurrent_state, scale=layer.scale,
                                    chunk_size=layer.chunk)
    o = gated_rmsnorm(o, z.reshape(t, layer.hv, layer.dv), layer.norm_weight, layer.eps)
    return layer.out_proj(o.reshape(t, vd)), GDNLayerState(conv_final, rec)


def test_gdn_sequence_sharded_layer_matches_whole_segment():
    """Outputs, final conv / recurrent state and every gradient (input, parameters, dh0 of both states)."""
    for r in run_ranks(2, _seq_layer_worker):
        worst = max(r.items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def _tpcp_worker(rank, world, backend, preset="tiny", gdn_cp_mode="head", executor="segment", nested=False):
    import torch

    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel.groups import build_parallel_state
    from tests.helpers import flat_ppo_loss, set_old_log_probs, tree_batch

    from tests.helpers import nested_tree_batch

    cfg = get_config(preset, num_layers=2 if preset == "tiny" else 4)
    batch = nested_tree_batch() if nested else tree_batch(n_trees=1, prefix=128, siblings=4, resp=64, seed=0)
    ref = build_model(cfg, dtype=torch.float32, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    from bridge_b200.models.checkpoint import hf_state_dict, load_hf_state_dict

    ps = build_parallel_state(tp=2, cp=2)
    model = build_model(cfg, dtype=torch.float32, seed=1, tp_group=ps.tp_group, sequence_parallel=nested)
    load_hf_state_dict(model, hf_state_dict(ref))          # TP shards of the reference weights
    eng = TPREngine(cfg, EngineConfig(tensor_model_parallel_size=2, context_parallel_size=2, tpr_cp_backend=backend,
                                      gdn_cp_mode=gdn_cp_mode, executor=executor, token_budget=160,
                                      sequence_parallel=nested),
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


def test_tp2_cp2_hybrid_gdn_sequence_sharded_matches_flattened():
    """Config #4's axes on the hybrid model: TP2 x CP2 ring with sequence-sharded GDN (one key head per
    TP rank, which the head-parallel schedule cannot split over CP) against the flattened batch."""
    res = run_ranks(4, _tpcp_worker, "ring", "tiny_hybrid", "sequence")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_hybrid_gdn_cp4_sequence_sharded_matches_flattened():
    """GDN under ring CP4 (eight zigzag pieces chained through the exchanged state maps)."""
    res = run_ranks(4, _worker, "ring", 4, "tiny_hybrid", 64, 32, "sequence")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst



# --------------------------------------------------------------------------- forest executor under CP
def _forest_worker(rank, world, preset, n_layers, budget, mode):
    """Segment-granular CP in the batched forest executor vs the flattened batch (FP32, gloo): two
    two-level trees, a per-rank budget small enough that parents and children land on different ranks."""
    import torch

    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.parallel.groups import build_parallel_state
    from tests.helpers import flat_ppo_loss, nested_tree_batch, set_old_log_probs

    cfg = get_config(preset, num_layers=n_layers)
    batch = nested_tree_batch()
    ref = build_model(cfg, dtype=torch.float32, seed=0)
    set_old_log_probs(ref, batch)
    loss_ref, _ = flat_ppo_loss(ref, batch)
    loss_ref.backward()
    ps = build_parallel_state(tp=1, cp=world)
    model = build_model(cfg, dtype=torch.float32, seed=0)
    ec = EngineConfig(context_parallel_size=world, tpr_cp_backend="ring", executor="forest", token_budget=budget,
                      forest_mode=mode)
    eng = TPREngine(cfg, ec, device="cpu", model=model, parallel_state=ps)
    out = eng.forward_backward_batch(batch)
    errs = {}
    for n, p in eng.model.named_parameters():
        g_ref = dict(ref.named_parameters())[n].grad
        errs[n] = float((p.main_grad - g_ref).norm() / (g_ref.norm() + 1e-12))
    return {"loss": out["loss"][0], "loss_ref": float(loss_ref), "grad_rel": errs,
            "chunks": out["metrics"]["tpr/chunks"][0]}


@pytest.mark.parametrize("mode", ["retain", "recompute"])
def test_forest_cp2_matches_flattened(mode):
    res = run_ranks(2, _forest_worker, "tiny", 2, 160, mode)
    for r in res:
        assert r["chunks"] >= 3, r
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_forest_cp2_hybrid_gdn_matches_flattened():
    """GDN final states of pushed segments are gathered over CP and seed children on the other rank."""
    res = run_ranks(2, _forest_worker, "tiny_hybrid", 4, 160, "retain")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


@pytest.mark.parametrize("preset,layers", [("tiny", 2), ("tiny_hybrid", 4)])
def test_forest_cp2_splits_long_segments_matches_flattened(preset, layers):
    """A per-rank budget (48) below the prompt length (128): long segments become prefix chains whose
    pieces are placed whole on CP ranks (K/V and GDN states of earlier pieces gathered like any prefix)."""
    res = run_ranks(2, _forest_worker, preset, layers, 48, "recompute")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_forest_cp3_idle_rank_matches_flattened():
    """More ranks than segments at some level: an idle rank forwards a pad segment and still joins every
    collective."""
    res = run_ranks(3, _forest_worker, "tiny", 2, 4096, "retain")
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_forest_tp2_cp2_sequence_parallel_matches_flattened():
    """BASELINE config #2's axes through the forest executor: TP2 (sequence parallel) x CP2."""
    res = run_ranks(4, _tpcp_worker, "ring", "tiny", "head", "forest", True)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def test_forest_tp2_cp2_sequence_parallel_hybrid_matches_flattened():
    """BASELINE config #4's axes through the forest executor: the hybrid GDN model at TP2 (sequence
    parallel: the GDN projections gather / scatter the token shard) x CP2 (GDN states gathered over CP)."""
    res = run_ranks(4, _tpcp_worker, "ring", "tiny_hybrid", "head", "forest", True)
    for r in res:
        assert abs(r["loss"] - r["loss_ref"]) < 1e-5 * max(1.0, abs(r["loss_ref"])), r
        worst = max(r["grad_rel"].items(), key=lambda kv: kv[1])
        assert worst[1] < 1e-4, worst


def _ordinary_ring_worker(rank, world, length):
    """Whole-sequence causal ring attention on zigzag shards vs full FP32 causal attention."""
    import torch
    import torch.distributed as dist

    from bridge_b200.parallel.ring_attention import ordinary_ring_cp_attention
    from bridge_b200.tpr.shard import make_ring_sequence_shard

    g = torch.Generator().manual_seed(5)
    hq, hkv, d = 4, 2, 16
    q = torch.randn(length, hq, d, generator=g)
    k = torch.randn(length, hkv, d, generator=g)
    v = torch.randn(length, hkv, d, generator=g)
    do = torch.randn(length, hq, d, generator=g)
    # reference: causal attention over the whole sequence (GQA)
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    s = torch.einsum("qhd,khd->hqk", qr, kr.repeat_interleave(hq // hkv, 1)) * d ** -0.5
    mask = torch.ones(length, length, dtype=torch.bool).tril()
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), -1)
    o_ref = torch.einsum("hqk,khd->qhd", p, vr.repeat_interleave(hq // hkv, 1))
    (o_ref * do).sum().backward()
    shard = make_ring_sequence_shard(length, cp_rank=rank, cp_size=world)
    # physical rows of this rank (padding rows past the sequence end carry zeros and no loss)
    idx = torch.cat([torch.arange(a, b) for a, b in shard.physical_global_ranges])
    valid = idx < length
    pick = lambda t: torch.where(valid[:, None, None], t[idx.clamp(max=length - 1)], torch.zeros(()))  # noqa: E731
    ql, kl, vl = (pick(t).clone().requires_grad_(True) for t in (q, k, v))
    o = ordinary_ring_cp_attention(ql, kl, vl, cp_group=dist.group.WORLD, global_length=length)
    (o * pick(do)).sum().backward()
    sel = valid
    err = lambda a, b: float((a[sel] - b[idx[sel]]).abs().max())  # noqa: E731
    return {"o": err(o.detach(), o_ref.detach()), "dq": err(ql.grad, qr.grad),
            # dK/dV of each key arrive at its owner rank after the ring; compare the owned rows
            "dk": err(kl.grad, kr.grad), "dv": err(vl.grad, vr.grad)}


@pytest.mark.parametrize("length", [40, 37])
def test_ordinary_ring_matches_full_causal_attention(length):
    """The whole-sequence ring entry (no external prefix), padded and unpadded zigzag shards."""
    for r in run_ranks(2, _ordinary_ring_worker, length):
        assert max(r.values()) < 1e-4, r

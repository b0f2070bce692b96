"""Gated DeltaNet kernels (causal conv1d, chunked gated delta rule) vs PyTorch FP32 references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, atol, rtol, name=""):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    tol = atol + rtol * b.abs().max().item()
    assert err <= tol, f"{name}: max err {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("W", [4, 3, 2])
@pytest.mark.parametrize("with_h0,with_bias,with_dht", [(True, False, True), (False, True, False),
                                                        (True, True, False)])
@pytest.mark.parametrize("bwd", ["stream2", "v1"])
def test_causal_conv1d(W, with_h0, with_bias, with_dht, bwd, monkeypatch):
    """Forward and both backward kernels (two-channel streaming default, one-channel v1)."""
    from bridge_b200.ops.gdn import causal_conv1d, causal_conv1d_reference

    if bwd == "v1":
        monkeypatch.setenv("BB_CONV_BWD_V1", "1")

    torch.manual_seed(W)
    lens = [100, 2, 64, 131, 1, 70]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    C, B = 384, len(lens)
    x = torch.randn(cu[-1], C, device=DEV).to(torch.bfloat16)
    w = (0.5 * torch.randn(C, W, device=DEV)).to(torch.bfloat16)
    bias = (0.1 * torch.randn(C, device=DEV)).to(torch.bfloat16) if with_bias else None
    h0 = None
    if with_h0:
        h0 = torch.randn(B, C, W, device=DEV).to(torch.bfloat16)
        h0[:, :, 0] = 0
    leaves = [t.detach().clone().requires_grad_() if t is not None else None for t in (x, w, bias, h0)]
    y, hT = causal_conv1d(leaves[0], leaves[1], leaves[2], cu, None, leaves[3], activation=True)
    refs = [t.detach().float().requires_grad_() if t is not None else None for t in (x, w, bias, h0)]
    yr, hTr = causal_conv1d_reference(refs[0], refs[1], refs[2], cu, refs[3], activation=True)
    _close(y, yr, 2e-2, 1e-2, "y")
    _close(hT, hTr, 1e-6, 0, "final state")
    dy = torch.randn_like(yr)
    dh = torch.randn_like(hTr) if with_dht else torch.zeros_like(hTr)
    dh[:, :, 0] = 0
    (y.float() * dy).sum().add_((hT.float() * dh).sum()).backward()
    (yr * dy).sum().add_((hTr * dh).sum()).backward()
    for name, a, b in zip(("dx", "dw", "db", "dh0"), leaves, refs):
        if a is not None:
            _close(a.grad, b.grad, 3e-2, 2e-2, name)


def _gdr_inputs(lens, H, K, V, with_h0, seed=0):
    from bridge_b200.ops.gdn import l2norm

    g = torch.Generator(device=DEV).manual_seed(seed)
    T = sum(lens)
    q = l2norm(torch.randn(T, H, K, device=DEV, generator=g)).to(torch.bfloat16)
    k = l2norm(torch.randn(T, H, K, device=DEV, generator=g)).to(torch.bfloat16)
    v = torch.randn(T, H, V, device=DEV, generator=g).to(torch.bfloat16)
    gate = -torch.nn.functional.softplus(torch.randn(T, H, device=DEV, generator=g)) * 0.5
    beta = torch.sigmoid(torch.randn(T, H, device=DEV, generator=g))
    h0 = 0.2 * torch.randn(len(lens), H, K, V, device=DEV, generator=g) if with_h0 else None
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return q, k, v, gate, beta, h0, cu


@pytest.mark.parametrize("K,V,H", [(128, 128, 4), (64, 64, 2), (32, 64, 3)])
@pytest.mark.parametrize("with_h0", [True, False])
def test_gated_delta_rule_forward_backward(K, V, H, with_h0):
    from bridge_b200.ops.gdn import chunk_gated_delta_rule, chunk_gated_delta_rule_reference

    lens = [150, 1, 64, 200, 37]
    q, k, v, gate, beta, h0, cu = _gdr_inputs(lens, H, K, V, with_h0, seed=K + H)
    scale = K ** -0.5
    xs = [t.detach().clone().requires_grad_() if t is not None else None for t in (q, k, v, gate, beta, h0)]
    o, hT = chunk_gated_delta_rule(*xs[:5], cu, None, xs[5], scale=scale)
    rs = [t.detach().float().requires_grad_() if t is not None else None for t in (q, k, v, gate, beta, h0)]
    orr, hTr = chunk_gated_delta_rule_reference(*rs[:5], cu, rs[5], scale=scale, chunk_size=64)
    _close(o, orr, 1e-2, 1e-2, "o")
    # the tensor cores see the chunk states as bf16 operands (FP32 accumulation), so the chained
    # final state carries bf16-level error
    _close(hT, hTr, 3e-3, 1e-2, "final state")
    do = torch.randn_like(orr)
    dh = torch.randn_like(hTr)
    ((o.float() * do).sum() + (hT * dh).sum()).backward()
    ((orr * do).sum() + (hTr * dh).sum()).backward()
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), xs, rs):
        if a is not None:
            _close(a.grad, b.grad, 2e-2, 2e-2, name)
    # no systematic bias: per-head token sums of dg (what a per-head decay parameter's gradient is)
    sa, sr = xs[3].grad.float().sum(0), rs[3].grad.float().sum(0)
    mass = rs[3].grad.float().abs().sum(0)
    assert bool(((sa - sr).abs() <= 1e-2 * mass + 1e-3).all()), (sa, sr, mass)


def test_gated_delta_rule_matches_recurrence():
    """The chunked kernel against the naive per-token recurrence (FP32 oracle)."""
    from bridge_b200.ops.gdn import chunk_gated_delta_rule, gated_delta_rule_recurrent

    q, k, v, gate, beta, h0, cu = _gdr_inputs([300], 2, 128, 128, True, seed=7)
    o, hT = chunk_gated_delta_rule(q, k, v, gate, beta, cu, None, h0, scale=0.1)
    orr, Sr = gated_delta_rule_recurrent(q.float(), k.float(), v.float(), gate, beta, h0[0], scale=0.1)
    _close(o, orr, 1e-2, 1e-2, "o")
    _close(hT[0], Sr, 3e-3, 1e-2, "state")


@pytest.mark.parametrize("D", [128, 64, 256])
def test_l2norm_strided_heads(D):
    """Fused L2 norm on a column slice of a wider projection (the conv output layout) vs FP32."""
    from bridge_b200.ops.gdn import l2norm, l2norm_reference

    torch.manual_seed(D)
    T, H = 333, 3
    base = torch.randn(T, 2 * H * D + 40, device=DEV).to(torch.bfloat16)
    x = base[:, H * D:2 * H * D].reshape(T, H, D).detach().requires_grad_()
    xr = x.detach().float().requires_grad_()
    y = l2norm(x)
    yr = l2norm_reference(xr)
    assert y.is_contiguous()
    _close(y, yr, 1e-2, 1e-2, "y")
    dy = torch.randn_like(yr)
    (y.float() * dy).sum().backward()
    (yr * dy).sum().backward()
    _close(x.grad, xr.grad, 2e-2, 1e-2, "dx")


@pytest.mark.parametrize("D", [128, 64])
def test_gated_rmsnorm_matches_fp32(D):
    from bridge_b200.ops.gdn import gated_rmsnorm, gated_rmsnorm_reference

    torch.manual_seed(D + 1)
    T, H = 517, 4
    o = torch.randn(T, H, D, device=DEV).to(torch.bfloat16).requires_grad_()
    proj = torch.randn(T, H * D + 24, device=DEV).to(torch.bfloat16)
    z = proj[:, 8:8 + H * D].reshape(T, H, D).detach().requires_grad_()
    w = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_()
    y = gated_rmsnorm(o, z, w, 1e-6)
    refs = [t.detach().float().requires_grad_() for t in (o, z, w)]
    yr = gated_rmsnorm_reference(*refs, 1e-6)
    _close(y, yr, 2e-2, 1e-2, "y")
    dy = torch.randn_like(yr)
    (y.float() * dy).sum().backward()
    (yr * dy).sum().backward()
    for name, a, b in zip(("do", "dz", "dw"), (o, z, w), refs):
        _close(a.grad, b.grad, 3e-2, 1e-2, name)


def test_gdn_gates_matches_fp32():
    from bridge_b200.ops.gdn import gdn_gates, gdn_gates_reference

    torch.manual_seed(7)
    T, H = 1000, 16
    proj = (2 * torch.randn(T, 3 * H + 16, device=DEV)).to(torch.bfloat16)
    a = proj[:, 16:16 + H].detach().requires_grad_()
    b = proj[:, 16 + H:16 + 2 * H].detach().requires_grad_()
    A_log = torch.log(torch.empty(H, device=DEV).uniform_(1, 16)).requires_grad_()
    dt = (0.5 * torch.randn(H, device=DEV)).requires_grad_()
    g, beta = gdn_gates(a, b, A_log, dt)
    refs = [t.detach().float().requires_grad_() for t in (a, b, A_log, dt)]
    gr, br = gdn_gates_reference(*refs)
    assert g.dtype == torch.float32 and beta.dtype == torch.float32
    _close(g, gr, 1e-4, 1e-5, "g")
    _close(beta, br, 1e-6, 1e-5, "beta")
    dg, db = torch.randn_like(gr), torch.randn_like(br)
    ((g * dg).sum() + (beta * db).sum()).backward()
    ((gr * dg).sum() + (br * db).sum()).backward()
    for name, x, r in zip(("da", "db", "dA_log", "ddt"), (a, b, A_log, dt), refs):
        _close(x.grad, r.grad, 1e-3, 1e-2, name)


def _seq_gpu_worker(rank, world):
    """One-rank sequence-sharded GDN on the GPU: O = O0 + O_I S0 and S_end = M S0 + C from the two
    tensor-core passes (the identity pass runs the (K, K) kernel) vs the direct stateful path."""
    import torch
    import torch.distributed as dist

    from bridge_b200.models import get_config
    from bridge_b200.models.layers import TPRGatedDeltaNet
    from bridge_b200.parallel.gdn_state import forward_gdn_cp_sequence
    from bridge_b200.tpr.prefix_state import GDNLayerState
    from tests.test_cp_gloo import _whole_segment

    group = dist.new_group(ranks=[0], backend="nccl")
    dev = torch.device("cuda", 0)
    cfg = get_config("tiny_hybrid", gdn_head_dim=64)
    torch.manual_seed(0)
    layer = TPRGatedDeltaNet(cfg, 1, device=dev)
    ref = TPRGatedDeltaNet(cfg, 1, device=dev)
    ref.load_state_dict(layer.state_dict())
    T = 200
    x = torch.randn(T, cfg.hidden_size, device=dev).to(torch.bfloat16)
    cc = 2 * layer.hk * layer.dk + layer.hv * layer.dv
    h_conv = torch.randn(1, cc, layer.w, device=dev).to(torch.bfloat16)
    h_conv[:, :, 0] = 0
    h_rec = 0.2 * torch.randn(1, layer.hv, layer.dk, layer.dv, device=dev)
    outs = {}
    for name, mod in (("seq", layer), ("ref", ref)):
        xs, hc, hr = (t.clone().requires_grad_() for t in (x, h_conv, h_rec))
        if name == "seq":
            o, fin = forward_gdn_cp_sequence(mod, xs, GDNLayerState(hc, hr), group)
        else:
            o, fin = _whole_segment(mod, xs, GDNLayerState(hc, hr))
        g = torch.Generator(device=dev).manual_seed(1)
        wo = torch.randn(o.shape, device=dev, generator=g)
        wr = torch.randn(fin.recurrent_state.shape, device=dev, generator=g)
        ((o.float() * wo).sum() + (fin.recurrent_state.float() * wr).sum()).backward()
        outs[name] = {"o": o.detach().float(), "rec": fin.recurrent_state.detach().float(),
                      "conv": fin.conv_state.detach().float(), "dx": xs.grad.float(), "dh_rec": hr.grad.float(),
                      "dh_conv": hc.grad.float(), **{"p:" + n: p.grad.float() for n, p in mod.named_parameters()}}
    return {k: float((outs["seq"][k] - outs["ref"][k]).norm() / (outs["ref"][k].norm() + 1e-12))
            for k in outs["ref"]}


def test_gdn_sequence_sharded_gpu_kernels():
    from tests.dist_utils import run_ranks

    (errs,) = run_ranks(1, _seq_gpu_worker)
    worst = max(errs.items(), key=lambda kv: kv[1])
    # bf16 activations; the identity pass adds one bf16 rounding of O_I before the FP32 correction
    assert worst[1] < 3e-2, errs

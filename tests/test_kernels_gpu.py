"""Numerics of every sm_100a kernel against a plain PyTorch FP32 reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, atol, rtol, name=""):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    tol = atol + rtol * b.abs().max().item()
    assert err <= tol, f"{name}: max err {err:.3e} > {tol:.3e}"


def test_extension_loaded():
    from bridge_b200 import _C

    assert hasattr(_C, "tree_attn_fwd") and hasattr(_C, "launch_count")


@pytest.mark.parametrize("rows,H", [(257, 2560), (64, 512), (3, 4096)])
def test_rmsnorm(rows, H):
    from bridge_b200.ops.norm import rmsnorm, rmsnorm_reference

    x = torch.randn(rows, H, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16).requires_grad_()
    y = rmsnorm(x, w, 1e-6)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = rmsnorm_reference(xr, wr, 1e-6)
    _close(y, yr, 2e-2, 1e-2, "y")
    g = torch.randn_like(yr)
    y.backward(g.to(y.dtype))
    yr.backward(g)
    _close(x.grad, xr.grad, 3e-2, 2e-2, "dx")
    _close(w.grad, wr.grad, 1e-1, 2e-2, "dw")


@pytest.mark.parametrize("rows,H", [(1000, 2560), (333, 64), (97, 4096), (50, 1000)])
def test_add_rmsnorm(rows, H):
    """Residual add fused into RMSNorm: h, y and the shared gradient of both addends vs FP32."""
    from bridge_b200.ops.norm import add_rmsnorm, rmsnorm_reference

    torch.manual_seed(rows + H)
    x = torch.randn(rows, H, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(rows, H, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16).requires_grad_()
    h, y = add_rmsnorm(x, r, w, 1e-6)
    xr, rr, wr = (t.detach().float().requires_grad_() for t in (x, r, w))
    hr = xr + rr
    yr = rmsnorm_reference(hr, wr, 1e-6)
    _close(h, hr, 2e-2, 1e-2, "h")
    _close(y, yr, 2e-2, 1e-2, "y")
    gh, gy = torch.randn_like(hr), torch.randn_like(yr)
    ((h.float() * gh).sum() + (y.float() * gy).sum()).backward()
    ((hr * gh).sum() + (yr * gy).sum()).backward()
    _close(x.grad, xr.grad, 3e-2, 2e-2, "dx")
    _close(r.grad, rr.grad, 3e-2, 2e-2, "dres")
    _close(w.grad, wr.grad, 1e-1, 2e-2, "dw")


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("fused_view", [False, True])
def test_qk_norm_rope(D, fused_view):
    """Contiguous q/k, and q/k read in place as column slices of a fused [q+gate | k | v] projection."""
    from bridge_b200.ops.norm import qk_norm_rope, qk_norm_rope_reference, rope_cos_sin

    T, Hq, Hk = 77, 8, 2
    if fused_view:
        qkv = torch.randn(T, Hq * 2 * D + 2 * Hk * D, device=DEV, dtype=torch.bfloat16, requires_grad=True)
        q_all, k, _ = qkv.split((Hq * 2 * D, Hk * D, Hk * D), dim=-1)
        q = q_all.view(T, Hq, 2 * D)[..., :D]
        k = k.view(T, Hk, D)
        q.retain_grad()
        k.retain_grad()
    else:
        q = torch.randn(T, Hq, D, device=DEV, dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn(T, Hk, D, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    qw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16).requires_grad_()
    kw = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16).requires_grad_()
    cos, sin = rope_cos_sin(torch.arange(1000, 1000 + T, device=DEV), D, 1e6)
    qo, ko = qk_norm_rope(q, k, qw, kw, cos, sin, 1e-6)
    ref = [t.detach().float().requires_grad_() for t in (q, k, qw, kw)]
    qr, kr = qk_norm_rope_reference(ref[0], ref[1], ref[2], ref[3], cos, sin, 1e-6)
    _close(qo, qr, 2e-2, 1e-2, "q")
    _close(ko, kr, 2e-2, 1e-2, "k")
    gq, gk = torch.randn_like(qr), torch.randn_like(kr)
    torch.autograd.backward([qo, ko], [gq.bfloat16(), gk.bfloat16()])
    torch.autograd.backward([qr, kr], [gq, gk])
    for a, b, n in zip((q, k, qw, kw), ref, ("dq", "dk", "dqw", "dkw")):
        _close(a.grad, b.grad, 5e-2, 2e-2, n)


def test_swiglu():
    from bridge_b200.ops.activation import swiglu, swiglu_reference

    gu = torch.randn(133, 2 * 9728, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    y = swiglu(gu)
    gr = gu.detach().float().requires_grad_()
    yr = swiglu_reference(gr)
    _close(y, yr, 2e-2, 1e-2, "y")
    g = torch.randn_like(yr)
    y.backward(g.bfloat16())
    yr.backward(g)
    _close(gu.grad, gr.grad, 3e-2, 2e-2, "dgu")


@pytest.mark.parametrize("entropy", [False, True])
def test_fused_lm_head_logprob(entropy):
    from bridge_b200.ops.logprob import fused_lm_head_logprob, logprob_entropy_reference

    U, H, V = 300, 256, 5000
    h = (torch.randn(U, H, device=DEV) * 0.5).to(torch.bfloat16).requires_grad_()
    W = (torch.randn(V, H, device=DEV) * 0.05).to(torch.bfloat16).requires_grad_()
    tg = torch.randint(0, V, (U,), device=DEV)
    temp = torch.rand(U, device=DEV) + 0.5
    lp, ent = fused_lm_head_logprob(h, W, tg, temp, with_entropy=entropy, chunk_rows=128)
    hr, Wr = h.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    lpr, entr = logprob_entropy_reference(hr @ Wr.t(), tg, temp, with_entropy=entropy)
    _close(lp, lpr, 5e-2, 1e-2, "lp")
    g = torch.randn(U, device=DEV)
    loss = (lp * g).sum() + ((ent * g).sum() if entropy else 0)
    lossr = (lpr * g).sum() + ((entr * g).sum() if entropy else 0)
    if entropy:
        _close(ent, entr, 5e-2, 1e-2, "entropy")
    loss.backward()
    lossr.backward()
    _close(h.grad, hr.grad, 5e-2, 3e-2, "dh")
    _close(W.grad, Wr.grad, 5e-2, 3e-2, "dW")


@pytest.mark.parametrize("main_grad", [False, True])
def test_fused_lm_head_ppo(main_grad):
    """Head + log-prob + PPO loss with the head backward run inside the forward, against FP32 torch: loss,
    dh (scaled by the loss gradient) and dW (into an FP32 main_grad, or returned to autograd)."""
    from bridge_b200.ops.logprob import fused_lm_head_ppo, logprob_entropy_reference
    from bridge_b200.ops.ppo import PPOLossConfig, ppo_loss_reference

    U, H, V, R = 300, 256, 5000, 420
    h = (torch.randn(U, H, device=DEV) * 0.5).to(torch.bfloat16).requires_grad_()
    W = (torch.randn(V, H, device=DEV) * 0.05).to(torch.bfloat16).requires_grad_()
    if main_grad:
        W.main_grad = torch.zeros(V, H, device=DEV)
    tg = torch.randint(0, V, (U,), device=DEV)
    temp = torch.rand(U, device=DEV) + 0.5
    inv = torch.randint(0, U, (R,), device=DEV)         # duplicate refs share a row
    old = torch.randn(R, device=DEV) * 0.3 - 9.0
    adv = torch.randn(R, device=DEV)
    wts = torch.rand(R, device=DEV)
    scale = 4.0
    loss, stats, lp, _ = fused_lm_head_ppo(h, W, tg, temp, inv, old, adv, wts, denom=777.0, clip_low=0.2,
                                           clip_high=0.2, clip_c=3.0, chunk_rows=128, grad_scale=scale)
    (loss * scale).backward()
    hr, Wr = h.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    lpr, _ = logprob_entropy_reference(hr @ Wr.t(), tg, temp)
    lr, sr = ppo_loss_reference(lpr[inv], old, adv, 777.0, PPOLossConfig(), wts)
    (lr * scale).backward()
    _close(lp, lpr, 5e-2, 1e-2, "lp")
    _close(loss, lr, 1e-3, 1e-2, "loss")
    _close(stats, sr, 1e-3, 1e-2, "stats")
    _close(h.grad, hr.grad, 5e-2, 3e-2, "dh")
    _close(W.main_grad if main_grad else W.grad, Wr.grad, 5e-2, 3e-2, "dW")


def test_ppo_loss():
    from bridge_b200.ops.ppo import PPOLossConfig, ppo_loss, ppo_loss_reference

    n = 5000
    x = (torch.randn(n, device=DEV) * 0.3 - 5).requires_grad_()
    old = x.detach() + torch.randn(n, device=DEV) * 0.3
    adv = torch.randn(n, device=DEV)
    w = torch.rand(n, device=DEV)
    loss, stats = ppo_loss(x, old, adv, denom=1234.0, weights=w)
    xr = x.detach().clone().requires_grad_()
    lr, sr = ppo_loss_reference(xr, old, adv, 1234.0, PPOLossConfig(), w)
    _close(loss, lr, 1e-5, 1e-4, "loss")
    _close(stats, sr, 1e-5, 1e-4, "stats")
    loss.backward()
    lr.backward()
    _close(x.grad, xr.grad, 1e-6, 1e-4, "dx")


@pytest.mark.parametrize("off", [0, 1])
def test_adamw_kernel(off):
    """16-byte vector path with a scalar tail (off = 0) and the scalar path for unaligned views (off = 1)."""
    from bridge_b200.ops._ext import kernels

    n = 10001
    master = torch.randn(n + off, device=DEV)[off:]
    param = torch.empty(n + off, device=DEV, dtype=torch.bfloat16)[off:]
    param.copy_(master)
    grad = torch.randn(n + off, device=DEV)[off:]
    m = torch.randn(n + off, device=DEV)[off:].abs() * 0.1
    v = torch.rand(n + off, device=DEV)[off:] * 0.01
    ref = [t.clone() for t in (master, m, v)]
    clip = torch.tensor([0.5], device=DEV)
    kernels().adamw_step(master, param, grad, m, v, clip, 1e-3, 0.9, 0.999, 1e-8, 0.01, 0.19, 0.002)
    mr, m2, v2 = ref
    g = grad * 0.5
    m2 = 0.9 * m2 + 0.1 * g
    v2 = 0.999 * v2 + 0.001 * g * g
    mr = mr * (1 - 1e-3 * 0.01) - 1e-3 * (m2 / 0.19) / ((v2 / 0.002).sqrt() + 1e-8)
    _close(master, mr, 1e-5, 1e-5, "master")
    _close(param, mr, 1e-2, 1e-2, "param")


def _tree_case(D, hq, hkv, lens, spans, P, seed=0):
    from bridge_b200.tpr.context import SegmentBatchLayout

    torch.manual_seed(seed)
    T = sum(lens)
    q = torch.randn(T, hq, D, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(T, hkv, D, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(T, hkv, D, device=DEV, dtype=torch.bfloat16)
    pk = torch.randn(max(P, 1), hkv, D, device=DEV, dtype=torch.bfloat16)
    pv = torch.randn(max(P, 1), hkv, D, device=DEV, dtype=torch.bfloat16)
    lay = SegmentBatchLayout.build(lens, spans, device=DEV)
    return q, k, v, pk, pv, lay


@pytest.mark.parametrize("D,hq,hkv,lens,spans,P", [
    (128, 8, 2, (512, 512, 300, 1), ((0, 512), (0, 512), (512, 77), (0, 0)), 589),   # siblings share span 0
    (128, 4, 4, (70,), ((0, 0),), 0),                                                  # plain causal, odd length
    (64, 4, 2, (129, 64, 200), ((5, 130), (5, 130), (0, 3)), 140),
    (128, 32, 8, (512,) * 8, ((0, 512),) * 8, 512),                                    # Qwen3-4B-shaped siblings
    (256, 4, 2, (100, 130, 64), ((0, 64), (0, 64), (64, 10)), 74),                      # gated-attention head dim
    (256, 16, 2, (256, 256), ((0, 256), (0, 256)), 256),
])
def test_tree_attention_fwd_bwd(D, hq, hkv, lens, spans, P):
    from bridge_b200.ops.attention import tree_attention, tree_attention_reference

    q, k, v, pk, pv, lay = _tree_case(D, hq, hkv, lens, spans, P)
    scale = 1 / math.sqrt(D)
    leaves = [t.clone().requires_grad_() for t in (q, k, v, pk, pv)]
    o = tree_attention(*leaves, lay, softmax_scale=scale)
    ref = [t.detach().float().requires_grad_() for t in (q, k, v, pk, pv)]
    orf = tree_attention_reference(ref[0], ref[1], ref[2], ref[3], ref[4], lay, softmax_scale=scale)
    _close(o, orf, 8e-3, 2e-2, "o")
    g = torch.randn_like(orf)
    o.backward(g.bfloat16())
    orf.backward(g)
    for a, b, n in zip(leaves, ref, ("dq", "dk", "dv", "dpk", "dpv")):
        if P == 0 and n in ("dpk", "dpv"):
            assert a.grad is None
            continue
        _close(a.grad, b.grad, 1e-2, 3e-2, n)


def test_tree_attention_d256_forward():
    from bridge_b200.ops.attention import tree_attention_reference
    from bridge_b200.ops._ext import kernels

    q, k, v, pk, pv, lay = _tree_case(256, 4, 2, (100, 130), ((0, 64), (0, 64)), 64)
    o, lse = kernels().tree_attn_fwd(q, k, v, pk, pv, lay.cu_seqlens, lay.prefix_offsets, lay.prefix_lengths,
                                     lay.max_seqlen, lay.max_prefix, 1 / 16)
    orf = tree_attention_reference(q.float(), k.float(), v.float(), pk.float(), pv.float(), lay, softmax_scale=1 / 16)
    _close(o, orf, 8e-3, 2e-2, "o")


@pytest.mark.parametrize("lens,spans,P,hq,hkv", [
    ((512,) * 4, ((0, 512),) * 4, 512, 32, 8),
    ((300, 77, 129), ((0, 200), (200, 13), (0, 0)), 213, 8, 2),
    ((1,), ((0, 1000),), 1000, 4, 4),
    ((640, 640), ((0, 0), (0, 0)), 0, 16, 4),
])
def test_tree_attention_sm100_forward(lens, spans, P, hq, hkv):
    from bridge_b200.ops._ext import kernels
    from bridge_b200.ops.attention import tree_attention_reference

    q, k, v, pk, pv, lay = _tree_case(128, hq, hkv, lens, spans, P, seed=3)
    if P == 0:
        pk = pv = q.new_empty((0, hkv, 128))
    o, lse = kernels().tree_attn_fwd_sm100(q, k, v, pk, pv, lay.cu_seqlens, lay.prefix_offsets, lay.prefix_lengths,
                                           lay.max_seqlen, lay.max_prefix, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert kernels().attn_error_code() == 0
    orf = tree_attention_reference(q.float(), k.float(), v.float(), pk.float() if P else None,
                                   pv.float() if P else None, lay, softmax_scale=1 / math.sqrt(128))
    _close(o, orf, 8e-3, 2e-2, "o")
    o2, lse2 = kernels().tree_attn_fwd(q, k, v, pk, pv, lay.cu_seqlens, lay.prefix_offsets, lay.prefix_lengths,
                                       lay.max_seqlen, lay.max_prefix, 1 / math.sqrt(128))
    _close(lse, lse2, 1e-3, 1e-3, "lse")


@pytest.mark.parametrize("lens,spans,P,hq,hkv", [
    ((512,) * 4, ((0, 512),) * 4, 512, 32, 8),
    ((300, 77, 129), ((0, 200), (200, 13), (0, 0)), 213, 8, 2),
    ((640, 640), ((0, 0), (0, 0)), 0, 16, 4),
    ((5, 260), ((0, 700), (100, 300)), 700, 4, 2),
])
def test_tree_attention_sm100_backward(lens, spans, P, hq, hkv):
    from bridge_b200.ops._ext import kernels
    from bridge_b200.ops.attention import tree_attention_reference

    q, k, v, pk, pv, lay = _tree_case(128, hq, hkv, lens, spans, P, seed=4)
    if P == 0:
        pk = pv = q.new_empty((0, hkv, 128))
    sc = 1 / math.sqrt(128)
    o, lse = kernels().tree_attn_fwd_sm100(q, k, v, pk, pv, lay.cu_seqlens, lay.prefix_offsets, lay.prefix_lengths,
                                           lay.max_seqlen, lay.max_prefix, sc)
    do = torch.randn_like(o)
    dq, dk, dv, dpk, dpv = kernels().tree_attn_bwd_sm100(do, q, k, v, pk, pv, o, lse, lay.cu_seqlens,
                                                         lay.prefix_offsets, lay.prefix_lengths, lay.max_seqlen,
                                                         lay.max_prefix, sc)
    torch.cuda.synchronize()
    assert kernels().attn_error_code() == 0
    ref = [t.detach().float().requires_grad_() for t in (q, k, v, pk, pv)]
    orf = tree_attention_reference(ref[0], ref[1], ref[2], ref[3] if P else None, ref[4] if P else None, lay,
                                   softmax_scale=sc)
    orf.backward(do.float())
    for a, b_, n in zip((dq, dk, dv), ref[:3], ("dq", "dk", "dv")):
        _close(a, b_.grad, 1e-2, 3e-2, n)
    if P:
        _close(dpk, ref[3].grad, 1e-2, 3e-2, "dpk")
        _close(dpv, ref[4].grad, 1e-2, 3e-2, "dpv")


@pytest.mark.parametrize("n", [1, 1003, 4 * 1000 + 3, 1 << 22])
def test_sumsq_into(n):
    from bridge_b200.ops._ext import kernels

    x = torch.randn(n + 1, device=DEV)[1:] if n % 2 else torch.randn(n, device=DEV)   # odd n: unaligned start
    out = torch.full((1,), 5.0, device=DEV)
    kernels().sumsq_into(x, out, False)
    ref = (x.double() ** 2).sum()
    assert abs(out.item() - ref.item()) <= 1e-5 * ref.item() + 1e-6
    kernels().sumsq_into(x, out, True)
    assert abs(out.item() - 2 * ref.item()) <= 2e-5 * ref.item() + 1e-6


def test_norm_weight_grads_accumulate_into_main_grad():
    """With an FP32 ``main_grad`` on the weight (the engine's gradient arena), the RMSNorm, fused add +
    RMSNorm and qk-norm + RoPE backward kernels add the weight gradient into it in place and hand
    autograd no gradient for the weight."""
    from bridge_b200.ops.norm import add_rmsnorm, qk_norm_rope, rmsnorm, rope_cos_sin

    torch.manual_seed(3)
    T, H = 300, 2560

    def grads(use_main):
        w1 = (1 + 0.1 * torch.randn(H, device=DEV, generator=torch.Generator(device=DEV).manual_seed(1))).to(
            torch.bfloat16).requires_grad_()
        w2 = w1.detach().clone().requires_grad_()
        qw = torch.linspace(0.5, 1.5, 128, device=DEV).to(torch.bfloat16).requires_grad_()
        kw = torch.linspace(1.5, 0.5, 128, device=DEV).to(torch.bfloat16).requires_grad_()
        base = {}
        for name, w in (("w1", w1), ("w2", w2), ("qw", qw), ("kw", kw)):
            base[name] = torch.full(w.shape, 0.25, device=DEV)
            if use_main:
                w.main_grad = base[name].clone()
        g = torch.Generator(device=DEV).manual_seed(2)
        x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16).requires_grad_()
        r = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
        q = torch.randn(T, 8, 128, device=DEV, generator=g).to(torch.bfloat16).requires_grad_()
        k = torch.randn(T, 2, 128, device=DEV, generator=g).to(torch.bfloat16).requires_grad_()
        cos, sin = rope_cos_sin(torch.arange(T, device=DEV), 128, 1e6)
        y1 = rmsnorm(x, w1, 1e-6)
        h, y2 = add_rmsnorm(x, r, w2, 1e-6)
        qo, ko = qk_norm_rope(q, k, qw, kw, cos, sin, 1e-6)
        loss = (y1.float() ** 2).sum() + (y2.float() * h.float()).sum() + (qo.float() ** 2).sum() + ko.float().sum()
        loss.backward()
        out = {"dx": x.grad.float(), "dq": q.grad.float(), "dk": k.grad.float()}
        for name, w in (("w1", w1), ("w2", w2), ("qw", qw), ("kw", kw)):
            if use_main:
                assert w.grad is None, name
                out[name] = w.main_grad - base[name]
            else:
                out[name] = w.grad.float()
        return out

    a, b = grads(True), grads(False)
    for name in a:
        _close(a[name], b[name], 1e-3, 2e-2, name)


@pytest.mark.parametrize("start,use_main", [(0, True), (0, False), (500, True)])
def test_embedding_lookup_and_scatter_add(start, use_main):
    """Vocab-parallel lookup (ids outside this rank's rows give zero rows) and the backward's scatter-add
    into main_grad (or a fresh gradient) against torch's embedding, repeated ids included."""
    from bridge_b200.ops.embedding import embedding

    torch.manual_seed(start + int(use_main))
    V, H, T = 1000, 256, 4000
    w = (0.1 * torch.randn(V, H, device=DEV)).to(torch.bfloat16).requires_grad_()
    ids = torch.randint(0, 1500, (T,), device=DEV)
    if use_main:
        w.main_grad = torch.full((V, H), 0.5, device=DEV)
    out = embedding(ids, w, start)
    local = ids - start
    inside = (local >= 0) & (local < V)
    ref = torch.zeros(T, H, device=DEV)
    ref[inside] = w.detach().float()[local[inside]]
    _close(out, ref, 0, 0, "out")
    dy = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    out.backward(dy)
    g_ref = torch.zeros(V, H, device=DEV).index_add_(0, local[inside], dy.float()[inside])
    if use_main:
        assert w.grad is None
        _close(w.main_grad - 0.5, g_ref, 1e-4, 1e-5, "main_grad")
    else:
        _close(w.grad, g_ref, 1e-2, 1e-2, "grad")


def test_moe_route_sort_and_combine():
    """Device routing vs torch: top-k ids (descending, ties to the lower id), renormalised weights, the
    stable expert sort, counts; the gather-reduce combine and both backward kernels vs autograd."""
    from bridge_b200.ops._ext import kernels

    m = kernels()
    T, E, k, H = 1000, 512, 10, 256
    logits = torch.randn(T, E, device=DEV)
    idx, w, counts, offsets, pos, order = m.moe_route(logits, k)
    lr = logits.clone().requires_grad_()
    p = torch.softmax(lr, -1)
    wr, ir = torch.topk(p, k, -1)
    wr = wr / wr.sum(-1, keepdim=True)
    assert torch.equal(idx.long(), ir)
    _close(w, wr, 1e-5, 1e-4, "w")
    flat = ir.reshape(-1)
    assert torch.equal(order.long(), torch.argsort(flat, stable=True))
    assert torch.equal(pos.long()[order.long()], torch.arange(T * k, device=DEV))
    assert torch.equal(counts.long(), torch.bincount(flat, minlength=E))
    assert int(offsets[-1]) == T * k
    ys = torch.randn(T * k, H, device=DEV).bfloat16()
    y = m.moe_combine(ys, pos, w.reshape(-1).contiguous(), T)
    ysr = ys.float().requires_grad_()
    yr = (ysr[pos.long()].view(T, k, H) * wr.detach()[..., None]).sum(1)
    _close(y, yr, 2e-2, 1e-2, "combine")
    dy = torch.randn(T, H, device=DEV).bfloat16()
    dys, dw = m.moe_combine_bwd(dy, ys, pos, w.reshape(-1).contiguous())
    yr.backward(dy.float())
    _close(dys, ysr.grad, 2e-2, 1e-2, "dys")
    dwr = (dy.float()[:, None, :] * ys.float()[pos.long()].view(T, k, H)).sum(-1)
    _close(dw.view(T, k), dwr, 5e-2, 1e-2, "dw")
    g = torch.randn(T, k, device=DEV)
    dl = m.moe_route_bwd(idx, w, g.contiguous(), E)
    (wr * g).sum().backward()
    _close(dl, lr.grad, 1e-5, 1e-4, "dlogits")

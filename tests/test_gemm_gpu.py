"""tcgen05 GEMM vs an FP32 torch reference: all operand majors, bf16 store and FP32 accumulate."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _check(out, ref, name):
    out, ref = out.float(), ref.float()
    err = (out - ref).abs().max().item()
    tol = 2e-2 * ref.abs().max().item() + 1e-2
    assert err <= tol, f"{name}: {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("acc", [False, True])
@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (200, 520, 136), (1024, 2560, 2560), (8, 8, 8)])
def test_gemm(a_mn, b_mn, acc, M, N, K):
    from bridge_b200.ops._ext import kernels

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    if acc:
        c0 = torch.randn(M, N, device="cuda", generator=g)
        out = c0.clone()
        kernels().gemm(a, b, a_mn, b_mn, out, True)
        ref = ref + c0
    else:
        out = kernels().gemm(a, b, a_mn, b_mn, None, False)
    torch.cuda.synchronize()
    assert kernels().gemm_error_code() == 0
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


def test_linear_autograd_main_grad():
    from bridge_b200.ops.gemm import linear

    x = torch.randn(300, 256, device="cuda").bfloat16().requires_grad_()
    w = torch.nn.Parameter(torch.randn(512, 256, device="cuda").bfloat16() * 0.05)
    w.main_grad = torch.zeros(512, 256, device="cuda")
    y = linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = xr @ wr.t()
    yr.backward(g.float())
    assert (y.float() - yr).abs().max() < 5e-2
    assert (x.grad.float() - xr.grad).abs().max() < 5e-2
    assert w.grad is None and (w.main_grad - wr.grad).abs().max() < 5e-2


@pytest.mark.parametrize("counts", [[130, 0, 1, 257, 64, 0], [5] * 9 + [300], [0, 0, 700]])
@pytest.mark.parametrize("N,K", [(256, 512), (520, 128)])
def test_grouped_gemm_modes(counts, N, K):
    """MoE grouped GEMMs (device expert offsets) vs per-expert FP32 matmuls: x W^T, x W, dy^T x."""
    from bridge_b200.ops._ext import kernels

    m = kernels()
    torch.manual_seed(sum(counts) + N)
    E, T = len(counts), sum(counts)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(torch.tensor(counts), 0)
    offd = off.cuda()
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (0.05 * torch.randn(E, N, K, device="cuda")).bfloat16()
    y = m.grouped_gemm(x, w, offd, False)
    ref = torch.cat([x[off[e]:off[e + 1]].float() @ w[e].float().t() for e in range(E)])
    _check(y, ref, "grouped x W^T")
    # transposed expert weight: out = dy W_e with W_e [N, K] -> reduction over N (multiple of 64 required)
    if N % 64 == 0:
        dy = torch.randn(T, N, device="cuda").bfloat16()
        dx = m.grouped_gemm(dy, w, offd, True)
        ref = torch.cat([dy[off[e]:off[e + 1]].float() @ w[e].float() for e in range(E)])
        _check(dx, ref, "grouped x W")
        acc = torch.randn(E, N, K, device="cuda")
        before = acc.clone()
        m.grouped_gemm_wgrad(dy, x, offd, acc)
        ref = before + torch.stack([dy[off[e]:off[e + 1]].float().t() @ x[off[e]:off[e + 1]].float()
                                    for e in range(E)])
        _check(acc, ref, "grouped dy^T x (accumulate)")
    torch.cuda.synchronize()
    assert m.gemm_error_code() == 0


def test_moe_layer_grouped_matches_expert_loop():
    from bridge_b200.models import get_config
    from bridge_b200.models.moe import MoELayer

    cfg = get_config("tiny_moe", hidden_size=256, moe_intermediate_size=128, num_experts=16, moe_top_k=3)
    torch.manual_seed(0)
    layer = MoELayer(cfg, device="cuda")
    with torch.no_grad():
        layer.router.mul_(20.0)   # well-separated routes: both paths pick the same experts
    x = torch.randn(300, 256, device="cuda").bfloat16().requires_grad_()
    y = layer(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    g = {n: p.grad.clone() for n, p in layer.named_parameters()}
    gx = x.grad.clone()
    import bridge_b200.models.moe as moe

    orig = moe._grouped_ok
    moe._grouped_ok = lambda *a: False
    try:
        layer.zero_grad()
        x2 = x.detach().clone().requires_grad_()
        y2 = layer(x2)
        y2.backward(dy)
    finally:
        moe._grouped_ok = orig
    _check(y, y2.float(), "moe y")
    _check(gx, x2.grad.float(), "moe dx")
    for n, p in layer.named_parameters():
        _check(g[n], p.grad.float(), "moe d" + n)

"""tcgen05 GEMM vs an FP32 torch reference: all operand majors, bf16 store and FP32 accumulate."""

import pytest
import torch

pytestmark = pytest.mark.gpu


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

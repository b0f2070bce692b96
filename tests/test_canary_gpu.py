"""Out-of-bounds and determinism checks without compute-sanitizer.

* Canary-padded outputs: every kernel that writes into a caller-provided buffer (GEMM ``out=`` and
  FP32 accumulate into a main-gradient view, embedding scatter-add into ``main_grad``, RMSNorm weight
  gradient accumulated in place, P2P row gather / reduce on one rank) writes into a view that sits
  between two guard zones of a known bit pattern.  After the call the guard zones must be bitwise
  unchanged.  Shapes are ragged (not multiples of the tiles) so tile tails are exercised.
* Determinism: the kernels without atomics (GEMM, forward attention, norms, the whole model forward)
  give bitwise-identical results when run twice on the same inputs.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
GUARD = 4096          # elements in each guard zone


def _guarded(n: int, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """A buffer with ``GUARD`` canary elements on both sides of an ``n``-element payload."""
    buf = torch.empty(n + 2 * GUARD, device=DEV, dtype=dtype)
    if dtype == torch.float32:
        buf.view(torch.int32).fill_(0x7FC0DEAD)          # a NaN payload nobody writes on purpose
    else:
        buf.view(torch.int16).fill_(0x7FCD)
    return buf, buf[GUARD:GUARD + n]


def _guards_intact(buf: torch.Tensor, n: int) -> bool:
    raw = buf.view(torch.int32) if buf.dtype == torch.float32 else buf.view(torch.int16)
    want = 0x7FC0DEAD if buf.dtype == torch.float32 else 0x7FCD
    return bool((raw[:GUARD] == want).all()) and bool((raw[GUARD + n:] == want).all())


@pytest.mark.parametrize("m,n,k", [(333, 2560, 2560), (129, 9728, 2560), (4099, 640, 1024)])
def test_gemm_out_and_accumulate_stay_inside(m, n, k):
    from bridge_b200.ops.gemm import gemm

    a = torch.randn(m, k, device=DEV).bfloat16()
    b = torch.randn(n, k, device=DEV).bfloat16()
    buf, out = _guarded(m * n, torch.bfloat16)
    gemm(a, b, out=out.view(m, n))
    torch.cuda.synchronize()
    assert _guards_intact(buf, m * n)
    ref = (a.float() @ b.float().t())
    assert (out.view(m, n).float() - ref).abs().max().item() <= 0.05 + 0.01 * ref.abs().max().item()
    # FP32 accumulate (the wgrad epilogue into main_grad): dW[n, k] += dy^T x with dy [m, n], x [m, k]
    dy = torch.randn(m, n, device=DEV).bfloat16()
    acc_buf, acc = _guarded(n * k, torch.float32)
    acc.fill_(1.0)
    gemm(dy, a, a_mn=True, b_mn=True, out=acc.view(n, k), accumulate=True)
    torch.cuda.synchronize()
    assert _guards_intact(acc_buf, n * k)
    ref = 1.0 + dy.float().t() @ a.float()
    assert (acc.view(n, k) - ref).abs().max().item() <= 0.05 + 0.01 * ref.abs().max().item()


def test_embedding_scatter_add_stays_inside():
    from bridge_b200.ops._ext import kernels

    vocab, h = 1000, 256
    ids = torch.randint(-50, vocab + 50, (777,), device=DEV)    # out-of-shard ids must be skipped
    dy = torch.randn(777, h, device=DEV).bfloat16()
    buf, g = _guarded(vocab * h, torch.float32)
    g.zero_()
    kernels().embedding_bwd_acc(ids, dy, g.view(vocab, h), 0)
    torch.cuda.synchronize()
    assert _guards_intact(buf, vocab * h)
    ref = torch.zeros(vocab, h, device=DEV)
    ok = (ids >= 0) & (ids < vocab)
    ref.index_add_(0, ids[ok], dy[ok].float())
    assert (g.view(vocab, h) - ref).abs().max().item() < 1e-3


def test_rmsnorm_weight_grad_accumulates_inside_main_grad():
    from bridge_b200.ops.norm import rmsnorm

    rows, h = 1031, 2560
    w = torch.nn.Parameter(torch.ones(h, device=DEV, dtype=torch.bfloat16))
    buf, mg = _guarded(h, torch.float32)
    mg.zero_()
    w.main_grad = mg
    x = torch.randn(rows, h, device=DEV).bfloat16().requires_grad_()
    rmsnorm(x, w, 1e-6).float().sum().backward()
    torch.cuda.synchronize()
    assert _guards_intact(buf, h)
    assert bool(torch.isfinite(mg).all()) and float(mg.abs().sum()) > 0


def test_p2p_row_movement_stays_inside_single_rank():
    """The P2P row kernels with one "peer" (this GPU): gather and FP32 / bf16 owner reduction."""
    from bridge_b200.ops._ext import kernels

    m = kernels()
    rows, w = 301, 1024
    src = torch.randn(rows, w, device=DEV).bfloat16()
    idx = torch.randperm(rows, device=DEV).int()
    buf, out = _guarded(rows * w, torch.bfloat16)
    m.p2p_gather_rows(out.view(rows, w), [src.data_ptr()], torch.zeros(rows, dtype=torch.int32, device=DEV), idx)
    torch.cuda.synchronize()
    assert _guards_intact(buf, rows * w)
    assert torch.equal(out.view(rows, w), src[idx.long()])
    src32 = torch.randn(rows, w, device=DEV)
    for out_dtype in (torch.bfloat16, torch.float32):
        buf, out = _guarded(rows * w, out_dtype)
        m.p2p_reduce_rows(out.view(rows, w), [src32.data_ptr()], idx, True, None)
        torch.cuda.synchronize()
        assert _guards_intact(buf, rows * w)
        ref = src32[idx.long()]
        tol = 1e-6 if out_dtype == torch.float32 else 8e-3          # bf16 rounding of the output
        assert bool(((out.view(rows, w).float() - ref).abs() <= tol * (1 + ref.abs())).all())


def test_forward_kernels_are_deterministic():
    """Twice-run bitwise identity of the atomics-free forward path (GEMM, attention, norms, model)."""
    from bridge_b200.models import get_config
    from bridge_b200.models.decoder import build_model
    from bridge_b200.ops.attention import tree_attention
    from bridge_b200.ops.gemm import gemm
    from bridge_b200.tpr.context import SegmentBatchLayout

    a = torch.randn(1000, 2560, device=DEV).bfloat16()
    b = torch.randn(3000, 2560, device=DEV).bfloat16()
    assert torch.equal(gemm(a, b), gemm(a, b))
    lay = SegmentBatchLayout.build((300, 212), ((0, 200), (0, 200)), device=DEV)
    q = torch.randn(512, 8, 128, device=DEV).bfloat16()
    k = torch.randn(512, 2, 128, device=DEV).bfloat16()
    v = torch.randn(512, 2, 128, device=DEV).bfloat16()
    pk = torch.randn(200, 2, 128, device=DEV).bfloat16()
    pv = torch.randn(200, 2, 128, device=DEV).bfloat16()
    o1 = tree_attention(q, k, v, pk, pv, lay, softmax_scale=0.088)
    o2 = tree_attention(q, k, v, pk, pv, lay, softmax_scale=0.088)
    assert torch.equal(o1, o2)
    cfg = get_config("tiny", hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=128, intermediate_size=1024)
    model = build_model(cfg, device=DEV, seed=0)
    ids = torch.randint(0, cfg.vocab_size, (700,), device=DEV)
    pos = torch.arange(700, device=DEV)
    with torch.no_grad():
        assert torch.equal(model(ids, pos, 700), model(ids, pos, 700))

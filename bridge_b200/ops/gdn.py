"""Gated DeltaNet ops: stateful causal depthwise conv1d and the chunked gated delta rule.

Both take packed varlen inputs (``cu_seqlens`` host list, one continuation
state per sequence) so a batch of sibling segments runs in one call.

causal_conv1d
    ``x [T, C]``, depthwise weight ``[C, W]``, optional bias, SiLU.  The state
    ``[B, C, W]`` holds the last ``W-1`` inputs in slots ``1..W-1`` (slot 0 is
    unused and always zero); output row ``t`` of a sequence convolves
    ``cat(h0[:, 1:], x)`` over a window of ``W``, so only rows ``t < W-1`` read
    the initial state and ``dh0[:, :, 0] == 0``.

gated delta rule (FLA convention)
    ``S_t = e^{g_t} S_{t-1};  u_t = beta_t (v_t - S_t^T k_t);  S_t += k_t u_t^T;
    o_t = scale * S_t^T q_t`` with FP32 state ``[B, H, K, V]``.  The chunked
    form (chunk C) uses, per chunk with cumulative decay ``Gamma_t``,
    ``A_ts = (Gamma_t/Gamma_s) k_t.k_s`` (s<t), ``T = (I + diag(beta) A)^-1``,
    ``U = T diag(beta) V - T diag(beta Gamma) K S0``,
    ``O = scale (diag(Gamma) Q S0 + (Mask ∘ Gamma_t/Gamma_s ∘ Q K^T) U)``,
    ``S_C = Gamma_C S0 + K^T diag(Gamma_C/Gamma) U`` -- i.e. the chunk end state is
    affine in ``S0`` (the basis of the sequence-sharded CP state chain).

Parity: MindSpeed-Ops causal_conv1d / chunk_gated_delta_rule as called from
verl/models/mcore/tpr/gated_delta_net.py:214-263; oracle restated from
tests/unit_tests/triton/test_chunk_gated_delta_rule_stateful_experiment.py:96-215
and tests/models/mcore/tpr/parallel/test_conv_dh0_bounds_npu.py:80-98.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from ._ext import kernels, on_gpu


# --------------------------------------------------------------------------- causal conv1d
def causal_conv1d_reference(x: Tensor, weight: Tensor, bias: Tensor | None, cu_seqlens: list[int],
                            initial_state: Tensor | None, *, activation: bool = True):
    """Returns ``y [T, C]`` and final state ``[B, C, W]`` (slot 0 zero)."""
    c, w = weight.shape
    ys, finals = [], []
    for i in range(len(cu_seqlens) - 1):
        xs = x[cu_seqlens[i]:cu_seqlens[i + 1]]                      # [L, C]
        if initial_state is not None:
            hist = initial_state[i, :, 1:].transpose(0, 1).to(xs.dtype)   # [W-1, C]
        else:
            hist = xs.new_zeros((w - 1, c))
        full = torch.cat((hist, xs), dim=0).float()                  # [L+W-1, C]
        win = full.unfold(0, w, 1)                                   # [L, C, W]
        y = (win * weight.float()[None]).sum(-1)
        if bias is not None:
            y = y + bias.float()
        if activation:
            y = F.silu(y)
        ys.append(y.to(x.dtype))
        tail = full[-(w - 1):].transpose(0, 1)                       # [C, W-1]
        finals.append(torch.cat((tail.new_zeros((c, 1)), tail), dim=1).to(x.dtype))
    return torch.cat(ys), torch.stack(finals)


class _ConvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, h0, cu_dev, cu_host, activation):
        m = kernels()
        x = x.contiguous()
        max_len = max(b - a for a, b in zip(cu_host[:-1], cu_host[1:]))
        h0c = h0.contiguous() if h0 is not None else None
        y, hT = m.causal_conv1d_fwd(x, weight.contiguous(), bias, h0c, cu_dev, max_len, bool(activation))
        ctx.save_for_backward(x, weight, bias, h0c, cu_dev)
        ctx.activation, ctx.max_len = activation, max_len
        ctx.h0_dtype = None if h0 is None else h0.dtype
        return y, hT.to(x.dtype)

    @staticmethod
    def backward(ctx, dy, dhT):
        m = kernels()
        x, weight, bias, h0, cu = ctx.saved_tensors
        dx, dw, db, dh0 = m.causal_conv1d_bwd(dy.contiguous(), x, weight.contiguous(), bias, h0,
                                              dhT.contiguous() if dhT is not None else None, cu, ctx.max_len,
                                              bool(ctx.activation))
        return dx, dw.to(weight.dtype), (db.to(bias.dtype) if bias is not None else None), \
            (dh0.to(ctx.h0_dtype) if h0 is not None else None), None, None, None


def causal_conv1d(x: Tensor, weight: Tensor, bias: Tensor | None, cu_seqlens: list[int], cu_dev: Tensor | None,
                  initial_state: Tensor | None, *, activation: bool = True):
    if cu_seqlens[-1] != x.shape[0]:
        raise ValueError(f"causal_conv1d: the sequences cover {cu_seqlens[-1]} rows but x has {x.shape[0]}")
    if on_gpu(x):
        if cu_dev is None:
            cu_dev = torch.tensor(cu_seqlens, dtype=torch.int32, device=x.device)
        return _ConvFn.apply(x, weight, bias, initial_state, cu_dev, tuple(cu_seqlens), activation)
    return causal_conv1d_reference(x, weight, bias, cu_seqlens, initial_state, activation=activation)


# --------------------------------------------------------------------------- gated delta rule
def gated_delta_rule_recurrent(q, k, v, g, beta, initial_state, *, scale: float):
    """Naive per-token recurrence for ONE sequence (oracle). ``q,k [L,H,K]``, ``v [L,H,V]``, ``g,beta [L,H]``."""
    L, H, K = q.shape
    V = v.shape[-1]
    S = initial_state.float().clone() if initial_state is not None else q.new_zeros((H, K, V), dtype=torch.float32)
    outs = []
    for t in range(L):
        S = S * torch.exp(g[t].float())[:, None, None]
        kt, vt, qt = k[t].float(), v[t].float(), q[t].float()
        pred = torch.einsum("hk,hkv->hv", kt, S)
        u = beta[t].float()[:, None] * (vt - pred)
        S = S + kt[:, :, None] * u[:, None, :]
        outs.append(torch.einsum("hk,hkv->hv", qt, S) * scale)
    return torch.stack(outs).to(q.dtype), S


def _chunk_one(q, k, v, g, beta, S0, scale: float, chunk: int):
    """Chunked form for one sequence; differentiable torch (FP32). Returns o [L,H,V], S [H,K,V]."""
    L, H, K = q.shape
    V = v.shape[-1]
    S = S0
    outs = []
    for s in range(0, L, chunk):
        e = min(L, s + chunk)
        n = e - s
        qc = q[s:e].float().transpose(0, 1)        # [H, n, K]
        kc = k[s:e].float().transpose(0, 1)
        vc = v[s:e].float().transpose(0, 1)        # [H, n, V]
        bc = beta[s:e].float().transpose(0, 1)     # [H, n]
        G = torch.cumsum(g[s:e].float().transpose(0, 1), dim=-1)   # [H, n]
        tri_strict = torch.ones(n, n, dtype=torch.bool, device=q.device).tril(-1)
        tri = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        # Gamma_t / Gamma_s, masked in the exponent: the upper triangle would overflow (and 0*inf -> NaN grads)
        diff = G[:, :, None] - G[:, None, :]
        decay = torch.exp(torch.where(tri, diff, torch.full_like(diff, float("-inf"))))
        kk = torch.matmul(kc, kc.transpose(1, 2))
        A = torch.where(tri_strict, decay * kk, torch.zeros_like(kk))
        eye = torch.eye(n, device=q.device, dtype=torch.float32).expand(H, n, n)
        Tm = torch.linalg.solve_triangular(eye + bc[:, :, None] * A, eye, upper=False)
        gam = torch.exp(G)
        Wv = torch.matmul(Tm, bc[:, :, None] * vc)
        Wk = torch.matmul(Tm, (bc * gam)[:, :, None] * kc)
        U = Wv - torch.matmul(Wk, S)                                # [H, n, V]
        qk = torch.where(tri, decay * torch.matmul(qc, kc.transpose(1, 2)), torch.zeros_like(kk))
        o = (gam[:, :, None] * torch.matmul(qc, S) + torch.matmul(qk, U)) * scale
        outs.append(o.transpose(0, 1))
        gl = gam[:, -1]
        S = gl[:, None, None] * S + torch.matmul((kc * torch.exp(G[:, -1:] - G)[:, :, None]).transpose(1, 2), U)
    return torch.cat(outs).to(q.dtype), S


def chunk_gated_delta_rule_reference(q, k, v, g, beta, cu_seqlens: list[int], initial_state: Tensor | None, *,
                                     scale: float, chunk_size: int = 64):
    """Packed varlen chunked GDR (torch). ``initial_state [B,H,K,V]`` FP32 or None."""
    H, K, V = q.shape[1], q.shape[2], v.shape[2]
    outs, finals = [], []
    for i in range(len(cu_seqlens) - 1):
        a, b = cu_seqlens[i], cu_seqlens[i + 1]
        S0 = initial_state[i].float() if initial_state is not None else q.new_zeros((H, K, V), dtype=torch.float32)
        o, S = _chunk_one(q[a:b], k[a:b], v[a:b], g[a:b], beta[a:b], S0, scale, chunk_size)
        outs.append(o)
        finals.append(S)
    return torch.cat(outs), torch.stack(finals)


_CHUNK_CACHE: dict = {}


def _chunk_table(cu_host: tuple, device) -> tuple[Tensor, Tensor, int]:
    """``(chunks [nct, 4] = (row0, n, seq, chunk), seq0 [B+1], max chunks per sequence)`` for 64-token chunks."""
    key = (cu_host, str(device))
    hit = _CHUNK_CACHE.get(key)
    if hit is not None:
        return hit
    rows, seq0, most = [], [0], 1
    for b, (a, e) in enumerate(zip(cu_host[:-1], cu_host[1:])):
        nc = (e - a + 63) // 64
        most = max(most, nc)
        for c in range(nc):
            rows.append((a + 64 * c, min(64, e - a - 64 * c), b, c))
        seq0.append(len(rows))
    t = torch.tensor(rows if rows else [(0, 0, 0, 0)], dtype=torch.int32).reshape(-1, 4)[:len(rows)]
    out = (t.to(device), torch.tensor(seq0, dtype=torch.int32, device=device), most)
    if len(_CHUNK_CACHE) > 256:
        _CHUNK_CACHE.clear()
    _CHUNK_CACHE[key] = out
    return out


class _GDRFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, h0, cu_host, scale):
        m = kernels()
        q, k, v = (t.contiguous() for t in (q, k, v))
        gf, bf = g.float().contiguous(), beta.float().contiguous()
        chunks, seq0, most = _chunk_table(cu_host, q.device)
        o, hT, ckpt, wk, u = m.gdr_fwd(q, k, v, gf, bf, h0, chunks, seq0, most, float(scale))
        ctx.save_for_backward(q, k, v, gf, bf, ckpt, wk, u, chunks, seq0)
        ctx.scale, ctx.most, ctx.has_h0 = scale, most, h0 is not None
        ctx.dtypes = (g.dtype, beta.dtype, None if h0 is None else h0.dtype)
        return o, hT

    @staticmethod
    def backward(ctx, do, dhT):
        m = kernels()
        q, k, v, g, beta, ckpt, wk, u, chunks, seq0 = ctx.saved_tensors
        dq, dk, dv, dg, db, dh0 = m.gdr_bwd(do.contiguous(), dhT.contiguous() if dhT is not None else None,
                                            q, k, v, g, beta, ckpt, wk, u, chunks, seq0, ctx.most, ctx.has_h0,
                                            float(ctx.scale))
        gdt, bdt, hdt = ctx.dtypes
        return (dq.to(q.dtype), dk.to(k.dtype), dv, dg.to(gdt), db.to(bdt),
                (dh0.to(hdt) if ctx.has_h0 else None), None, None)


_GDR_SHAPES = {(128, 128), (64, 64), (32, 64), (64, 128), (32, 32)}


def chunk_gated_delta_rule(q, k, v, g, beta, cu_seqlens: list[int], cu_dev: Tensor | None,
                           initial_state: Tensor | None, *, scale: float, chunk_size: int = 64):
    """Packed varlen chunked gated delta rule; ``o [T,H,V]`` (q dtype) and final state ``[B,H,K,V]`` FP32.

    On CUDA this runs the tensor-core chunked kernels (bf16; (key, value) head dims (128, 128),
    (64, 64), (64, 128), (32, 64), (32, 32)).  The kernels always work in 64-token chunks: the
    chunking changes rounding only, not the result, so ``chunk_size`` applies to the PyTorch path.
    """
    if cu_seqlens[-1] != q.shape[0] or k.shape[0] != q.shape[0] or v.shape[0] != q.shape[0]:
        raise ValueError(f"chunk_gated_delta_rule: the sequences cover {cu_seqlens[-1]} rows but q/k/v have "
                         f"{q.shape[0]}/{k.shape[0]}/{v.shape[0]}")
    if on_gpu(q):
        if (q.shape[-1], v.shape[-1]) not in _GDR_SHAPES or q.dtype != torch.bfloat16:
            raise NotImplementedError("gated delta rule kernel: bf16 with (key dim, value dim) in "
                                      f"{sorted(_GDR_SHAPES)}")
        return _GDRFn.apply(q, k, v, g, beta, initial_state, tuple(cu_seqlens), scale)
    return chunk_gated_delta_rule_reference(q, k, v, g, beta, cu_seqlens, initial_state, scale=scale,
                                            chunk_size=chunk_size)


def l2norm_reference(x: Tensor, eps: float = 1e-6) -> Tensor:
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


def gated_rmsnorm_reference(o: Tensor, z: Tensor, weight: Tensor, eps: float) -> Tensor:
    of = o.float()
    y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return (y * F.silu(z.float())).to(o.dtype)


def gdn_gates_reference(a: Tensor, b: Tensor, A_log: Tensor, dt_bias: Tensor) -> tuple[Tensor, Tensor]:
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g, torch.sigmoid(b.float())


_ROW_WIDTHS = (32, 64, 128, 256)


def _heads_view_ok(x: Tensor) -> bool:
    return (x.dim() == 3 and x.dtype == torch.bfloat16 and x.shape[-1] in _ROW_WIDTHS and x.stride(2) == 1
            and (x.shape[1] == 1 or x.stride(1) == x.shape[2]))


class _L2NormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eps):
        y, rn = kernels().l2norm_fwd(x, eps)
        ctx.save_for_backward(x, rn)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, rn = ctx.saved_tensors
        return kernels().l2norm_bwd(dy.contiguous(), x, rn), None


class _GatedRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, z, weight, eps):
        o = o.contiguous()
        y, rstd = kernels().gated_rmsnorm_fwd(o, z, weight, eps)
        ctx.save_for_backward(o, z, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        o, z, weight, rstd = ctx.saved_tensors
        do, dz, dw = kernels().gated_rmsnorm_bwd(dy.contiguous(), o, z, weight, rstd)
        return do, dz, dw.to(weight.dtype), None


class _GatesFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, A_log, dt_bias):
        g, beta = kernels().gdn_gates_fwd(a, b, A_log, dt_bias)
        ctx.save_for_backward(a, b, A_log, dt_bias)
        return g, beta

    @staticmethod
    def backward(ctx, dg, dbeta):
        a, b, A_log, dt_bias = ctx.saved_tensors
        if dg is None:
            dg = torch.zeros(a.shape, dtype=torch.float32, device=a.device)
        if dbeta is None:
            dbeta = torch.zeros(b.shape, dtype=torch.float32, device=b.device)
        da, db, dA, ddt = kernels().gdn_gates_bwd(dg, dbeta, a, b, A_log, dt_bias)
        return da, db, dA.to(A_log.dtype), ddt.to(dt_bias.dtype)


def l2norm(x: Tensor, eps: float = 1e-6) -> Tensor:
    """Row L2 normalisation of ``x [T, H, D]`` (q / k before the delta rule); fused kernel on CUDA.

    ``x`` may be a column slice of the conv output (token stride wider than ``H * D``)."""
    if on_gpu(x) and _heads_view_ok(x):
        return _L2NormFn.apply(x, eps)
    return l2norm_reference(x, eps)


def gated_rmsnorm(o: Tensor, z: Tensor, weight: Tensor, eps: float) -> Tensor:
    """``RMSNorm(o) * weight * silu(z)`` per head (last dim); fused kernel on CUDA."""
    if on_gpu(o) and _heads_view_ok(o) and _heads_view_ok(z) and o.shape == z.shape:
        return _GatedRMSNormFn.apply(o, z, weight, eps)
    return gated_rmsnorm_reference(o, z, weight, eps)


def gdn_gates(a: Tensor, b: Tensor, A_log: Tensor, dt_bias: Tensor) -> tuple[Tensor, Tensor]:
    """Decay and write gates of the delta rule: ``g = -exp(A_log) softplus(a + dt_bias)`` (log-space
    decay per token and head) and ``beta = sigmoid(b)``, both FP32 ``[T, H]``.  ``a, b`` may be
    column slices of the fused input projection (unit column stride)."""
    if (on_gpu(a) and a.dim() == 2 and a.shape == b.shape and a.dtype == torch.bfloat16
            and b.dtype == torch.bfloat16 and a.stride(1) == 1 and b.stride(1) == 1):
        return _GatesFn.apply(a, b, A_log, dt_bias)
    return gdn_gates_reference(a, b, A_log, dt_bias)

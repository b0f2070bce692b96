"""RMSNorm (row-wise over the last dim) and fused per-head qk-RMSNorm + RoPE.

CUDA kernels (``csrc/elementwise.cu``): one warp per row, FP32 accumulation,
vectorised 16-byte loads; backward recomputes ``rstd`` from the saved input
and reduces the weight gradient per CTA before a final column sum.

RoPE follows the Qwen/HF "rotate-half" convention: with
``inv_freq[i] = theta^(-2i/d)`` and angle ``a = pos * inv_freq``,
``x' = x*cos(a) + rotate_half(x)*sin(a)`` where ``rotate_half([x1, x2]) = [-x2, x1]``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ._ext import kernels, on_gpu


def _main_grad(w: Tensor):
    """The weight's FP32 gradient accumulator when it has one (the engine's ``main_grad`` arena view):
    the backward kernels then add the weight gradient into it and autograd gets ``None`` for it."""
    g = getattr(w, "main_grad", None)
    if g is not None and g.dtype == torch.float32 and g.is_cuda and g.is_contiguous():
        return g.view(-1)
    return None


def rmsnorm_reference(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * weight.float()).to(x.dtype)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        m = kernels()
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, rstd = m.rmsnorm_fwd(x2, weight.contiguous(), float(eps))
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        m = kernels()
        x2, weight, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).contiguous()
        acc = _main_grad(weight)
        if acc is not None:
            dx = m.rmsnorm_bwd_acc(dy2, x2, weight.contiguous(), rstd, dy2.new_empty(0), acc)
            return dx.view(ctx.shape), None, None
        dx, dw = m.rmsnorm_bwd(dy2, x2, weight.contiguous(), rstd)
        return dx.view(ctx.shape), dw.to(weight.dtype), None


def rmsnorm(x: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    if on_gpu(x):
        return _RMSNormFn.apply(x, weight, eps)
    return rmsnorm_reference(x, weight, eps)


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, res, weight, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        r2 = res.reshape(x2.shape).contiguous()
        y, rstd, h = kernels().add_rmsnorm_fwd(x2, r2, weight.contiguous(), float(eps))
        ctx.save_for_backward(h, weight, rstd)
        ctx.shape = shape
        return h.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, weight, rstd = ctx.saved_tensors
        m = kernels()
        if dy is None:
            return dh, dh, None, None
        dy2 = dy.reshape(h.shape).contiguous()
        dh2 = dh.reshape(h.shape).contiguous() if dh is not None else dy2.new_empty(0)
        acc = _main_grad(weight)
        if acc is not None:
            d = m.rmsnorm_bwd_acc(dy2, h, weight.contiguous(), rstd, dh2, acc).view(ctx.shape)
            return d, d, None, None
        if dh is None:
            d, dw = m.rmsnorm_bwd(dy2, h, weight.contiguous(), rstd)
        else:
            d, dw = m.add_rmsnorm_bwd(dy2, h, weight.contiguous(), rstd, dh2)
        d = d.view(ctx.shape)
        return d, d, dw.to(weight.dtype), None


def add_rmsnorm(x: Tensor, res: Tensor, weight: Tensor, eps: float = 1e-6) -> tuple[Tensor, Tensor]:
    """Residual add fused with the RMSNorm that follows it: ``h = x + res``, ``y = RMSNorm(h) * w``.

    Returns ``(h, y)``.  ``h`` is rounded to the activation dtype before it is normalised, exactly as
    a separate add would; the backward returns ``RMSNorm'(dy) + dh`` for both ``x`` and ``res`` in one
    pass (the residual-gradient add is folded into the norm backward)."""
    if on_gpu(x) and x.dtype == torch.bfloat16 and res.dtype == torch.bfloat16:
        return _AddRMSNormFn.apply(x, res, weight, eps)
    h = x + res
    return h, rmsnorm_reference(h, weight, eps)


# --------------------------------------------------------------------------- RoPE
def rope_cos_sin(positions: Tensor, head_dim: int, theta: float) -> tuple[Tensor, Tensor]:
    """FP32 ``cos, sin [T, head_dim/2]`` for integer positions."""
    inv = theta ** (-torch.arange(0, head_dim, 2, device=positions.device, dtype=torch.float64) / head_dim)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope_reference(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """``x [T, H, D]``; cos/sin ``[T, D/2]``."""
    d2 = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :d2], xf[..., d2:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1).to(x.dtype)


def qk_norm_rope_reference(q, k, q_weight, k_weight, cos, sin, eps):
    if q_weight is not None:
        q = rmsnorm_reference(q, q_weight, eps)
        k = rmsnorm_reference(k, k_weight, eps)
    return apply_rope_reference(q, cos, sin), apply_rope_reference(k, cos, sin)


def _view_ok(t: Tensor) -> bool:
    return t.stride(2) == 1 and t.stride(0) % 8 == 0 and t.stride(1) % 8 == 0 and t.data_ptr() % 16 == 0


class _QKNormRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, qw, kw, cos, sin, eps):
        m = kernels()
        # strided views (column slices of the fused QKV output) are read in place
        q_ = q if _view_ok(q) else q.contiguous()
        k_ = k if _view_ok(k) else k.contiguous()
        qo, ko, rq, rk = m.qk_norm_rope_fwd(q_, k_, qw, kw, cos, sin, float(eps))
        ctx.save_for_backward(q_, k_, qw, kw, cos, sin, rq, rk)
        ctx.eps = eps
        return qo, ko

    @staticmethod
    def backward(ctx, dqo, dko):
        m = kernels()
        q, k, qw, kw, cos, sin, rq, rk = ctx.saved_tensors
        aq, ak = _main_grad(qw), _main_grad(kw)
        if aq is not None and ak is not None:
            dq, dk = m.qk_norm_rope_bwd_acc(dqo.contiguous(), dko.contiguous(), q, k, qw, kw, cos, sin, rq, rk, aq, ak)
            return dq, dk, None, None, None, None, None
        dq, dk, dqw, dkw = m.qk_norm_rope_bwd(dqo.contiguous(), dko.contiguous(), q, k, qw, kw, cos, sin, rq, rk)
        return dq, dk, dqw.to(qw.dtype), dkw.to(kw.dtype), None, None, None


def qk_norm_rope(q: Tensor, k: Tensor, q_weight: Tensor | None, k_weight: Tensor | None, cos: Tensor, sin: Tensor,
                 eps: float = 1e-6) -> tuple[Tensor, Tensor]:
    """Per-head RMSNorm of q and k (when weights are given) then RoPE; ``q [T,Hq,D]``, ``k [T,Hkv,D]``."""
    if on_gpu(q) and q_weight is not None:
        return _QKNormRopeFn.apply(q, k, q_weight, k_weight, cos.contiguous(), sin.contiguous(), eps)
    return qk_norm_rope_reference(q, k, q_weight, k_weight, cos, sin, eps)

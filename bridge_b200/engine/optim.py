"""Mixed-precision AdamW over one flat parameter arena.

Layout (per dtype group, bf16 model parameters):

* ``model params`` -- views into one contiguous bf16 arena (what the kernels read);
* ``master``       -- FP32 copy of the arena;
* ``main_grad``    -- FP32 gradient accumulator; after every backward each
                      parameter's bf16 ``.grad`` is folded into it by a
                      post-accumulate hook and released, so gradients
                      accumulate in FP32 across the forest's chunks;
* ``exp_avg / exp_avg_sq`` -- FP32 Adam moments.

The update is one fused CUDA kernel over the whole arena (decoupled weight
decay, bias correction, FP32 math, writes master + bf16 params in the same
pass).  Non-bf16 parameters (e.g. FP32 GDN ``A_log``) live in a second FP32
arena handled by the same kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from ..ops._ext import kernels, on_gpu


@dataclass(frozen=True)
class AdamWConfig:
    lr: float = 1e-6
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.01
    grad_clip: float = 1.0


class _Arena:
    def __init__(self, params: list[nn.Parameter], dtype, device) -> None:
        self.params = params
        n = sum(p.numel() for p in params)
        self.numel = n
        self.data = torch.empty(n, dtype=dtype, device=device)
        self.master = torch.empty(n, dtype=torch.float32, device=device)
        self.main_grad = torch.zeros(n, dtype=torch.float32, device=device)
        self.m = torch.zeros(n, dtype=torch.float32, device=device)
        self.v = torch.zeros(n, dtype=torch.float32, device=device)
        off = 0
        self.offsets = []
        for p in params:
            k = p.numel()
            self.data[off:off + k].copy_(p.data.reshape(-1))
            p.data = self.data[off:off + k].view_as(p)
            p.main_grad = self.main_grad[off:off + k].view(p.shape)  # type: ignore[attr-defined]
            self.offsets.append(off)
            off += k
        self.master.copy_(self.data.float())


class MixedPrecisionAdamW:
    """FP32-master AdamW for a module whose parameters are bf16 (or fp32)."""

    def __init__(self, module: nn.Module, cfg: AdamWConfig = AdamWConfig()) -> None:
        self.cfg = cfg
        params = [p for p in module.parameters() if p.requires_grad]
        dev = params[0].device
        self.arenas = []
        for dt in (torch.bfloat16, torch.float32):
            group = [p for p in params if p.dtype == dt]
            if group:
                self.arenas.append(_Arena(group, dt, dev))
        other = [p for p in params if p.dtype not in (torch.bfloat16, torch.float32)]
        if other:
            raise TypeError(f"unsupported parameter dtype {other[0].dtype}")
        self.step_count = 0
        self._hooks = [p.register_post_accumulate_grad_hook(self._fold) for a in self.arenas for p in a.params]

    @staticmethod
    def _fold(p: Tensor) -> None:
        if p.grad is not None:
            p.main_grad.add_(p.grad.view(p.main_grad.shape))
            p.grad = None

    def zero_grad(self) -> None:
        for a in self.arenas:
            a.main_grad.zero_()
            for p in a.params:
                p.grad = None

    def grad_buffers(self) -> list[Tensor]:
        return [a.main_grad for a in self.arenas]

    def grad_norm(self) -> Tensor:
        sq = [a.main_grad.float().pow(2).sum() for a in self.arenas]
        return torch.sqrt(torch.stack(sq).sum())

    def step(self, *, grad_norm: Tensor | None = None) -> Tensor:
        """One AdamW update; returns the pre-clip gradient norm (device scalar, no host sync)."""
        c = self.cfg
        self.step_count += 1
        norm = self.grad_norm() if grad_norm is None else grad_norm
        clip = torch.clamp(c.grad_clip / (norm + 1e-6), max=1.0) if c.grad_clip > 0 else torch.ones_like(norm)
        b1, b2 = c.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        for a in self.arenas:
            if on_gpu(a.master):
                kernels().adamw_step(a.master, a.data, a.main_grad, a.m, a.v, clip, float(c.lr), float(b1), float(b2),
                                     float(c.eps), float(c.weight_decay), float(bc1), float(bc2))
            else:
                g = a.main_grad * clip
                a.m.mul_(b1).add_(g, alpha=1 - b1)
                a.v.mul_(b2).addcmul_(g, g, value=1 - b2)
                denom = (a.v / bc2).sqrt_().add_(c.eps)
                a.master.mul_(1 - c.lr * c.weight_decay).addcdiv_(a.m / bc1, denom, value=-c.lr)
                a.data.copy_(a.master.to(a.data.dtype))
        return norm

    # -- checkpoint support
    def state_dict(self) -> dict:
        return {"step": self.step_count, "arenas": [{"master": a.master, "m": a.m, "v": a.v} for a in self.arenas]}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for a, s in zip(self.arenas, sd["arenas"]):
            a.master.copy_(s["master"])
            a.m.copy_(s["m"])
            a.v.copy_(s["v"])
            a.data.copy_(a.master.to(a.data.dtype))

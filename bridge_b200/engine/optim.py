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
        grads = [a.main_grad for a in self.arenas]
        if grads and all(on_gpu(g) and g.dtype == torch.float32 and g.is_contiguous() for g in grads):
            acc = torch.zeros(1, dtype=torch.float32, device=grads[0].device)
            for i, g in enumerate(grads):     # one read of each FP32 arena, no squared copy
                kernels().sumsq_into(g, acc, i > 0)
            return torch.sqrt(acc[0])
        sq = [g.float().pow(2).sum() for g in grads]
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


class _ShardedArena:
    """Arena whose bf16 (or FP32) parameters and FP32 gradients live in symmetric peer memory;
    the FP32 master and Adam moments hold only this rank's shard."""

    def __init__(self, params: list[nn.Parameter], dtype, heap) -> None:
        self.params = params
        n = sum(p.numel() for p in params)
        self.numel = n
        ranks = heap.size
        self.shard = max(8, -(-n // (ranks * 8)) * 8)
        total = self.shard * ranks
        esize = torch.tensor([], dtype=dtype).element_size()
        self.data_buf = heap.alloc(total * esize)
        self.grad_buf = heap.alloc(total * 4)
        self.data = self.data_buf.view(dtype, total)
        self.main_grad = self.grad_buf.view(torch.float32, total)
        self.bf16 = dtype == torch.bfloat16
        off = 0
        for p in params:
            k = p.numel()
            self.data[off:off + k].copy_(p.data.reshape(-1))
            p.data = self.data[off:off + k].view_as(p)
            p.main_grad = self.main_grad[off:off + k].view(p.shape)  # type: ignore[attr-defined]
            off += k
        self.lo = heap.rank * self.shard
        self.master = self.data[self.lo:self.lo + self.shard].float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)


class ShardedNVLinkAdamW(MixedPrecisionAdamW):
    """Data-parallel AdamW whose gradient reduction and parameter broadcast are NVLink P2P kernels.

    ``step()`` runs, on the current stream: barrier -> per-arena P2P reduce-scatter (FP32, fixed rank
    order, scale 1/N) -> payload barrier carrying the norm partials -> AdamW on this rank's shard with
    the new parameters stored into every peer's arena -> barrier.  Master weights and Adam moments
    are sharded (1/N of the FP32 optimizer state per rank).  After ``step`` returns, every rank holds
    identical parameters; ``main_grad`` holds the averaged gradient only in this rank's shard.
    """

    def __init__(self, module: nn.Module, cfg: AdamWConfig, heap) -> None:
        self.cfg = cfg
        self.heap = heap
        params = [p for p in module.parameters() if p.requires_grad]
        self.arenas = []
        for dt in (torch.bfloat16, torch.float32):
            group = [p for p in params if p.dtype == dt]
            if group:
                self.arenas.append(_ShardedArena(group, dt, heap))
        if any(p.dtype not in (torch.bfloat16, torch.float32) for p in params):
            raise TypeError("unsupported parameter dtype")
        self.step_count = 0
        self._partials = torch.zeros(len(self.arenas) * 1184, dtype=torch.float32, device=heap.device)
        self._norm = torch.zeros(1, dtype=torch.float32, device=heap.device)
        self._hooks = [p.register_post_accumulate_grad_hook(self._fold) for a in self.arenas for p in a.params]

    def step(self, *, grad_norm: Tensor | None = None) -> Tensor:
        c = self.cfg
        m = kernels()
        h = self.heap
        self.step_count += 1
        b1, b2 = c.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        h.barrier()                                        # every rank's backward has finished
        for i, a in enumerate(self.arenas):
            m.dp_reduce_scatter(a.grad_buf.ptrs, h.rank, a.lo, a.shard, 1.0 / h.size,
                                self._partials[i * 1184:(i + 1) * 1184])
        h.barrier(payload=self._partials)                  # norm partials -> every peer; reads are done
        for a in self.arenas:
            m.dp_adamw_allgather(a.master, a.m, a.v, a.main_grad[a.lo:a.lo + a.shard], a.data_buf.ptrs, a.lo,
                                 a.bf16, h.pad.ptrs[h.rank], float(c.grad_clip), float(c.lr), float(b1), float(b2),
                                 float(c.eps), float(c.weight_decay), float(bc1), float(bc2), self._norm)
        h.barrier()                                        # all parameter stores have landed
        return self._norm[0].clone()

    def grad_norm(self) -> Tensor:
        raise NotImplementedError("the sharded optimizer computes the norm inside step()")

    def state_dict(self) -> dict:
        import torch.distributed as dist

        out = []
        for a in self.arenas:
            full = {}
            for name in ("master", "m", "v"):
                parts = [torch.empty_like(a.master) for _ in range(self.heap.size)]
                dist.all_gather(parts, getattr(a, name).contiguous(), group=self.heap.group)
                full[name] = torch.cat(parts)[:a.numel]
            out.append(full)
        return {"step": self.step_count, "arenas": out}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for a, s in zip(self.arenas, sd["arenas"]):
            for name in ("master", "m", "v"):
                src = s[name].to(a.master.device).float().reshape(-1)
                pad = torch.zeros(a.shard * self.heap.size, dtype=torch.float32, device=a.master.device)
                pad[:src.numel()] = src
                getattr(a, name).copy_(pad[a.lo:a.lo + a.shard])
            full = torch.zeros(a.shard * self.heap.size, dtype=torch.float32, device=a.master.device)
            full[:s["master"].numel()] = s["master"].to(a.master.device).float().reshape(-1)
            a.data.copy_(full.to(a.data.dtype))

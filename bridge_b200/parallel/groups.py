"""Process-group layout for TP x CP x EP x DP on one node (or any world).

Ranks are laid out TP-fastest: ``rank = ((dp * CP) + cp) * TP + tp``, so a TP
group is a set of adjacent GPUs (same NVSwitch domain either way on one HGX
box, but adjacent ranks keep the layout identical to Megatron's default).  The
expert-parallel group reuses the data-parallel x context-parallel ranks of one
TP slice (EP is carved out of DP*CP, as in Megatron's expert layout).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    tp: int = 1
    cp: int = 1
    dp: int = 1
    ep: int = 1
    tp_group: object = None
    cp_group: object = None
    dp_group: object = None
    ep_group: object = None
    dp_cp_group: object = None
    cp_ranks: tuple[int, ...] = (0,)

    @property
    def tp_rank(self) -> int:
        return self.rank % self.tp

    @property
    def cp_rank(self) -> int:
        return (self.rank // self.tp) % self.cp

    @property
    def dp_rank(self) -> int:
        return self.rank // (self.tp * self.cp)


def init_distributed(backend: str | None = None, timeout_s: float = 600.0) -> tuple[int, int]:
    """Initialise the default process group from torchrun env vars (no-op when absent)."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    if "RANK" not in os.environ or "WORLD_SIZE" not in os.environ:
        return 0, 1
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()


def build_parallel_state(tp: int = 1, cp: int = 1, ep: int = 1) -> ParallelState:
    if not dist.is_initialized():
        if tp * cp * ep != 1:
            raise RuntimeError("TP/CP/EP > 1 needs an initialised process group")
        return ParallelState()
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % (tp * cp):
        raise ValueError(f"world size {world} is not divisible by TP*CP = {tp * cp}")
    dp = world // (tp * cp)
    if (dp * cp) % ep:
        raise ValueError(f"EP {ep} must divide DP*CP = {dp * cp}")
    st = ParallelState(world, rank, tp, cp, dp, ep)

    def grp(ranks):
        return dist.new_group(ranks)

    # Every rank must call new_group for every group, in the same order.
    for d in range(dp):
        for c in range(cp):
            ranks = [(d * cp + c) * tp + t for t in range(tp)]
            g = grp(ranks)
            if rank in ranks:
                st.tp_group = g
    for d in range(dp):
        for t in range(tp):
            ranks = [(d * cp + c) * tp + t for c in range(cp)]
            g = grp(ranks)
            if rank in ranks:
                st.cp_group, st.cp_ranks = g, tuple(ranks)
    for c in range(cp):
        for t in range(tp):
            ranks = [(d * cp + c) * tp + t for d in range(dp)]
            g = grp(ranks)
            if rank in ranks:
                st.dp_group = g
    for t in range(tp):
        ranks = [i for i in range(world) if i % tp == t]
        g = grp(ranks)
        if rank in ranks:
            st.dp_cp_group = g
        for e0 in range(0, len(ranks), ep):
            sub = ranks[e0:e0 + ep]
            ge = grp(sub)
            if rank in sub:
                st.ep_group = ge
    if tp == 1:
        st.tp_group = None
    if cp == 1:
        st.cp_group = None
    if ep == 1:
        st.ep_group = None
    return st


def collective_probe(group=None, device=None) -> None:
    """Pre-flight rank-coded all-reduce: ``sum(rank+1)`` must equal ``n(n+1)/2`` (fails loudly otherwise)."""
    if not dist.is_initialized():
        return
    n = dist.get_world_size(group)
    r = dist.get_rank(group)
    t = torch.tensor([float(r + 1)], device=device)
    dist.all_reduce(t, group=group)
    want = n * (n + 1) / 2
    if abs(float(t.item()) - want) > 1e-3:
        raise RuntimeError(f"collective probe failed: got {float(t.item())}, expected {want}")

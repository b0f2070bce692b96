"""Symmetric peer memory for one process group on one node (CUDA IPC over NVLink / NVSwitch).

Every rank of the group allocates the same-sized buffer; the IPC handles are exchanged once over
the process group and opened, so each rank holds a device pointer to every peer's copy.  Kernels
then read and write peers' buffers directly (P2P loads / stores).  A 256-byte signal pad per rank
carries the flags of :meth:`SymmetricHeap.barrier` (a cross-GPU barrier kernel with a bounded
wait) and an optional FP64 payload per peer (used for the global gradient-norm partials).

The group must be single-node (all peers reachable by NVLink P2P) and at most 8 ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops._ext import kernels


class SymmetricBuffer:
    """``local`` (uint8 device tensor of this rank) plus ``ptrs[j]`` = device address of rank j's copy."""

    def __init__(self, local: Tensor, ptrs: list[int], opened: list[int]) -> None:
        self.local = local
        self.ptrs = ptrs
        self._opened = opened

    def view(self, dtype: torch.dtype, numel: int | None = None) -> Tensor:
        t = self.local.view(dtype)
        return t if numel is None else t[:numel]

    def close(self) -> None:
        m = kernels()
        for p in self._opened:
            m.symm_close(p)
        self._opened = []


class SymmetricHeap:
    def __init__(self, group, device: torch.device | None = None, *, timeout_s: float | None = None) -> None:
        import os

        if timeout_s is None:
            timeout_s = float(os.environ.get("BB_SYMM_TIMEOUT_S", "60"))
        self._debug = os.environ.get("BB_SYMM_DEBUG") == "1"
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        if self.size > 8:
            raise ValueError("symmetric heap supports at most 8 ranks (one NVLink domain)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.timeout_s = timeout_s
        self.epoch = 0
        self.buffers: list[SymmetricBuffer] = []
        self.pad = self.alloc(kernels().symm_pad_bytes())

    def alloc(self, nbytes: int) -> SymmetricBuffer:
        """Zero-filled symmetric buffer of ``nbytes`` (rounded up to 256 B) on every rank (collective call)."""
        m = kernels()
        nbytes = (int(nbytes) + 255) // 256 * 256
        with torch.cuda.device(self.device):
            local, handle = m.symm_alloc(nbytes)
            local.zero_()
            torch.cuda.synchronize()
            handles: list = [None] * self.size
            dist.all_gather_object(handles, handle.tolist(), group=self.group)
            ptrs, opened = [], []
            for j, h in enumerate(handles):
                if j == self.rank:
                    ptrs.append(local.data_ptr())
                else:
                    p = m.symm_open(torch.tensor(h, dtype=torch.uint8))
                    ptrs.append(p)
                    opened.append(p)
        dist.barrier(group=self.group)
        buf = SymmetricBuffer(local, ptrs, opened)
        self.buffers.append(buf)
        return buf

    def barrier(self, payload: Tensor | None = None, *, timeout_s: float | None = None) -> None:
        """Stream-ordered cross-GPU barrier; ``payload`` (FP32 partials) is summed and published to every peer."""
        self.epoch += 1
        if self._debug:
            import sys
            import traceback

            where = traceback.extract_stack(limit=4)[0]
            print(f"[symm r{self.rank}] barrier epoch {self.epoch} from {where.name}:{where.lineno}",
                  file=sys.stderr, flush=True)
        kernels().symm_barrier(self.pad.ptrs, self.rank, self.epoch, payload,
                               float(self.timeout_s if timeout_s is None else timeout_s))

    def payload_slots(self) -> Tensor:
        """This rank's view of the FP64 payload slots (one per peer) written by the last payload barrier."""
        return self.pad.local[64:64 + 8 * self.size].view(torch.float64)

    def check(self) -> None:
        """Raise if any barrier wait on this device timed out (a peer never arrived)."""
        code = kernels().symm_error_code()
        if code:
            kernels().symm_clear_error()
            raise RuntimeError(f"symmetric-memory barrier timed out waiting for peer {code - 0x100}")

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for b in self.buffers:
            b.close()
        dist.barrier(group=self.group)
        self.buffers = []

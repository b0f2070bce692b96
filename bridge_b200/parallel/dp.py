"""Data-parallel gradient finalisation over the FP32 main-gradient arenas.

``finalize`` averages every arena across the DP (x CP) group in fixed-size
buckets.  Each bucket is cast to bf16 for the wire (halving NVLink bytes) on the
compute stream and all-reduced by NCCL on a side stream while the next bucket is
being cast; afterwards each reduced bucket is copied back into the FP32 arena and
scaled by ``1/dp`` (two torch elementwise ops).  ``comm_dtype=float32`` keeps the
wire in FP32.  This is the NCCL baseline path; the fused path (P2P reduce-scatter
with the scale applied in the same kernel, then sharded AdamW) is
:class:`~bridge_b200.engine.optim.ShardedNVLinkAdamW`.

Parity: the once-per-forest ``finalize_model_grads(force_all_reduce=True)``
call of verl/models/mcore/tpr/tpr_batch_runner.py:75 and
megatron_adapter.py:189-192,457-461.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


class DataParallelGradReducer:
    def __init__(self, group, *, bucket_bytes: int = 256 << 20, comm_dtype=torch.bfloat16) -> None:
        self.group = group
        self.size = 1 if group is None else dist.get_world_size(group)
        self.bucket_elems = max(1, bucket_bytes // 4)
        self.comm_dtype = comm_dtype
        self._stream = torch.cuda.Stream() if torch.cuda.is_available() else None

    def finalize(self, buffers: list[Tensor]) -> None:
        if self.size == 1:
            return
        scale = 1.0 / self.size
        for buf in buffers:
            n = buf.numel()
            if not buf.is_cuda or self.comm_dtype == torch.float32:
                for s in range(0, n, self.bucket_elems):
                    part = buf[s:s + self.bucket_elems]
                    dist.all_reduce(part, group=self.group)
                    part.mul_(scale)
                continue
            pending = []
            main = torch.cuda.current_stream()
            for s in range(0, n, self.bucket_elems):
                part = buf[s:s + self.bucket_elems]
                wire = part.to(self.comm_dtype)
                ev = torch.cuda.Event()
                ev.record(main)
                with torch.cuda.stream(self._stream):
                    self._stream.wait_event(ev)
                    dist.all_reduce(wire, group=self.group)
                    wire.record_stream(self._stream)
                    done = torch.cuda.Event()
                    done.record(self._stream)
                pending.append((part, wire, done))
            for part, wire, done in pending:
                main.wait_event(done)
                part.copy_(wire).mul_(scale)

"""Opt-in capture of the real actor-update mini-batch for offline replay and benchmarks.

Enabled by ``TPR_CAPTURE_DIR`` (directory).  Each call writes
``step{global_step:08d}_rank{rank:05d}_capture{index:06d}_batch{batch_idx}.pt`` atomically (write to a
temporary name in the same directory, then ``os.replace``) and refuses to overwrite an existing
capture.  The file holds the batch exactly as the engine receives it (tensors moved to CPU), the
trajectory keys the engine will use, and the step / rank / index labels.  All rows of a mini-batch
must share one integer ``global_steps`` value.  Captures contain trajectory data; keep them private.

:func:`load_capture` returns the batch dict ready for ``TPREngine.forward_backward_batch``.

Parity: verl/models/mcore/tpr/actor_capture.py:30-120 (fail-closed global step, atomic,
no-overwrite, rank labels).
"""

from __future__ import annotations

import os
import tempfile
from typing import Any

import torch

ENV_DIR = "TPR_CAPTURE_DIR"


def _global_step(batch: dict) -> int:
    raw = batch.get("global_steps")
    if raw is None:
        raise ValueError("actor capture needs the batch's global_steps field")
    values = torch.as_tensor(raw).reshape(-1)
    if values.dtype not in (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64):
        raise TypeError(f"global_steps must be integer, got {values.dtype}")
    if values.numel() == 0 or not bool(torch.all(values == values[0])):
        raise ValueError("global_steps must be one value shared by every row of the mini-batch")
    step = int(values[0])
    if step < 0:
        raise ValueError(f"global_steps must be non-negative, got {step}")
    return step


def _to_cpu(x: Any) -> Any:
    if isinstance(x, torch.Tensor):
        return x.detach().cpu()
    if isinstance(x, (list, tuple)):
        return type(x)(_to_cpu(v) for v in x)
    if isinstance(x, dict):
        return {k: _to_cpu(v) for k, v in x.items()}
    return x


def capture_actor_update_minibatch(batch: dict, *, batch_idx: int, capture_index: int = 0, rank: int | None = None,
                                   directory: str | None = None) -> str | None:
    """Write one capture when ``TPR_CAPTURE_DIR`` (or ``directory``) is set; returns its path."""
    directory = directory or os.environ.get(ENV_DIR)
    if not directory:
        return None
    if not isinstance(capture_index, int) or capture_index < 0:
        raise ValueError("capture_index must be a non-negative integer")
    step = _global_step(batch)
    if rank is None:
        import torch.distributed as dist

        rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
    os.makedirs(directory, exist_ok=True)
    target = os.path.join(directory, f"step{step:08d}_rank{rank:05d}_capture{capture_index:06d}_batch{batch_idx}.pt")
    if os.path.exists(target):
        raise FileExistsError(f"refusing to overwrite an existing actor-update capture: {target}")
    from ..engine.api import trajectory_keys_from_minibatch

    payload = {"batch": _to_cpu(batch), "trajectory_keys": list(trajectory_keys_from_minibatch(batch)),
               "capture_stage": "actor_update_mini_batch", "capture_global_rank": rank,
               "capture_global_step": step, "capture_index": capture_index, "capture_mini_batch_idx": batch_idx}
    fd, tmp = tempfile.mkstemp(dir=directory, prefix=".capture_", suffix=".tmp")
    try:
        with os.fdopen(fd, "wb") as f:
            torch.save(payload, f)
        if os.path.exists(target):
            raise FileExistsError(f"refusing to overwrite an existing actor-update capture: {target}")
        os.replace(tmp, target)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)
    return target


def load_capture(path: str) -> dict:
    payload = torch.load(path, map_location="cpu", weights_only=False)
    batch = dict(payload["batch"])
    batch.setdefault("tpr_trajectory_keys", payload["trajectory_keys"])
    return batch

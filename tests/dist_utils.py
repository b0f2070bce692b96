"""Spawn helpers for multi-process gloo tests (CPU, 127.0.0.1)."""

from __future__ import annotations

import os
import socket
import traceback

import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, "err", f"{exc!r}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(world: int, fn, *args, timeout: float = 600.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    import queue as _q

    try:
        for _ in range(world):
            rank, status, out = q.get(timeout=timeout)
            if status != "ok":
                raise AssertionError(f"rank {rank} failed:\n{out}")
            results[rank] = out
    except _q.Empty as exc:
        raise AssertionError("ranks timed out") from exc
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [results[r] for r in range(world)]

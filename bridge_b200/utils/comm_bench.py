"""Fused compute+collective kernels vs their NCCL baselines (run under torch.distributed.run).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m bridge_b200.utils.comm_bench --op all

Each case is timed with CUDA events on the launching stream (3 warm-up, median of 10, barrier +
synchronize around each timed launch) and reported as the max over ranks, with the fused path's
roofline: the slower of its GEMM FLOPs at the measured bf16 peak and its NVLink bytes per GPU at the
measured 770 GB/s peer-copy bandwidth.
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .kernel_bench import peaks

NVLINK_GBS = 770.0


def _time(fn, warmup=3, iters=10) -> float:
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    t = torch.tensor([times[len(times) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _emit(rank, d):
    if rank == 0:
        print(json.dumps(d), flush=True)


def bench_tp(rank: int, world: int, tokens: int):
    from bridge_b200.ops.gemm import gemm
    from bridge_b200.parallel import tp_fused as tf

    _, tflops, _ = peaks()
    g = dist.group.WORLD
    ms = tokens // world
    cases = [("ag_qkv", 2560, 6144 // world), ("ag_fc1", 2560, 19456 // world)]
    for name, k, n in cases:
        x = torch.randn(ms, k, device="cuda").bfloat16()
        w = torch.randn(n, k, device="cuda").bfloat16()
        comm = tf.fused_comm(g, x)
        full = torch.empty(ms * world, k, device="cuda", dtype=torch.bfloat16)
        fused = _time(lambda: comm.ag_gemm(x, w, b_mn=False))

        def base():
            dist.all_gather_into_tensor(full, x, group=g)
            gemm(full, w)

        nccl = _time(base)
        flops = 2.0 * ms * world * n * k
        roof = max(flops / (tflops * 1e9), (world - 1) * ms * k * 2 / (NVLINK_GBS * 1e6))
        _emit(rank, {"op": f"tp_{name}", "tp": world, "M": ms * world, "N": n, "K": k, "fused_ms": round(fused, 4),
                     "nccl_gemm_ms": round(nccl, 4), "roofline_ms": round(roof, 4),
                     "frac_of_roofline": round(roof / fused, 3), "speedup_vs_nccl": round(nccl / fused, 3)})
    cases = [("rs_o", 4096 // world, 2560), ("rs_fc2", 9728 // world, 2560)]
    for name, k, n in cases:
        x = torch.randn(ms * world, k, device="cuda").bfloat16()
        w = torch.randn(n, k, device="cuda").bfloat16()
        comm = tf.fused_comm(g, x)
        out = torch.empty(ms, n, device="cuda", dtype=torch.bfloat16)
        fused = _time(lambda: comm.gemm_rs(x, w, b_mn=False))

        def base():
            y = gemm(x, w)
            dist.reduce_scatter_tensor(out, y, group=g)

        nccl = _time(base)
        flops = 2.0 * ms * world * n * k
        roof = max(flops / (tflops * 1e9), (world - 1) * ms * n * 2 / (NVLINK_GBS * 1e6))
        _emit(rank, {"op": f"tp_{name}", "tp": world, "M": ms * world, "N": n, "K": k, "fused_ms": round(fused, 4),
                     "nccl_gemm_ms": round(nccl, 4), "roofline_ms": round(roof, 4),
                     "frac_of_roofline": round(roof / fused, 3), "speedup_vs_nccl": round(nccl / fused, 3)})


def bench_dp(rank: int, world: int, numel: int):
    """Optimizer step with gradient reduction: fused NVLink (RS -> sharded AdamW -> P2P AG) vs NCCL."""
    from torch import nn

    from bridge_b200.engine.optim import AdamWConfig, MixedPrecisionAdamW, ShardedNVLinkAdamW
    from bridge_b200.parallel.dp import DataParallelGradReducer
    from bridge_b200.parallel.symmetric import SymmetricHeap

    cfg = AdamWConfig(lr=1e-6)
    m1 = nn.Linear(numel // 4096, 4096, bias=False, device="cuda", dtype=torch.bfloat16)
    m2 = nn.Linear(numel // 4096, 4096, bias=False, device="cuda", dtype=torch.bfloat16)
    heap = SymmetricHeap(dist.group.WORLD)
    fused_opt = ShardedNVLinkAdamW(m1, cfg, heap)
    base_opt = MixedPrecisionAdamW(m2, cfg)
    red = DataParallelGradReducer(dist.group.WORLD)
    for o in (fused_opt, base_opt):
        for a in o.arenas:
            a.main_grad.normal_()
    fused = _time(lambda: fused_opt.step())

    def base():
        red.finalize(base_opt.grad_buffers())
        base_opt.step()

    nccl = _time(base)
    n = m1.weight.numel()
    nv_bytes = (world - 1) / world * n * (4 + 2)        # FP32 gradient shards in, bf16 parameter shards out
    roof = max(nv_bytes / (NVLINK_GBS * 1e6), (n / world * 30 + n * 4 * 2) / (peaks()[0] * 1e6))
    _emit(rank, {"op": "dp_grad_reduce_adamw", "dp": world, "params": n, "fused_ms": round(fused, 3),
                 "nccl_bf16_allreduce_plus_adamw_ms": round(nccl, 3), "roofline_ms": round(roof, 3),
                 "frac_of_roofline": round(roof / fused, 3), "speedup_vs_nccl": round(nccl / fused, 3)})
    heap.close()


def main(argv=None):
    from bridge_b200.parallel.groups import init_distributed

    p = argparse.ArgumentParser()
    p.add_argument("--op", default="all", choices=["all", "tp", "dp"])
    p.add_argument("--tokens", type=int, default=4608)
    p.add_argument("--dp-params", type=int, default=1 << 30)
    a = p.parse_args(argv)
    rank, world = init_distributed(timeout_s=300)
    if a.op in ("all", "tp"):
        bench_tp(rank, world, a.tokens)
    if a.op in ("all", "dp"):
        bench_dp(rank, world, a.dp_params)
    from bridge_b200.parallel import tp_fused as tf

    tf.close_all()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""PPO actor-update throughput with tree-prefix reuse on B200.

Config (BASELINE config #2): Qwen3-4B (36 layers, hidden 2560, 32q/8kv heads of 128, FFN 9728,
vocab 151936, qk-RMSNorm, RoPE 1e6), bf16 weights with FP32 master weights and Adam state; every
tree is a 512-token prompt with 8 sibling responses of 512 tokens; ids uniform from a seed,
advantages ~ N(0,1), response mask all ones; random-init weights (no checkpoint access).
Weak scaling: ``--trees-per-gpu`` trees per GPU (8 -> 64 trees on 8 GPUs, the named config).

Parallel layout: by default the named config's TP2 x CP4 at 8 GPUs, scaled down along the same axes
(1 GPU: none, 2: TP2, 4: TP2 x CP2, 8: TP2 x CP4); TP runs with sequence parallelism.  ``--tp`` /
``--cp`` override it (``--tp 1 --cp 1`` = pure data parallelism).

``--config 3|4|5`` runs the other BASELINE configs (same metric, same timing): #3 multi-turn session
trees (qwen_turn policy, 50 % loss mask) on Qwen3-4B at CP = N with activation offload; #4 the hybrid
GDN/attention model (24 layers, 3 GDN : 1 gated attention, head_dim 256) on 512 + 8 x 512 trees at
the #2 layout; #5 the Qwen3-Next-shape hybrid MoE (512 experts, top-10, 24 layers) on 1024 + 8 x 1024
trees at CP2 x EP(N) (CP only from 2 GPUs).

One step = plan the token-trie forest, forward + backward of every segment (prefix KV relayed),
PPO loss over all supervised tokens, DP gradient finalisation, fused AdamW update.

``value``: device time of K steps (CUDA events on the launching stream, barrier + synchronize on
both sides, max over ranks), with planned inputs already staged.  ``e2e``: the same K steps through
the public API (``TPREngine.train_step`` on a pinned-host batch: planning, H2D of the inputs, D2H
of the loss each step), wall clock, max over ranks.

``--impl reference`` runs the reference implementation; it cannot run on this machine (see the
JSON line it prints).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

PUBLISHED_TPR_TOKENS_PER_S = 2456.0  # 36 933 PPO tokens / 15.035786 s, TPR TP2xCP4 on 8x Ascend 910B
METRIC = "PPO actor-update tokens/s (whole box, max over ranks) w/ TPR at 1/2/4/8 B200"


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="bridge", choices=["bridge", "reference"])
    p.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5], help="BASELINE config number")
    p.add_argument("--model", default=None, help="default: the config's model")
    p.add_argument("--num-layers", type=int, default=None,
                   help="truncate the model (a functional check on fewer GPUs; not the named config)")
    p.add_argument("--trees-per-gpu", type=int, default=None, help="default: the config's (8, #3: 2 sessions)")
    p.add_argument("--prefix", type=int, default=None)
    p.add_argument("--siblings", type=int, default=8)
    p.add_argument("--resp", type=int, default=None)
    p.add_argument("--token-budget", type=int, default=int(os.environ.get("TPR_TOKEN_BUDGET", "0")) or None)
    p.add_argument("--mode", default=os.environ.get("TPR_FOREST_MODE"), help="default: the config's (#3: recompute)")
    p.add_argument("--tp", type=int, default=None, help="default: the config-#2 layout for --gpus")
    p.add_argument("--cp", type=int, default=None, help="default: the config-#2 layout for --gpus")
    p.add_argument("--no-sp", action="store_true", help="TP without sequence parallelism")
    p.add_argument("--dp-comm", default="auto", choices=["auto", "nvlink", "nccl"],
                   help="DP gradient path: fused NVLink P2P kernels + sharded optimizer, or NCCL all-reduce")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--ep", type=int, default=None, help="expert parallel size (MoE; default: config #5 layout)")
    p.add_argument("--profile-step", default=None, metavar="PATH",
                   help="instead of timing: profile one step after the warm-up (torch.profiler CUDA activity) and "
                        "write the per-kernel self device time table of each rank to PATH.rank<r>.txt")
    a = p.parse_args()
    d = CONFIG_DEFAULTS[a.config]
    for k, v in d.items():
        if getattr(a, k) is None:
            setattr(a, k, v)
    return a


# per-config defaults: model, tree shape, per-rank token budget
CONFIG_DEFAULTS = {
    2: dict(model="qwen3_4b", trees_per_gpu=8, prefix=512, resp=512, token_budget=16384, mode="retain"),
    # sessions: shared turns of up to 24k tokens (cut into budget-sized prefix pieces), pushed segments
    # recomputed at pop time (the reference's memory profile) so only one chunk's activations exist at a
    # time, offloaded to pinned host memory
    3: dict(model="qwen3_4b", trees_per_gpu=2, prefix=0, resp=0, token_budget=16384, mode="recompute"),
    4: dict(model="hybrid_gdn_2b", trees_per_gpu=8, prefix=512, resp=512, token_budget=16384, mode="retain"),
    5: dict(model="qwen3_next_24l", trees_per_gpu=4, prefix=1024, resp=1024, token_budget=16384, mode="retain"),
}


# gpus -> (tp, cp, ep): each config's named layout at 8 GPUs, scaled down along the same axes
DEFAULT_LAYOUT = {
    2: {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 4, 1)},
    3: {1: (1, 1, 1), 2: (1, 2, 1), 4: (1, 4, 1), 8: (1, 8, 1)},
    4: {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (2, 4, 1)},
    5: {1: (1, 1, 1), 2: (1, 2, 2), 4: (1, 2, 4), 8: (1, 2, 8)},
}


def layout(args) -> tuple[int, int, int]:
    tp_d, cp_d, ep_d = DEFAULT_LAYOUT[args.config].get(args.gpus, (1, 1, 1))
    pick = lambda v, d: d if v is None else v  # noqa: E731
    return pick(args.tp, tp_d), pick(args.cp, cp_d), pick(args.ep, ep_d)


def parallelism_name(tp: int, cp: int, dp: int, ep: int = 1) -> str:
    parts = [f"tp{tp}"] if tp > 1 else []
    parts += [f"cp{cp}"] if cp > 1 else []
    parts += [f"ep{ep}"] if ep > 1 else []
    parts += [f"dp{dp}"] if (dp > 1 and ep == 1) or not parts else []
    return "".join(parts)


def local_gpu_indices() -> str | None:
    """nvidia-smi indices of the GPUs this node's ranks use (local rank i -> visible device i)."""
    n = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = [x.strip() for x in vis.split(",") if x.strip()] if vis else [str(i) for i in range(n)]
    return ",".join(ids[:n]) if ids else None


def reference_unavailable(args) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({
            "impl": "reference",
            "unavailable": "the reference is a verl/Megatron extension with no setup.py/pyproject (pip: 'not "
                           "installable') whose kernels are Ascend-only (torch_npu, MindSpeed, MindSpeed-Ops); none "
                           "of them exists on this CUDA image",
            "metric": METRIC, "n_gpus": args.gpus,
        }), flush=True)


def synthetic_batch(args, n_trees: int, rank: int, dp: int, vocab: int, device_pin: bool) -> dict:
    """``n_trees`` trees for data-parallel rank ``rank`` (the mini-batch of one model replica)."""
    g = torch.Generator().manual_seed(args.seed * 1000003 + rank)
    ids, masks, old, adv, uids = [], [], [], [], []
    for t in range(n_trees):
        prompt = torch.randint(0, vocab, (args.prefix,), generator=g)
        for s in range(args.siblings):
            resp = torch.randint(0, vocab, (args.resp,), generator=g)
            ids.append(torch.cat([prompt, resp]))
            masks.append(torch.ones(args.resp, dtype=torch.bool))
            adv.append(torch.randn(args.resp, generator=g))
            old.append(torch.full((args.resp,), -11.93) - torch.rand(args.resp, generator=g) * 0.01)
            uids.append(f"r{rank}t{t}")
    if device_pin and torch.cuda.is_available():
        ids = [x.pin_memory() for x in ids]
        masks = [x.pin_memory() for x in masks]
        old = [x.pin_memory() for x in old]
        adv = [x.pin_memory() for x in adv]
    per_rank = n_trees * args.siblings * args.resp
    return {"input_ids": ids, "response_mask": masks, "old_log_probs": old, "advantages": adv, "uid": uids,
            "temperature": 1.0, "batch_num_tokens": per_rank * dp, "dp_size": dp}


IM_END = 151645          # Qwen ChatML <|im_end|>: the turn boundary the qwen_turn trie policy cuts at


def session_batch(args, n_sessions: int, rank: int, dp: int, vocab: int, device_pin: bool) -> dict:
    """Config #3: multi-turn agent sessions.  Six turns of U[2k, 6k] tokens (each ending in <|im_end|>);
    every session forks into 4 branches at each of its last two turn boundaries (16 rows per session),
    capped at 48k tokens; the prompt is turn 1 and the loss covers a random half of the response
    tokens (the assistant spans)."""
    g = torch.Generator().manual_seed(args.seed * 1000003 + 7919 * rank + 3)

    def turn():
        n = int(torch.randint(2048, 6145, (1,), generator=g))
        t = torch.randint(0, vocab - 1, (n,), generator=g)
        t[t == IM_END] = IM_END - 1
        t[-1] = IM_END
        return t

    ids, masks, old, adv, uids = [], [], [], [], []
    for sess in range(n_sessions):
        shared = [turn() for _ in range(4)]
        for b in range(4):
            t5 = turn()
            for c in range(4):
                t6 = turn()
                row = torch.cat(shared + [t5, t6])[:48 * 1024]
                n_resp = row.numel() - shared[0].numel()
                m = torch.rand(n_resp, generator=g) < 0.5
                ids.append(row)
                masks.append(m)
                adv.append(torch.randn(n_resp, generator=g))
                old.append(torch.full((n_resp,), -11.93) - torch.rand(n_resp, generator=g) * 0.01)
                uids.append(f"r{rank}s{sess}")
    if device_pin and torch.cuda.is_available():
        ids, masks, old, adv = ([x.pin_memory() for x in lst] for lst in (ids, masks, old, adv))
    local = sum(int(m.sum()) for m in masks)
    return {"input_ids": ids, "response_mask": masks, "old_log_probs": old, "advantages": adv, "uid": uids,
            "temperature": 1.0, "batch_num_tokens": local, "dp_size": dp}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str | None) -> None:
        self.proc = None
        self.lines: list[str] = []
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if gpus:
            cmd[1:1] = ["-i", gpus]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        clocks, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                clocks.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(clocks) if clocks else None,
                "sm_max_mhz": max(maxes) if maxes else None, "reasons": sorted(reasons), "samples": len(clocks)}


def profile_one_step(args, device_step, rank: int, world: int) -> None:
    """Per-kernel self device time of one step (the number a profiled run prints is not a bench value)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        device_step()
        torch.cuda.synchronize()
    rows = []
    for evt in prof.key_averages():
        t = getattr(evt, "self_device_time_total", None)
        if t is None:
            t = getattr(evt, "self_cuda_time_total", 0)
        if t > 0:
            rows.append((t / 1e3, evt.count, evt.key))
    rows.sort(reverse=True)
    total = sum(r[0] for r in rows)
    lines = [f"# one step, rank {rank} of {world}, config #{args.config}, model {args.model}",
             f"# TOTAL device ms {total:.2f}", "| kernel | ms / step | launches |", "|---|---|---|"]
    lines += [f"| {k[:90]} | {ms:.2f} | {n} |" for ms, n, k in rows[:60]]
    with open(f"{args.profile_step}.rank{rank}.txt", "w") as f:
        f.write("\n".join(lines) + "\n")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return
    from bridge_b200.engine import EngineConfig, TPREngine
    from bridge_b200.engine.api import execute_prepared_tpr_batch, prepare_tpr_batch
    from bridge_b200.engine.optim import AdamWConfig
    from bridge_b200.models import get_config
    from bridge_b200.ops._ext import ext
    from bridge_b200.parallel.groups import collective_probe, init_distributed

    rank, world = init_distributed(timeout_s=900)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        collective_probe(device=dev)
    cfg = get_config(args.model) if args.num_layers is None else get_config(args.model, num_layers=args.num_layers)
    tp, cp, ep = layout(args)
    sp = tp > 1 and not args.no_sp
    ec = EngineConfig(tensor_model_parallel_size=tp, context_parallel_size=cp, expert_model_parallel_size=ep,
                      sequence_parallel=sp, token_budget=args.token_budget, forest_mode=args.mode,
                      tpr_cp_backend="ring" if cp > 1 else None, dp_comm=args.dp_comm,
                      activation_offload=args.config == 3,
                      tree_policy="qwen_turn" if args.config == 3 else "exact",
                      gdn_cp_mode="sequence" if args.config in (4, 5) else "head")
    eng = TPREngine(cfg, ec, AdamWConfig(lr=1e-6), device=dev, seed=args.seed)
    dp = eng.parallel.dp
    n_trees = args.trees_per_gpu * world                  # weak scaling: trees (sessions) per GPU fixed
    make = session_batch if args.config == 3 else synthetic_batch
    batch = make(args, n_trees // dp, eng.parallel.dp_rank, dp, cfg.vocab_size, device_pin=True)
    tok = torch.tensor([float(batch["batch_num_tokens"])], device=dev)
    if dp > 1 and args.config == 3:                       # random loss masks: the global count is a sum
        dist.all_reduce(tok, group=eng.parallel.dp_group)
        batch["batch_num_tokens"] = int(tok.item())
    ppo_tokens_global = int(batch["batch_num_tokens"])
    prepared = prepare_tpr_batch(eng, batch)
    m = ext()

    def device_step():
        out = execute_prepared_tpr_batch(eng, prepared, sync_loss=False)
        eng.optimizer_step()
        return out

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if args.profile_step:
        profile_one_step(args, device_step, rank, world)
        return
    sampler = ClockSampler(local_gpu_indices()) if rank == 0 else None
    launches0 = m.launch_count()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        out = device_step()
    end.record()
    torch.cuda.synchronize()
    launches = m.launch_count() - launches0
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    loss = float(out["loss"][0].item()) if isinstance(out["loss"][0], torch.Tensor) else out["loss"][0]

    e2e = None
    if not args.no_e2e:
        h2d = sum(x.numel() * x.element_size() for k in ("input_ids", "response_mask", "old_log_probs", "advantages")
                  for x in batch[k])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            r = eng.train_step(batch)      # public API: plan + H2D + F/B + finalize + AdamW + D2H(loss)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps
        w = torch.tensor([wall], device=dev)
        if world > 1:
            dist.all_reduce(w, op=dist.ReduceOp.MAX)
        wall = float(w.item())
        e2e = {"value": ppo_tokens_global / wall, "unit": "tokens/s", "ms_per_step": wall * 1e3,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4 * (1 + len(r["metrics"])),
               "timing": "wall clock around K public-API train_step calls, max over ranks"}

    if rank == 0:
        value = ppo_tokens_global / (ms / 1e3)
        par = parallelism_name(tp, cp, dp, ep)
        named = (args.config, args.model, par, world, n_trees, args.prefix, args.siblings, args.resp) == \
            (2, "qwen3_4b", "tp2cp4", 8, 64, 512, 8, 512) and args.num_layers is None
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            # the published figure is TPR at TP2 x CP4 on 8 Ascend 910B; it is quoted only for that layout
            "vs_baseline": value / PUBLISHED_TPR_TOKENS_PER_S if named else None,
            "dtype": "bf16",
            "data": "synthetic (uniform token ids from seed, advantages N(0,1), random-init weights)",
            "config": {
                "baseline_config": args.config, "model": args.model, "num_layers": cfg.num_layers,
                "truncated": args.num_layers is not None,
                "global_batch": n_trees * (16 if args.config == 3 else args.siblings),
                "seq_len": "6 turns of 2k-6k, <= 48k" if args.config == 3 else args.prefix + args.resp,
                "parallelism": par, "sequence_parallel": sp, "activation_offload": ec.activation_offload,
                "cp_placement": "segment-granular (forest executor)" if cp > 1 else None,
                "trees": n_trees, "prefix": args.prefix, "siblings": args.siblings,
                "response": args.resp, "ppo_tokens_per_step": ppo_tokens_global, "forest_mode": args.mode,
                "token_budget": args.token_budget,
                "dp_comm": "nvlink-p2p-fused" if eng.symm_heap is not None else ("nccl" if world > 1 else "none"),
                "l2": "no flush: every step streams 8 GB of bf16 weights and GB-scale activations (>> 126 MB L2)",
            },
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": launches,
            "peak_mem_gib": round(torch.cuda.max_memory_allocated() / 2**30, 1),
            "loss": loss,
            "impl": "bridge_b200",
        }
        print(json.dumps(line), flush=True)
    if eng.symm_heap is not None:
        eng.symm_heap.check()
        eng.symm_heap.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Per-kernel microbenchmarks at the flagship (Qwen3-4B, 512 + 8x512 tree) shapes.

Every op is timed with CUDA events on the launching stream after warm-up, with an L2 flush
(a 256 MiB write) before each timed launch, and reported as one JSON line with the achieved
bandwidth or FLOP rate and its fraction of the measured roofline (``MEASURED_PEAKS.json`` at the
repository root; fallback 6.65 TB/s and 1.59 PFLOP/s).

    python -m bridge_b200.utils.kernel_bench --op all
    python -m bridge_b200.utils.kernel_bench --op gemm --iters 1 --warmup 1   # small driver for ncu

``--small`` shrinks token counts (inputs stay above the 126 MB L2 for the bandwidth kernels) so a
profiler capture of one launch stays short.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks() -> tuple[float, float, str]:
    """(HBM GB/s, bf16 TFLOP/s burst, label)."""
    try:
        with open(os.path.join(_ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


class Timer:
    def __init__(self, warmup: int, iters: int):
        self.warmup, self.iters = warmup, iters
        self.flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(self.iters):
            self.flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        times.sort()
        return times[len(times) // 2]


def _report(op: str, shape: dict, ms: float, *, bytes_: float = 0.0, flops: float = 0.0) -> dict:
    hbm, tf, label = peaks()
    out = {"op": op, "shape": shape, "ms": round(ms, 4)}
    if bytes_:
        gbs = bytes_ / ms / 1e6
        out.update(gbs=round(gbs, 1), frac_hbm=round(gbs / hbm, 3))
    if flops:
        tfs = flops / ms / 1e9
        out.update(tflops=round(tfs, 1), frac_bf16=round(tfs / tf, 3))
    out["peak"] = label
    print(json.dumps(out), flush=True)
    return out


def bench_gemm(t: Timer, small: bool):
    from bridge_b200.ops.gemm import gemm

    M = 4608 if not small else 2048
    shapes = [("qkv", M, 6144, 2560), ("fc1", M, 19456, 2560), ("fc2", M, 2560, 9728), ("o", M, 2560, 4096)]
    for name, m, n, k in shapes:
        a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        ms = t(lambda: gemm(a, b, out=c))
        _report(f"gemm_{name}", {"M": m, "N": n, "K": k}, ms, flops=2.0 * m * n * k)
        # dgrad (B is MN-major) and wgrad accumulating into an FP32 main_grad
        ms = t(lambda: gemm(c, b, b_mn=True))
        _report(f"gemm_{name}_dgrad", {"M": m, "N": k, "K": n}, ms, flops=2.0 * m * n * k)
        mg = torch.zeros(n, k, device="cuda", dtype=torch.float32)
        ms = t(lambda: gemm(c, a, a_mn=True, b_mn=True, out=mg, accumulate=True))
        _report(f"gemm_{name}_wgrad_acc", {"M": n, "N": k, "K": m}, ms, flops=2.0 * m * n * k)
        if small:
            break


def _tree(small: bool):
    from bridge_b200.tpr.context import SegmentBatchLayout

    sib = 8 if not small else 4
    lens = (512,) * sib
    spans = ((0, 512),) * sib
    hq, hkv, D = 32, 8, 128
    T = sum(lens)
    q = torch.randn(T, hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, hkv, D, device="cuda", dtype=torch.bfloat16)
    pk = torch.randn(512, hkv, D, device="cuda", dtype=torch.bfloat16)
    pv = torch.randn(512, hkv, D, device="cuda", dtype=torch.bfloat16)
    lay = SegmentBatchLayout.build(lens, spans, device="cuda")
    # causal self part + full prefix part per sibling
    flops_fwd = 4.0 * D * hq * sib * (512 * 513 / 2 + 512 * 512)
    return q, k, v, pk, pv, lay, flops_fwd, {"siblings": sib, "len": 512, "prefix": 512, "hq": hq, "hkv": hkv}


def bench_attention(t: Timer, small: bool):
    from bridge_b200.ops._ext import kernels

    m = kernels()
    q, k, v, pk, pv, lay, fl, shape = _tree(small)
    sc = 1 / math.sqrt(128)
    args = (lay.cu_seqlens, lay.prefix_offsets, lay.prefix_lengths, lay.max_seqlen, lay.max_prefix, sc)
    ms = t(lambda: m.tree_attn_fwd_sm100(q, k, v, pk, pv, *args))
    _report("attn_fwd_tcgen05", shape, ms, flops=fl)
    o, lse = m.tree_attn_fwd_sm100(q, k, v, pk, pv, *args)
    do = torch.randn_like(o)
    ms = t(lambda: m.tree_attn_bwd_sm100(do, q, k, v, pk, pv, o, lse, *args))
    _report("attn_bwd_tcgen05", shape, ms, flops=2.5 * fl)
    # forward CTA time split: entry -> first S tile, tile loop, epilogue (one untimed launch)
    m.attn_phase_profile(True)
    m.tree_attn_fwd_sm100(q, k, v, pk, pv, *args)
    torch.cuda.synchronize()
    st, loop, epi, tiles, ctas = [int(x) for x in m.attn_phase_read().tolist()[:5]]
    m.attn_phase_profile(False)
    tot = max(st + loop + epi, 1)
    print(json.dumps({"op": "attn_fwd_phases", "ctas": ctas, "tiles": tiles,
                      "cycles_per_cta": round(tot / max(ctas, 1)), "loop_cycles_per_tile": round(loop / max(tiles, 1)),
                      "share": {"startup": round(st / tot, 3), "loop": round(loop / tot, 3),
                                "epilogue": round(epi / tot, 3)}}))


def bench_elementwise(t: Timer, small: bool):
    from bridge_b200.ops._ext import kernels
    from bridge_b200.ops.norm import rope_cos_sin

    m = kernels()
    T = 32768 if small else 36864  # > L2 for every tensor pair below
    H = 2560
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    y, rstd = m.rmsnorm_fwd(x, w, 1e-6)
    ms = t(lambda: m.rmsnorm_fwd(x, w, 1e-6))
    _report("rmsnorm_fwd", {"T": T, "H": H}, ms, bytes_=2 * x.numel() * 2)
    ms = t(lambda: m.rmsnorm_bwd(y, x, w, rstd))
    _report("rmsnorm_bwd", {"T": T, "H": H}, ms, bytes_=3 * x.numel() * 2)
    r = torch.randn_like(x)
    ms = t(lambda: m.add_rmsnorm_fwd(x, r, w, 1e-6))
    _report("add_rmsnorm_fwd", {"T": T, "H": H}, ms, bytes_=4 * x.numel() * 2)
    ms = t(lambda: m.add_rmsnorm_bwd(y, x, w, rstd, r))
    _report("add_rmsnorm_bwd", {"T": T, "H": H}, ms, bytes_=4 * x.numel() * 2)
    F = 9728
    Ts = T // 4
    gu = torch.randn(Ts, 2 * F, device="cuda", dtype=torch.bfloat16)
    ms = t(lambda: m.swiglu_fwd(gu))
    _report("swiglu_fwd", {"T": Ts, "F": F}, ms, bytes_=3 * Ts * F * 2)
    dy = torch.randn(Ts, F, device="cuda", dtype=torch.bfloat16)
    ms = t(lambda: m.swiglu_bwd(dy, gu))
    _report("swiglu_bwd", {"T": Ts, "F": F}, ms, bytes_=5 * Ts * F * 2)
    Tq = T // 2
    # q and k read in place from the fused QKV projection output, as the attention layer does
    qkv = torch.randn(Tq, 48 * 128, device="cuda", dtype=torch.bfloat16)
    q = qkv[:, :32 * 128].view(Tq, 32, 128)
    k = qkv[:, 32 * 128:40 * 128].view(Tq, 8, 128)
    qw = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    cos, sin = rope_cos_sin(torch.arange(Tq, device="cuda"), 128, 1e6)
    qo, ko, rq, rk = m.qk_norm_rope_fwd(q, k, qw, qw, cos, sin, 1e-6)
    nb = (q.numel() + k.numel()) * 2
    ms = t(lambda: m.qk_norm_rope_fwd(q, k, qw, qw, cos, sin, 1e-6))
    _report("qk_norm_rope_fwd", {"T": Tq, "hq": 32, "hk": 8, "D": 128}, ms, bytes_=2 * nb)
    ms = t(lambda: m.qk_norm_rope_bwd(qo, ko, q, k, qw, qw, cos, sin, rq, rk))
    _report("qk_norm_rope_bwd", {"T": Tq, "hq": 32, "hk": 8, "D": 128}, ms, bytes_=3 * nb)
    n = 50_000_000 if not small else 20_000_000
    master = torch.randn(n, device="cuda")
    param = master.to(torch.bfloat16)
    grad = torch.randn(n, device="cuda")
    mm_, vv = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    clip = torch.ones(1, device="cuda")
    ms = t(lambda: m.adamw_step(master, param, grad, mm_, vv, clip, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0, 1.0))
    _report("adamw_step", {"n": n}, ms, bytes_=n * (4 * 4 + 3 * 4 + 2))


def bench_logprob(t: Timer, small: bool):
    from bridge_b200.ops.logprob import fused_lm_head_logprob

    U = 4096 if not small else 2048
    V, H = 151936, 2560
    h = torch.randn(U, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    W = (0.02 * torch.randn(V, H, device="cuda")).to(torch.bfloat16).requires_grad_()
    tg = torch.randint(0, V, (U,), device="cuda")
    temp = torch.ones(U, device="cuda")

    def fb():
        lp, _ = fused_lm_head_logprob(h, W, tg, temp)
        lp.sum().backward()

    ms = t(fb)
    _report("lm_head_logprob_fwd_bwd", {"U": U, "V": V, "H": H}, ms, flops=3 * 2.0 * U * V * H)


def bench_ppo(t: Timer, small: bool):
    from bridge_b200.ops._ext import kernels

    n = 4096 * 64
    x = torch.randn(n, device="cuda") - 3
    old = x + 0.01 * torch.randn(n, device="cuda")
    adv = torch.randn(n, device="cuda")
    ms = t(lambda: kernels().ppo_loss_fwd(x, old, adv, None, float(n), 0.8, 1.2, 3.0))
    _report("ppo_loss_fwd", {"n": n}, ms, bytes_=n * 4 * 4)


def bench_gdn(t: Timer, small: bool):
    from bridge_b200.ops._ext import kernels

    m = kernels()
    lens = [512] * (9 if not small else 4)
    cu_l = [0]
    for n in lens:
        cu_l.append(cu_l[-1] + n)
    cu = torch.tensor(cu_l, dtype=torch.int32, device="cuda")
    T, C, W = cu_l[-1], 8192, 4
    x = torch.randn(T, C, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(C, W, device="cuda", dtype=torch.bfloat16)
    h0 = torch.randn(len(lens), C, W, device="cuda", dtype=torch.bfloat16)
    ms = t(lambda: m.causal_conv1d_fwd(x, w, None, h0, cu, 512, True))
    _report("causal_conv1d_fwd", {"T": T, "C": C, "W": W}, ms, bytes_=2 * x.numel() * 2)
    dy = torch.randn_like(x)
    ms = t(lambda: m.causal_conv1d_bwd(dy, x, w, None, h0, None, cu, 512, True))
    _report("causal_conv1d_bwd", {"T": T, "C": C, "W": W}, ms, bytes_=3 * x.numel() * 2)
    H, K, V = 32, 128, 128
    q = torch.nn.functional.normalize(torch.randn(T, H, K, device="cuda"), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(T, H, K, device="cuda"), dim=-1).to(torch.bfloat16)
    v = torch.randn(T, H, V, device="cuda", dtype=torch.bfloat16)
    g = -torch.rand(T, H, device="cuda") * 0.1
    beta = torch.rand(T, H, device="cuda")
    s0 = torch.zeros(len(lens), H, K, V, device="cuda")
    from bridge_b200.ops.gdn import _chunk_table

    chunks, seq0, most = _chunk_table(tuple(cu_l), torch.device("cuda"))
    # chunk math: A, P (n^2 K), W/U/O/S1 (n K V-ish) per 64-token chunk and head
    fl = 2.0 * T * H * (2 * 64 * K + 64 * V + 3 * K * V)
    ms = t(lambda: m.gdr_fwd(q, k, v, g, beta, s0, chunks, seq0, most, K ** -0.5))
    _report("gated_delta_rule_fwd", {"T": T, "H": H, "K": K, "V": V}, ms, flops=fl)
    o, hT, ck, wk, u = m.gdr_fwd(q, k, v, g, beta, s0, chunks, seq0, most, K ** -0.5)
    do = torch.randn_like(o)
    ms = t(lambda: m.gdr_bwd(do, None, q, k, v, g, beta, ck, wk, u, chunks, seq0, most, True, K ** -0.5))
    _report("gated_delta_rule_bwd", {"T": T, "H": H, "K": K, "V": V}, ms, flops=3 * fl)
    # where the cycles of each kernel go: one timed-off fwd + bwd with the in-kernel phase clocks on
    m.gdr_phase_profile(True)
    m.gdr_fwd(q, k, v, g, beta, s0, chunks, seq0, most, K ** -0.5)
    m.gdr_bwd(do, None, q, k, v, g, beta, ck, wk, u, chunks, seq0, most, True, K ** -0.5)
    torch.cuda.synchronize()
    tab = m.gdr_phase_read()
    m.gdr_phase_profile(False)
    sub = {12: "T:KK^T", 13: "T:diag", 14: "T:levels", 15: "T:bf16"}   # inside build_T (prep, bwd chunk)
    names = {0: ("prep", ["load", "build_T", "Wk/Wv"]),
             1: ("scan", ["ckpt+load", "P,U", "O", "S1"]),
             2: ("bwd_scan", ["ckpt+load", "P", "dU", "dq", "dk", "dwk", "dG", "dS0", "dG tail"]),
             3: ("bwd_chunk", ["load", "build_T", "P", "dP", "dq/dk", "dT", "dv/dk", "X2", "dL", "dk", "tail"])}
    for kid, (kname, phases) in names.items():
        row = [int(x) for x in tab[kid].tolist()]
        tot = sum(row) or 1
        share = {p: round(row[i] / tot, 3) for i, p in enumerate(phases)}
        share.update({v: round(row[k] / tot, 3) for k, v in sub.items() if row[k]})
        print(json.dumps({"op": f"gdr_phases_{kname}", "block_cycles": tot, "share": share}))


def bench_moe(t: Timer, small: bool):
    """Device MoE routing (top-k + stable expert sort), combine and its backward at the config #5 shape
    (512 experts, top-10, hidden 2048; 16384 tokens per rank, 4096 with --small)."""
    from bridge_b200.ops._ext import kernels

    m = kernels()
    T, E, k, H = (4096 if small else 16384), 512, 10, 2048
    logits = torch.randn(T, E, device="cuda")
    idx, w, counts, offsets, pos, order = m.moe_route(logits, k)
    ms = t(lambda: m.moe_route(logits, k))
    _report("moe_route", {"T": T, "E": E, "k": k}, ms, bytes_=T * E * 4 + T * k * 16)
    ys = torch.randn(T * k, H, device="cuda", dtype=torch.bfloat16)
    wf = w.reshape(-1).contiguous()
    ms = t(lambda: m.moe_combine(ys, pos, wf, T))
    _report("moe_combine", {"T": T, "k": k, "H": H}, ms, bytes_=(T * k + T) * H * 2)
    dy = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    ms = t(lambda: m.moe_combine_bwd(dy, ys, pos, wf))
    _report("moe_combine_bwd", {"T": T, "k": k, "H": H}, ms, bytes_=(2 * T * k + T) * H * 2)


OPS = {"gemm": bench_gemm, "attention": bench_attention, "elementwise": bench_elementwise,
       "logprob": bench_logprob, "ppo": bench_ppo, "gdn": bench_gdn, "moe": bench_moe}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--op", default="all", choices=["all", *OPS])
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--small", action="store_true")
    a = p.parse_args(argv)
    t = Timer(a.warmup, a.iters)
    for name, fn in OPS.items():
        if a.op in ("all", name):
            fn(t, a.small)


if __name__ == "__main__":
    main()

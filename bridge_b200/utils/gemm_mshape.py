"""BF16 GEMM sensitivity to the physical M (row count) of the call.

TPR computes a prefix's rows in a different physical batch than the flattened path does, so the
same logical row can go through GEMMs of different M.  This tool multiplies identical operands once
as one ``[M, K] x [N, K]^T`` call and once split into row blocks, and reports how far the two results
differ (relative L2, max abs) for the framework's GEMM (tcgen05 on CUDA) and for torch.matmul.

    python -m bridge_b200.utils.gemm_mshape --m 192 --k 2048 --n 4096 --split 64

Parity: tools/tpr_gemm_mshape_repro.py of the reference (X = [192, 2048], W = [4096, 2048]).
"""

from __future__ import annotations

import argparse
import json

import torch


def mshape_drift(m: int = 192, k: int = 2048, n: int = 4096, split: int = 64, *, device=None, seed: int = 0) -> dict:
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(device, torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(device, torch.bfloat16)
    out = {"m": m, "k": k, "n": n, "split": split, "device": str(device)}
    impls = {"torch": lambda a: torch.matmul(a, w.t())}
    if str(device).startswith("cuda"):
        from ..ops.gemm import gemm

        impls["bridge_b200"] = lambda a: gemm(a.contiguous(), w)
    for name, fn in impls.items():
        full = fn(x).float()
        parts = torch.cat([fn(x[i:i + split]).float() for i in range(0, m, split)])
        diff = full - parts
        out[name] = {"rel_l2": float(diff.norm() / full.norm().clamp_min(1e-30)),
                     "max_abs": float(diff.abs().max()), "bitwise_equal": bool(torch.equal(full, parts))}
    return out


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, default=192)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--split", type=int, default=64)
    a = p.parse_args(argv)
    print(json.dumps(mshape_drift(a.m, a.k, a.n, a.split)))


if __name__ == "__main__":
    main()

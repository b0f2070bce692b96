"""Compare per-token log-probs of two runs (e.g. context-parallel vs single-rank, TPR vs flattened).

Inputs are ``torch.save`` files holding either a 1-D tensor of response-token log-probs or a dict with
``"log_probs"`` (a tensor, or a list of per-row tensors concatenated in order) and optionally
``"response_mask"``.  Reports relative L2, cosine, max abs difference and the NLL of each run.

    python -m bridge_b200.utils.cp_drift cp1.pt cp2.pt [cp4.pt ...]

Parity: tools/compare_native_cp_drift.py of the reference (response log-prob rel-L2 / NLL per CP size).
"""

from __future__ import annotations

import argparse
import json

import torch


def _flat(obj) -> torch.Tensor:
    if isinstance(obj, torch.Tensor):
        return obj.detach().float().flatten()
    lp = obj["log_probs"]
    if isinstance(lp, (list, tuple)):
        masks = obj.get("response_mask")
        if masks is not None:
            lp = [r[m.bool()] if r.numel() == m.numel() else r for r, m in zip(lp, masks)]
        lp = torch.cat([torch.as_tensor(r).float().flatten() for r in lp])
    return torch.as_tensor(lp).detach().float().flatten()


def drift(reference: torch.Tensor, other: torch.Tensor) -> dict:
    if reference.numel() != other.numel():
        raise ValueError(f"token counts differ: {reference.numel()} vs {other.numel()}")
    d = other - reference
    return {"rel_l2": float(d.norm() / reference.norm().clamp_min(1e-30)),
            "cosine": float(torch.nn.functional.cosine_similarity(reference, other, dim=0)),
            "max_abs": float(d.abs().max()) if d.numel() else 0.0,
            "nll_reference": float(-reference.mean()), "nll_other": float(-other.mean())}


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("reference")
    p.add_argument("others", nargs="+")
    a = p.parse_args(argv)
    ref = _flat(torch.load(a.reference, map_location="cpu", weights_only=False))
    for path in a.others:
        out = drift(ref, _flat(torch.load(path, map_location="cpu", weights_only=False)))
        print(json.dumps({"reference": a.reference, "other": path, **out}))


if __name__ == "__main__":
    main()

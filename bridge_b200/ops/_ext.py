"""Loader for the in-tree sm_100a extension ``bridge_b200._C``.

Ops run their CUDA kernels whenever their inputs live on a CUDA device.  The
PyTorch formulation is used for CPU tensors (gloo tests, oracles) and, on the
GPU, only when ``BRIDGE_B200_IMPL=reference`` asks for the library baseline
explicitly.  A GPU run without the built extension fails loudly instead of
falling back silently.
"""

from __future__ import annotations

import os

import torch

_EXT = None
_TRIED = False


def ext():
    global _EXT, _TRIED
    if not _TRIED:
        _TRIED = True
        try:
            from .. import _C  # type: ignore[attr-defined]

            _EXT = _C
        except ImportError as exc:  # pragma: no cover - depends on the build
            _EXT = None
            if torch.cuda.is_available() and os.environ.get("BRIDGE_B200_IMPL", "fused") != "reference":
                raise RuntimeError(
                    "bridge_b200._C (sm_100a kernels) is not built; run `python setup.py build_ext --inplace`"
                ) from exc
    return _EXT


def reference_forced() -> bool:
    return os.environ.get("BRIDGE_B200_IMPL", "fused") == "reference"


def on_gpu(*tensors) -> bool:
    """True when the CUDA kernels must run (tensors on CUDA and not forced to the baseline)."""
    if reference_forced():
        return False
    for t in tensors:
        if t is not None and isinstance(t, torch.Tensor):
            return t.is_cuda
    return False


def kernels():
    m = ext()
    if m is None:
        raise RuntimeError("bridge_b200._C is required for CUDA tensors but is not built")
    return m

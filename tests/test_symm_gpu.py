"""Symmetric peer memory and the fused NVLink data-parallel optimizer path."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_barrier_wait_runs_out_and_reports():
    """A barrier whose peer never signals (a pad nobody writes) returns after its limit with an error code;
    the context stays usable."""
    from bridge_b200.ops._ext import kernels

    m = kernels()
    m.symm_clear_error()
    a, _ = m.symm_alloc(m.symm_pad_bytes())
    b, _ = m.symm_alloc(m.symm_pad_bytes())
    a.zero_()
    b.zero_()
    m.symm_barrier([a.data_ptr(), b.data_ptr()], 0, 1, None, 0.3)
    torch.cuda.synchronize()
    assert m.symm_error_code() == 0x101          # waited for "peer" 1
    m.symm_clear_error()
    x = torch.ones(1000, device="cuda")
    assert float(x.sum()) == 1000.0              # context still healthy
    # a satisfied barrier (single rank) leaves no error
    m.symm_barrier([a.data_ptr()], 0, 2, None, 0.3)
    torch.cuda.synchronize()
    assert m.symm_error_code() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_worker(name: str, token: str, nproc: int = 2) -> None:
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "mgpu_worker.py"), name]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env=env, timeout=700)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert token in out.stdout


@pytest.mark.multigpu
def test_nvlink_dp_matches_nccl_two_gpus():
    _run_worker("dp_nvlink", "DP_NVLINK_OK")


@pytest.mark.multigpu
def test_tp_fused_linears_match_nccl_two_gpus():
    _run_worker("tp_fused", "TP_FUSED_OK")


@pytest.mark.multigpu
def test_cp_p2p_attention_matches_flattened_two_gpus():
    _run_worker("cp_p2p", "CP_P2P_OK")


@pytest.mark.multigpu
def test_ep_p2p_moe_matches_unsharded_two_gpus():
    _run_worker("ep_p2p", "EP_P2P_OK")

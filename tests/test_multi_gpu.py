"""Fused GEMV + all-gather on 2 GPUs (skipped with fewer than 2 GPUs).

Runs tests/multi_gpu_worker.py under torchrun as child processes with a hard
time limit; every rank checks its gathered output against the CPU oracle,
through the two-launch gathering call and through the single-launch one.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("path,ncols", [("two", 1), ("two", 2), ("single", 1), ("single", 2)])
def test_fused_allgather_two_ranks(path, ncols):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, Q4K_NCOLS=str(ncols), Q4K_PATH=path, NCCL_NVLS_ENABLE="0")
    port = 29600 + ncols + (10 if path == "single" else 0)
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(ROOT / "tests" / "multi_gpu_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    errs = [ln for ln in (r.stdout + r.stderr).splitlines() if "Error" in ln or "rank" in ln.lower()]
    assert r.returncode == 0, "\n".join(errs[:40]) + "\n...\n" + r.stderr[-2000:]
    assert '"multi_gpu_allgather": "ok"' in r.stdout

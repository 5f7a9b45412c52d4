"""q4k_gemv_sharded: the row-sharded GEMV gathered with NCCL over the caller's
communicator (the reference's row split, kernels/mmvq.cu:764-793, with the
slices brought together on the device).

One GPU: a one-rank communicator made here through the process's own NCCL
(the library must use the same instance), checked against the CPU oracle at
ncols 1, 2 and 8 and on a row count that is not a multiple of 32; a call
whose world / rank disagree with the communicator is refused with Q4K_EINVAL.
Two GPUs: two ranks under torchrun (tests/nccl_shard_worker.py) on ragged
row splits, each rank's gathered rows against the oracle.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
TOL_ABS, TOL_REL = 1e-4, 1e-5
EINVAL = 1


class NcclUniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]


def process_nccl():
    """The NCCL library torch loaded into this process."""
    import torch  # noqa: F401  (libtorch_cuda needs libnccl.so.2)
    L = ctypes.CDLL("libnccl.so.2", mode=os.RTLD_NOLOAD | os.RTLD_NOW)
    L.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, NcclUniqueId, ctypes.c_int]
    L.ncclGetUniqueId.argtypes = [ctypes.POINTER(NcclUniqueId)]
    L.ncclCommDestroy.argtypes = [ctypes.c_void_p]
    return L


def one_rank_comm(L):
    uid = NcclUniqueId()
    assert L.ncclGetUniqueId(ctypes.byref(uid)) == 0
    comm = ctypes.c_void_p()
    assert L.ncclCommInitRank(ctypes.byref(comm), 1, uid, 0) == 0
    return comm


def test_sharded_one_rank_matches_oracle(q4k, oracle):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N = process_nccl()
    comm = one_rank_comm(N)
    try:
        rng = np.random.default_rng(31)
        for nrows, K, ncols in [(1000, 4096, 1), (4096, 4096, 2), (333, 2048, 8)]:
            W = torch.from_numpy(q4k.gen_q4k_numpy(rng, nrows, K)).to(dev)
            x = torch.from_numpy(rng.standard_normal((ncols, K)).astype(np.float32)).to(dev)
            for call in range(2):  # the second call reuses the workspace the first left behind
                got = q4k.gemv_sharded(W, x, nrows, comm.value, 0, 1)
                torch.cuda.synchronize()
                want = oracle.gemv_f32(W.cpu().numpy(), x.cpu().numpy()).astype(np.float64)
                g = got.cpu().numpy().astype(np.float64)
                assert np.all(np.abs(g - want) <= TOL_ABS + TOL_REL * np.abs(want)), (nrows, K, ncols, call)
        # a call that disagrees with the communicator is refused before any launch
        L = q4k.lib()
        ws = q4k.Workspace(q4k.sharded_workspace_bytes(64, 256, 1, 2), dev)
        st = L.q4k_gemv_sharded(W.data_ptr(), x.data_ptr(), got.data_ptr(), 256, 64, 1, 1, 256, 64, comm.value,
                                0, 2, ws.ptr, ws.nbytes, torch.cuda.current_stream().cuda_stream)
        assert st == EINVAL and b"communicator has 1 ranks" in L.q4k_last_error()
    finally:
        torch.cuda.synchronize()
        N.ncclCommDestroy(comm)


def test_sharded_two_ranks():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29561", str(ROOT / "tests" / "nccl_shard_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "240"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("nccl shard ok") == 2, r.stdout[-2000:]

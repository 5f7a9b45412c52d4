"""One rank of the q4k_gemv_sharded check (run under torchrun, >= 2 GPUs).

The ranks make one NCCL communicator through the process's own NCCL (the
unique id travels over a gloo process group), generate the same full
matrices (same seed), each pass only its ceil-split rows to
q4k_gemv_sharded, and check the gathered (ncols, nrows) output against the
CPU oracle's GEMV of the full matrix (1e-4 absolute + 1e-5 relative), on row
counts that leave the last rank short, for two calls in a row.  Prints
"nccl shard ok" and exits 0 on success.  Used by tests/test_gpu_sharded_nccl.py.
"""
from __future__ import annotations

import ctypes
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent))
from conftest import load_package  # noqa: E402
import oracle as O  # noqa: E402  (tests/conftest.py puts oracle/ on the path; the checker only)
from test_gpu_sharded_nccl import NcclUniqueId, process_nccl  # noqa: E402

TOL_ABS, TOL_REL = 1e-4, 1e-5


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))  # the unique id only
    q4k = load_package()
    N = process_nccl()
    uid = NcclUniqueId()
    if rank == 0:
        assert N.ncclGetUniqueId(ctypes.byref(uid)) == 0
    # the raw 128 bytes (the c_char array's value would stop at the first zero byte)
    box = [ctypes.string_at(ctypes.addressof(uid), 128) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    if rank != 0:
        ctypes.memmove(ctypes.addressof(uid), box[0], 128)
    comm = ctypes.c_void_p()
    rc = N.ncclCommInitRank(ctypes.byref(comm), world, uid, rank)
    assert rc == 0, f"ncclCommInitRank: {rc}"
    try:
        rng = np.random.default_rng(1234)  # identical on every rank
        for nrows, K, ncols in [(1001, 4096, 1), (4099, 4096, 2), (77, 2048, 8)]:
            W = q4k.gen_q4k_numpy(rng, nrows, K)
            x = rng.standard_normal((ncols, K)).astype(np.float32)
            want = O.gemv_f32(W, x).astype(np.float64)
            lo, hi, _ = q4k.shard_rows(nrows, rank, world)
            Ws = torch.from_numpy(W[lo:hi]).to(dev)
            xd = torch.from_numpy(x).to(dev)
            for call in range(2):
                got = q4k.gemv_sharded(Ws, xd, nrows, comm.value, rank, world)
                torch.cuda.synchronize()
                g = got.cpu().numpy().astype(np.float64)
                bad = np.abs(g - want) > TOL_ABS + TOL_REL * np.abs(want)
                if bad.any():
                    raise AssertionError(f"rank {rank} {nrows}x{K} ncols {ncols} call {call}: {int(bad.sum())} off")
        print(f"nccl shard ok rank {rank}", flush=True)
    finally:
        torch.cuda.synchronize()
        N.ncclCommDestroy(comm)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

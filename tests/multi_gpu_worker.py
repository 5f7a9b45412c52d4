"""One rank of the fused GEMV + all-gather check (run under torchrun, >= 2 GPUs).

Every rank generates the same full matrices (same seed), computes its
contiguous row shard with q4k_gemv_batch_allgather, waits for its peers'
rows (q4k_gather_wait), and then checks that its own full output buffer --
filled by all ranks' kernels over NVLink -- matches the CPU oracle's GEMV of
the full matrices (1e-4 absolute + 1e-5 relative), for several consecutive
calls and for replays of a captured CUDA graph (the epoch handshake keeps
counting).  Exit status 0 on success.  Used by tests/test_multi_gpu.py.
"""
from __future__ import annotations

import json
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

TOL_ABS, TOL_REL = 1e-4, 1e-5


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))  # host-side handle exchange only
    q4k = load_package()
    ncols = int(os.environ.get("Q4K_NCOLS", "2"))
    shapes = [(1000, 4096), (257, 4096), (4096, 14336), (7, 512)]
    g = torch.Generator(device=dev)
    g.manual_seed(77)  # identical on every rank
    fullW = [q4k.gen_q4k_torch(r, K, generator=g, device=dev) for r, K in shapes]
    xs = [torch.randn((ncols, K), device=dev, generator=g) for _, K in shapes]
    ref = [torch.from_numpy(O.gemv_f32(W.cpu().numpy(), x.cpu().numpy())).to(dev) for W, x in zip(fullW, xs)]

    # full-output layout (same on every rank): matrix t at off[t], column stride = rows
    off, tot = [], 0
    for r, _ in shapes:
        off.append(tot)
        tot += r * ncols
    pg = q4k.PeerGather(tot)
    shards, outs = [], []
    for (r, K), W, o in zip(shapes, fullW, off):
        lo, hi, _ = q4k.shard_rows(r, rank, world)
        shards.append(W[lo:hi])
        outs.append(pg.out[o:o + r * ncols].view(ncols, r)[:, lo:hi])
    tasks = q4k.make_tasks(shards, xs, outs)
    for i, (r, _) in enumerate(shapes):
        tasks[i].stride_col_dst = r
    ws = q4k.Workspace(q4k.batch_workspace_bytes(tasks, ncols))
    s = torch.cuda.Stream()

    def check(tag):
        for (r, _), o, want in zip(shapes, off, ref):
            got = pg.out[o:o + r * ncols].view(ncols, r)
            err = (got - want).abs()
            tol = TOL_ABS + TOL_REL * want.abs()
            if not bool((err <= tol).all()):
                raise AssertionError(f"rank {rank} {tag}: {int((err > tol).sum())} values off, max err {float(err.max())}")

    with torch.cuda.stream(s):
        for it in range(3):
            # A rank may store into a peer's buffer as soon as its own launch
            # starts: every rank's fill must be complete before anyone launches.
            pg.out.fill_(float("nan"))
            s.synchronize()
            dist.barrier()
            q4k.gemv_batch_allgather(tasks, ncols, pg, ws, stream=s)
            q4k.gather_wait(pg, ws, stream=s)
            s.synchronize()
            dist.barrier()
            assert ws.status(s) == 0
            check(f"call {it}")
            dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            q4k.gemv_batch_allgather(tasks, ncols, pg, ws, stream=s)
            q4k.gather_wait(pg, ws, stream=s)
        for it in range(3):
            dist.barrier()
            pg.out.fill_(float("nan"))
            s.synchronize()
            dist.barrier()
            graph.replay()
            s.synchronize()
            dist.barrier()
            assert ws.status(s) == 0
            check(f"graph replay {it}")
    del graph
    dist.barrier()
    pg.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"multi_gpu_allgather": "ok", "world": world, "ncols": ncols}))


if __name__ == "__main__":
    main()

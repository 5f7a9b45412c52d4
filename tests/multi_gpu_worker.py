"""One rank of the fused GEMV + all-gather check (run under torchrun, >= 2 GPUs).

Every rank generates the same full matrices (same seed), computes its
contiguous row shard with q4k_gemv_batch_allgather (Q4K_PATH=single:
q4k_gemv_batch_persistent with the gather), waits for its peers'
rows (q4k_gather_wait), and then checks that its own full output buffer --
filled by all ranks' kernels over NVLink -- matches the CPU oracle's GEMV of
the full matrices (1e-4 absolute + 1e-5 relative), for several consecutive
calls and for replays of a captured CUDA graph (the epoch handshake keeps
counting), and then for a chain of six large single-matrix launches into
fresh gather buffers, three times over.  Exit status 0 on success.  Used by tests/test_multi_gpu.py.
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
    single = os.environ.get("Q4K_PATH", "two") == "single"  # q4k_gemv_batch_persistent
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
    if single:
        ws.init(s)
        assert q4k.batch_persistent_kernel(tasks, ncols) == "k_gemv (single launch)"

    def call():
        if single:
            q4k.gemv_batch_persistent(tasks, ncols, ws, stream=s, gather=pg)
        else:
            q4k.gemv_batch_allgather(tasks, ncols, pg, ws, stream=s)

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
            call()
            q4k.gather_wait(pg, ws, stream=s)
            s.synchronize()
            dist.barrier()
            assert ws.status(s) == 0
            check(f"call {it}")
            dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            call()
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

    # A chain of launches as a decode step runs them (the benchmark's row-split
    # configs): six launches of one large matrix each into six regions of a
    # fresh gather buffer, one wait at the end, sampled rows of every region
    # against the oracle; three rounds, each with its own buffer allocated
    # after the previous one was released (the buffers' addresses get reused).
    rows, K, nl = 20000, 8192, 6
    chainW = [q4k.gen_q4k_torch(rows, K, generator=g, device=dev) for _ in range(nl)]
    chainX = [torch.randn((ncols, K), device=dev, generator=g) for _ in range(nl)]
    rng = np.random.default_rng(5)
    sel = [np.sort(rng.choice(rows, size=256, replace=False)) for _ in range(nl)]
    want = [O.gemv_f32(W[torch.from_numpy(sl).to(dev)].cpu().numpy(), x.cpu().numpy())
            for W, x, sl in zip(chainW, chainX, sel)]
    lo, hi, _ = q4k.shard_rows(rows, rank, world)
    for rnd in range(3):
        pg2 = q4k.PeerGather(nl * rows * ncols)
        launches = []
        for i in range(nl):
            full = pg2.out[i * rows * ncols:(i + 1) * rows * ncols].view(ncols, rows)
            t = q4k.make_tasks([chainW[i][lo:hi]], [chainX[i]], [full[:, lo:hi]])
            t[0].stride_col_dst = rows
            launches.append(t)
        ws2 = q4k.Workspace(q4k.batch_workspace_bytes(launches[0], ncols))
        with torch.cuda.stream(s):
            if single:
                ws2.init(s)
            pg2.out.fill_(float("nan"))
            s.synchronize()
            dist.barrier()
            for t in launches:
                if single:
                    q4k.gemv_batch_persistent(t, ncols, ws2, stream=s, gather=pg2)
                else:
                    q4k.gemv_batch_allgather(t, ncols, pg2, ws2, stream=s)
            q4k.gather_wait(pg2, ws2, stream=s)
            s.synchronize()
        dist.barrier()
        assert ws2.status(s) == 0
        for i in range(nl):
            full = pg2.out[i * rows * ncols:(i + 1) * rows * ncols].view(ncols, rows)
            got = full[:, torch.from_numpy(sel[i]).to(dev)].cpu().numpy().astype(np.float64)
            w = want[i].astype(np.float64)
            bad = np.abs(got - w) > TOL_ABS + TOL_REL * np.abs(w)
            if bad.any():
                rr = sel[i][np.nonzero(bad)[1]]
                raise AssertionError(f"rank {rank} chain round {rnd} launch {i}: {int(bad.sum())} values off "
                                     f"(rows {rr[:8].tolist()}, owners {[int(r >= hi) for r in rr[:8]]})")
        dist.barrier()
        pg2.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"multi_gpu_allgather": "ok", "world": world, "ncols": ncols,
                          "path": "single" if single else "two"}))


if __name__ == "__main__":
    main()

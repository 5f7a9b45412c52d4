"""Host logic of the row-sharded path on CPU, with world_size-2 gloo ranks:
row ranges cover every row exactly once, all ranks agree on the shared
full-output layout, and the C ABI rejects bad gather descriptors before
touching a device."""
from __future__ import annotations

import ctypes
import os
import socket
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT / "tests"))
    from conftest import load_package
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q4k = load_package()
    shapes = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (32000, 4096), (7, 256), (1, 256), (5, 512)]
    mine = [q4k.shard_rows(r, rank, world) for r, _ in shapes]
    allv = [None] * world
    dist.all_gather_object(allv, mine)
    ok = True
    for t, (r, _) in enumerate(shapes):
        rows = []
        for rk in range(world):
            lo, hi, per = allv[rk][t]
            ok &= 0 <= lo <= hi <= r and hi - lo <= per
            rows.extend(range(lo, hi))
        ok &= sorted(rows) == list(range(r))
    dist.destroy_process_group()
    q.put((rank, ok))


@pytest.mark.parametrize("world", [2, 3])
def test_shards_cover_rows_exactly_once(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in res)


def test_bad_gather_descriptors_rejected(q4k):
    L = q4k.lib()
    tasks = (q4k.Task * 1)()
    tasks[0].W, tasks[0].x, tasks[0].dst = 256, 512, 1024
    tasks[0].nrows, tasks[0].K, tasks[0].stride_row_x, tasks[0].stride_col_x, tasks[0].stride_col_dst = 32, 256, 1, 256, 32

    def call(g):
        return L.q4k_gemv_batch_allgather(tasks, 1, 1, ctypes.byref(g) if g is not None else None, 4096, 1 << 20, None)

    assert call(None) == 1
    g = q4k.Gather()
    g.world, g.rank = 9, 0
    assert call(g) == 1
    g.world, g.rank = 2, 2
    assert call(g) == 1
    g.world, g.rank = 2, 0
    g.out_local, g.epoch = 1024, 2048
    g.out_peer[0], g.out_peer[1] = 1024, 4096
    g.flags_peer[0] = 8192
    assert call(g) == 1  # flags_peer[1] missing
    g.flags_peer[1] = 8448
    g.out_peer[0] = 4096
    assert call(g) == 1  # out_peer[rank] != out_local
    assert b"gather" in L.q4k_last_error()


def test_gather_tasks_outside_the_buffer_rejected(q4k):
    """Every output of a gathering call is also stored into each peer's buffer at
    the same offset, so a task whose columns reach past the full buffer (or
    start outside it) is refused on the host, before any launch."""
    L = q4k.lib()
    g = q4k.Gather()
    g.world, g.rank = 2, 0
    g.out_local, g.epoch = 1 << 20, 2048
    g.out_peer[0], g.out_peer[1] = 1 << 20, 1 << 24
    g.flags_peer[0], g.flags_peer[1] = 8192, 8448
    g.out_elems = 1000
    tasks = (q4k.Task * 1)()
    t = tasks[0]
    t.W, t.x = 256, 512
    t.nrows, t.K, t.stride_row_x, t.stride_col_x = 32, 256, 1, 256

    def call(dst, stride_col_dst, ncols):
        # no workspace: a call that passes validation stops at Q4K_EWORKSPACE,
        # before any launch (the pointers here are not device memory)
        t.dst, t.stride_col_dst = dst, stride_col_dst
        return L.q4k_gemv_batch_allgather(tasks, 1, ncols, ctypes.byref(g), None, 0, None)

    base = 1 << 20
    assert call(base - 4, 32, 1) == 1                   # starts before out_local
    assert b"gather buffer" in L.q4k_last_error()
    assert call(base + 2, 32, 1) == 1                   # not float-aligned inside it
    assert call(base + 4 * 969, 32, 1) == 1             # rows [969, 1001) reach past 1000
    assert b"reach past" in L.q4k_last_error()
    assert call(base + 4 * 500, 500, 2) == 1            # second column ends at 1032
    assert call(base + 4 * 400, 16, 2) == 1             # stride_col_dst < nrows
    # in range ([468, 1000)): accepted, then refused for the missing workspace
    # (or, without a GPU, for the device set-up) -- anything but Q4K_EINVAL
    st = call(base + 4 * 468, 500, 2)
    assert st in (2, 5), (st, L.q4k_last_error())

"""Single-launch path (q4k_gemv_batch_persistent): quantization inside the
GEMV grid behind a grid-wide barrier.

Its outputs must equal the two-launch path's bit for bit (same quantizer, same
summation order) and the oracle within the fp32 tolerance; the workspace's
control words must be zero again after every completed call, so calls chain
(back to back, mixed with the two-launch path, inside a CUDA graph).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-4, 1e-5


def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > TOL_ABS + TOL_REL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def dev(q4k, torch_mod):
    assert q4k.lib().q4k_device_supported() == 1
    return torch_mod.device("cuda", 0)


def layer(q4k, torch, dev, seed, shapes, x_of, ncols, on_device=False):
    """Weights, shared activations (x_of[i] = index of task i's activation) and outputs."""
    rng = np.random.default_rng(seed)
    if on_device:
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        Wd = [q4k.gen_q4k_torch(r, K, generator=g, device=dev) for r, K in shapes]
        Ws = None
    else:
        Ws = [q4k.gen_q4k_numpy(rng, r, K) for r, K in shapes]
        Wd = [torch.from_numpy(w).to(dev) for w in Ws]
    xs = {}
    for (r, K), i in zip(shapes, x_of):
        if i not in xs:
            xs[i] = torch.from_numpy(rng.standard_normal((ncols, K)).astype(np.float32)).to(dev)
    xl = [xs[i] for i in x_of]
    return Ws, Wd, xl


def n_rowgroups(shapes, ncols):
    """Row groups of a plain launch: 32 rows, or 64 (two rows per lane) from 3 columns on."""
    g = 64 if ncols >= 3 else 32
    return sum((r + g - 1) // g for r, _ in shapes)


def control_words_zero(ws, n_rowgroups):
    """status and gdone (bytes 0..7) and the row-group counters (from 256);
    the barrier's arrival counter (128) counts up by design."""
    head = ws.buf[:8].cpu().numpy()
    cnt = ws.buf[256:256 + 4 * n_rowgroups].cpu().numpy()
    return not head.any() and not cnt.any()


MISTRAL = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
MISTRAL_X = [0, 0, 0, 1, 2, 2, 3]


@pytest.mark.parametrize("ncols", [1, 2, 3, 5, 8])
def test_persistent_equals_two_launch_path_and_oracle(q4k, oracle, torch_mod, dev, ncols):
    torch = torch_mod
    shapes = [(96, 1024), (32, 1024), (32, 1024), (96, 1024), (200, 1024), (200, 1024), (96, 3584)]
    x_of = [0, 0, 0, 1, 2, 2, 3]
    Ws, Wd, xs = layer(q4k, torch, dev, 100 + ncols, shapes, x_of, ncols)
    a = [torch.empty((ncols, r), device=dev) for r, _ in shapes]
    b = [torch.full((ncols, r), float("nan"), device=dev) for r, _ in shapes]
    ws_a, ws_b = q4k.Workspace(), q4k.Workspace()
    q4k.gemv_batch(q4k.make_tasks(Wd, xs, a), ncols, ws_a)
    q4k.gemv_batch_persistent(q4k.make_tasks(Wd, xs, b), ncols, ws_b)
    for i, (W, x, oa, ob) in enumerate(zip(Ws, xs, a, b)):
        ob_np = ob.cpu().numpy()
        assert np.array_equal(oa.cpu().numpy(), ob_np), f"task {i}: differs from the two-launch path"
        assert_close(ob_np, oracle.gemv_f32(W, x.cpu().numpy()), f"task {i}")
    assert ws_b.status() == 0
    assert control_words_zero(ws_b, n_rowgroups(shapes, ncols))


@pytest.mark.parametrize("ncols", [1, 4])
def test_persistent_full_layer(q4k, oracle, torch_mod, dev, ncols):
    """A whole 7-matrix decoder layer at full size through the single-launch
    path, three times: bit-identical calls, every row at the parity bar.  The
    two-launch path runs this layer on the dynamically scheduled kernel, whose
    per-row sums are split differently (eight warp shares per row group), so
    the two agree to the parity bar, not bit for bit."""
    torch = torch_mod
    _, Wd, xs = layer(q4k, torch, dev, 7, MISTRAL, MISTRAL_X, ncols, on_device=True)
    a = [torch.empty((ncols, r), device=dev) for r, _ in MISTRAL]
    ws_a, ws_b = q4k.Workspace(), q4k.Workspace()
    q4k.gemv_batch(q4k.make_tasks(Wd, xs, a), ncols, ws_a)
    runs = []
    for _ in range(3):
        b = [torch.empty((ncols, r), device=dev) for r, _ in MISTRAL]
        q4k.gemv_batch_persistent(q4k.make_tasks(Wd, xs, b), ncols, ws_b)
        runs.append(b)
    for i in range(len(MISTRAL)):
        assert torch.equal(runs[0][i], runs[1][i]) and torch.equal(runs[0][i], runs[2][i]), f"task {i}"
        want = oracle.gemv_f32(Wd[i].cpu().numpy(), xs[i].cpu().numpy())
        assert_close(runs[0][i].cpu().numpy(), want, f"task {i} single launch")
        assert_close(a[i].cpu().numpy(), want, f"task {i} two launches")
    assert ws_b.status() == 0 and ws_a.status() == 0
    assert control_words_zero(ws_b, n_rowgroups(MISTRAL, ncols))


def test_persistent_small_unpacked_and_empty_tasks(q4k, oracle, torch_mod, dev):
    """Fewer atoms than warps (spread mapping), a K = 0 task and an empty task."""
    torch = torch_mod
    rng = np.random.default_rng(3)
    W1 = q4k.gen_q4k_numpy(rng, 5, 256)
    x1 = rng.standard_normal((2, 256)).astype(np.float32)
    o1 = torch.full((2, 5), float("nan"), device=dev)
    o2 = torch.full((2, 7), 3.0, device=dev)
    W0 = torch.zeros((0, 144), dtype=torch.uint8, device=dev)
    o0 = torch.empty((2, 0), device=dev)
    x1d = torch.from_numpy(x1).to(dev)
    W1d = torch.from_numpy(W1).to(dev)  # held: the tasks keep only its address
    t = q4k.make_tasks([W1d, W0], [x1d, x1d], [o1, o0])
    tk = (q4k.Task * 3)(t[0], t[1], q4k.Task())
    tk[2].W, tk[2].x, tk[2].dst = t[0].W, t[0].x, o2.data_ptr()
    tk[2].nrows, tk[2].K, tk[2].stride_row_x, tk[2].stride_col_x, tk[2].stride_col_dst = 7, 0, 0, 0, 7
    ws = q4k.Workspace()
    q4k.gemv_batch_persistent(tk, 2, ws)
    assert_close(o1.cpu().numpy(), oracle.gemv_f32(W1, x1))
    assert (o2.cpu() == 0).all()
    assert ws.status() == 0


def test_persistent_repeated_and_mixed_with_two_launch_path(q4k, oracle, torch_mod, dev):
    """New inputs every call, both paths on one workspace in alternating order.

    Every call must equal the two-launch path bit for bit.  The oracle bar is
    the stated one (1e-4 abs + 1e-5 rel) for unit-scale inputs; for inputs
    scaled by s the fp32 rounding of the sums scales with them, so the
    absolute part becomes 1e-4 * s."""
    torch = torch_mod
    rng = np.random.default_rng(11)
    shapes = [(160, 2048), (64, 2048), (300, 5120)]
    Ws = [q4k.gen_q4k_numpy(rng, r, K) for r, K in shapes]
    Wd = [torch.from_numpy(w).to(dev) for w in Ws]
    ncols = 2
    ws = q4k.Workspace()
    for it in range(12):
        s = 10.0 ** (it % 3 - 1)
        xs_np = [(rng.standard_normal((ncols, K)) * s).astype(np.float32) for _, K in shapes]
        xs = [torch.from_numpy(x).to(dev) for x in xs_np]
        a = [torch.empty((ncols, r), device=dev) for r, _ in shapes]
        b = [torch.empty((ncols, r), device=dev) for r, _ in shapes]
        ta, tb = q4k.make_tasks(Wd, xs, a), q4k.make_tasks(Wd, xs, b)
        if it % 2:
            q4k.gemv_batch(ta, ncols, ws)
            q4k.gemv_batch_persistent(tb, ncols, ws)
        else:
            q4k.gemv_batch_persistent(tb, ncols, ws)
            q4k.gemv_batch(ta, ncols, ws)
        for W, x, oa, ob in zip(Ws, xs_np, a, b):
            assert torch.equal(oa, ob), f"call {it}: paths differ"
            got, want = ob.cpu().numpy().astype(np.float64), oracle.gemv_f32(W, x).astype(np.float64)
            bad = np.abs(got - want) > TOL_ABS * max(s, 1.0) + TOL_REL * np.abs(want)
            assert not bad.any(), f"call {it} (scale {s}): {bad.sum()} outside tolerance"
    assert ws.status() == 0


def test_persistent_chain_in_cuda_graph(q4k, torch_mod, dev):
    """Consecutive single-launch calls captured in a graph and replayed, each
    call reading the previous call's output (a chain of dependent launches)."""
    torch = torch_mod
    ncols, n, K = 1, 6, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    Ws = [q4k.gen_q4k_torch(K, K, generator=g, device=dev) for _ in range(n)]
    # d = 5e-5 and dmin = 7.5 d in every super-block: zero-mean weights with a
    # gain near 1, so the values stay finite along the chain
    dd = torch.tensor([5e-5, 7.5 * 5e-5], dtype=torch.float16).view(torch.uint8).to(dev)
    for W in Ws:
        W.view(K, K // 256, 144)[:, :, 0:4] = dd
    bufs = [torch.randn((ncols, K), device=dev, generator=g) for _ in range(n + 1)]
    ws = q4k.Workspace(q4k.batch_workspace_bytes(q4k.make_tasks(Ws[:1], bufs[:1], bufs[1:2]), ncols)).init()
    tasks = [q4k.make_tasks([Ws[i]], [bufs[i]], [bufs[i + 1]]) for i in range(n)]

    def eager():
        for t in tasks:
            q4k.gemv_batch_persistent(t, ncols, ws)

    eager()
    want = bufs[n].clone()
    assert torch.isfinite(want).all()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for t in tasks:
                q4k.gemv_batch_persistent(t, ncols, ws, stream=stream)
    torch.cuda.current_stream().wait_stream(stream)
    for _ in range(4):
        bufs[n].zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(bufs[n], want)
    assert ws.status() == 0
    del graph

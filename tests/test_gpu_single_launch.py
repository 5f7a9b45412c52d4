"""The single-launch GEMV (q4k_gemv_batch_persistent, kernel k_gemv in its
single-launch mode): every CTA quantizes the activations its rows need into
shared memory, with a fast quotient (x times an approximate reciprocal of d,
the IEEE division only for values near a rounding tie), then runs the plain
kernel's partition and arithmetic.

Checked here: which launches take the mode (CPU, no device); that its
outputs equal the two-launch path's statically partitioned kernel bit for
bit -- so its q8_1 quants equal the exact quantizer's, ties, near-ties,
zeros, saturation and subnormal scales included -- and the CPU oracle within
1e-4 absolute + 1e-5 relative, at full decoder-layer sizes, for thin and
spread launches, and for batches with many distinct activations.
"""
from __future__ import annotations

import numpy as np
import pytest

TOL_ABS, TOL_REL = 1e-4, 1e-5

MISTRAL = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
MISTRAL_X = [0, 0, 0, 1, 2, 2, 3]
LLAMA70 = [(8192, 8192), (1024, 8192), (1024, 8192), (8192, 8192), (28672, 8192), (28672, 8192), (8192, 28672)]


def fake_tasks(q4k, specs, ncols, x_offset=0):
    """Task arrays with made-up (never dereferenced) addresses, for the host-side choice."""
    arr = (q4k.Task * len(specs))()
    for i, (r, K, a) in enumerate(specs):
        arr[i].W, arr[i].x, arr[i].dst = 1 << 20, (1 << 24) + a * (1 << 20) + x_offset, 1 << 28
        arr[i].nrows, arr[i].K, arr[i].stride_row_x = r, K, K // 256
        arr[i].stride_col_x, arr[i].stride_col_dst = K, r
    return arr


@pytest.mark.parametrize("specs,ncols,want", [
    ([(r, K, a) for (r, K), a in zip(MISTRAL, MISTRAL_X)], 1, "k_gemv (single launch)"),
    ([(r, K, a) for (r, K), a in zip(MISTRAL, MISTRAL_X)], 2, "k_gemv (single launch)"),
    ([(r, K, a) for (r, K), a in zip(LLAMA70, MISTRAL_X)], 1, "k_gemv (single launch)"),
    # 2 columns of the down (K = 28672) and up activations exceed the 81 KB table
    ([(r, K, a) for (r, K), a in zip(LLAMA70, MISTRAL_X)], 2, "k_gemv"),
    ([(128256, 8192, 0)], 1, "k_gemv (single launch)"),
    ([(4096, 4096, 0)], 2, "k_gemv (single launch)"),
    ([(14336, 4096, 0)], 3, "k_gemv (two rows per lane)"),   # three columns: two launches
    ([(64, 28672, a) for a in range(16)], 2, "k_gemv"),      # 16 activations: too many records
])
def test_single_launch_choice(q4k, specs, ncols, want):
    import os
    if "Q4K_LIB" in os.environ:
        pytest.skip("another build of the library")
    assert q4k.batch_persistent_kernel(fake_tasks(q4k, specs, ncols), ncols, num_sms=148) == want


def test_single_launch_needs_aligned_activation_columns(q4k):
    specs = [(4096, 4096, 0)]
    assert q4k.batch_persistent_kernel(fake_tasks(q4k, specs, 1), 1, num_sms=148) == "k_gemv (single launch)"
    # column starts that are not 32-byte aligned cannot be read in whole L2 sectors
    assert q4k.batch_persistent_kernel(fake_tasks(q4k, specs, 1, x_offset=4), 1, num_sms=148) == "k_gemv"
    assert q4k.batch_persistent_kernel(fake_tasks(q4k, specs, 1, x_offset=16), 1, num_sms=148) == "k_gemv"
    assert q4k.batch_persistent_kernel(fake_tasks(q4k, specs, 1, x_offset=32), 1, num_sms=148) == \
        "k_gemv (single launch)"


# ------------------------------------------------------------------ on the GPU
def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    bad = np.abs(got - want) > TOL_ABS + TOL_REL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"


def run_both(q4k, torch, Wd, xs, ncols, dev):
    """(single-launch outputs, two-launch outputs, two-launch kernel, single-launch kernel)."""
    a = [torch.full((ncols, W.shape[0]), float("nan"), device=dev) for W in Wd]
    b = [torch.full((ncols, W.shape[0]), float("nan"), device=dev) for W in Wd]
    ta, tb = q4k.make_tasks(Wd, xs, a), q4k.make_tasks(Wd, xs, b)
    ws_a, ws_b = q4k.Workspace(), q4k.Workspace()
    q4k.gemv_batch_persistent(ta, ncols, ws_a)
    q4k.gemv_batch(tb, ncols, ws_b)
    assert ws_a.status() == 0 and ws_b.status() == 0
    return a, b, q4k.batch_kernel(tb, ncols), q4k.batch_persistent_kernel(ta, ncols)


@pytest.mark.gpu
@pytest.mark.parametrize("shapes,x_of,ncols", [
    (MISTRAL, MISTRAL_X, 1), (MISTRAL, MISTRAL_X, 2), (LLAMA70, MISTRAL_X, 1),
    ([(4096, 4096)], [0], 1), ([(512, 4096)], [0], 2), ([(37, 256), (300, 1280), (5, 2048)], [0, 1, 0], 2),
])
def test_single_launch_matches_two_launch_and_oracle(q4k, oracle, shapes, x_of, ncols):
    import torch
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(sum(r + K for r, K in shapes) + ncols)
    Wd = [q4k.gen_q4k_torch(r, K, generator=g, device=dev) for r, K in shapes]
    xd = {}
    for (r, K), i in zip(shapes, x_of):
        if i not in xd:
            xd[i] = torch.randn((ncols, K), device=dev, generator=g)
    xs = [xd[i] for i in x_of]
    a, b, k2, k1 = run_both(q4k, torch, Wd, xs, ncols, dev)
    assert k1 == "k_gemv (single launch)"
    rng = np.random.default_rng(0)
    for i, (W, x) in enumerate(zip(Wd, xs)):
        if k2 == "k_gemv":  # same partition and arithmetic: bit for bit
            assert torch.equal(a[i], b[i]), f"task {i}: differs from the two-launch kernel"
        rows = W.shape[0]
        sel = np.sort(rng.choice(rows, size=min(rows, 512), replace=False))
        want = oracle.gemv_f32(W[torch.from_numpy(sel).to(dev)].cpu().numpy(), x.cpu().numpy())
        assert_close(a[i][:, torch.from_numpy(sel).to(dev)].cpu().numpy(), want, f"task {i} vs oracle")


def adversarial_activations(rng, ncols, K):
    """fp32 columns whose q8_1 blocks hit every corner of the quantizer: exact
    .5 ties of x/d, values one ulp either side of a tie, zero blocks, lone
    nonzeros, amax at +-127 d, large and tiny (fp32- and fp16-subnormal scale)
    magnitudes, and plain Gaussian blocks."""
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    nblk = K // 32
    for c in range(ncols):
        for b in range(nblk):
            kind = (b + 3 * c) % 10
            blk = x[c, 32 * b: 32 * b + 32]
            if kind == 0:      # exact ties: d = 0.5 (amax 63.5), x = (k + .5) * d
                k = rng.integers(-127, 127, 32)
                blk[:] = ((k + 0.5) * 0.5).astype(np.float32)
                blk[0] = 63.5
            elif kind == 1:    # a few ulps either side of ties
                d = np.float32(0.013)
                k = rng.integers(-126, 126, 32).astype(np.float32)
                t = (k + np.float32(0.5)) * d
                blk[:] = np.nextafter(t, np.where(rng.random(32) < 0.5, -np.inf, np.inf).astype(np.float32))
                blk[1] = np.float32(127.0) * d
            elif kind == 2:
                blk[:] = 0.0
            elif kind == 3:
                blk[:] = 0.0
                blk[rng.integers(32)] = np.float32(rng.standard_normal())
            elif kind == 4:    # large (the scale d stays below fp16's largest finite value)
                blk *= np.float32(1e5)
            elif kind == 5:    # d in the fp16-subnormal range
                blk *= np.float32(1e-6)
            elif kind == 6:    # d in the fp32-subnormal range
                blk *= np.float32(1e-37)
            elif kind == 7:    # ties at amax: every value +-amax
                blk[:] = np.where(rng.random(32) < 0.5, -1.0, 1.0).astype(np.float32) * np.float32(3.7)
    return x


@pytest.mark.gpu
@pytest.mark.parametrize("ncols", [1, 2])
def test_single_launch_quantizer_corners_bit_exact(q4k, oracle, ncols):
    """The fast quotient must give the exact quantizer's q8_1 quants on every
    corner case: any differing quant would move the output (random nibbles
    and scales), so bit-identical outputs with the two-launch kernel (exact
    division) over many such blocks pin it."""
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(17 + ncols)
    K, rows = 4096, 2048
    W = q4k.gen_q4k_numpy(rng, rows, K)
    x = adversarial_activations(rng, ncols, K)
    Wd, xd = torch.from_numpy(W).to(dev), torch.from_numpy(x).to(dev)
    a, b, k2, k1 = run_both(q4k, torch, [Wd], [xd], ncols, dev)
    assert k1 == "k_gemv (single launch)" and k2 == "k_gemv", (k1, k2)
    assert torch.equal(a[0], b[0])
    want = oracle.gemv_f32(W, x).astype(np.float64)
    got = a[0].cpu().numpy().astype(np.float64)
    # The 1e5-scaled blocks make single terms of ~1e7 that cancel: fp32
    # rounding then scales with the terms, not with the result, so the bar
    # is relative to each output's L1 magnitude sum |w| |q8 value|.
    import gguf
    Wf = gguf.quants.dequantize(W, gguf.GGMLQuantizationType.Q4_K).astype(np.float64)
    blk = oracle.quantize_q8_1(x).reshape(ncols, -1, 36)
    xq = (blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)[:, :, None] *
          blk[:, :, 4:].view(np.int8).astype(np.float64)).reshape(ncols, -1)[:, :K]
    mag = np.abs(xq) @ np.abs(Wf).T
    assert np.all(np.abs(got - want) <= TOL_ABS + TOL_REL * mag)


@pytest.mark.gpu
def test_single_launch_many_activations_and_repeats(q4k, oracle):
    """Ten tasks with ten distinct activations (a CTA's table holds several),
    three calls in a row on one workspace: bit-identical every time and with
    the two-launch kernel."""
    import torch
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    shapes = [(512 + 96 * i, 1024 * (1 + i % 4)) for i in range(10)]
    Wd = [q4k.gen_q4k_torch(r, K, generator=g, device=dev) for r, K in shapes]
    xs = [torch.randn((2, K), device=dev, generator=g) for _, K in shapes]
    outs = []
    ws = q4k.Workspace()
    for _ in range(3):
        o = [torch.empty((2, r), device=dev) for r, _ in shapes]
        t = q4k.make_tasks(Wd, xs, o)
        assert q4k.batch_persistent_kernel(t, 2) == "k_gemv (single launch)"
        q4k.gemv_batch_persistent(t, 2, ws)
        outs.append(o)
    assert ws.status() == 0
    b = [torch.empty((2, r), device=dev) for r, _ in shapes]
    tb = q4k.make_tasks(Wd, xs, b)
    q4k.gemv_batch(tb, 2, q4k.Workspace())
    same_kernel = q4k.batch_kernel(tb, 2) == "k_gemv"
    for i in range(len(shapes)):
        assert torch.equal(outs[0][i], outs[1][i]) and torch.equal(outs[0][i], outs[2][i]), f"task {i}"
        if same_kernel:
            assert torch.equal(outs[0][i], b[i]), f"task {i}"
        assert_close(outs[0][i].cpu().numpy(), oracle.gemv_f32(Wd[i].cpu().numpy(), xs[i].cpu().numpy()),
                     f"task {i}")

"""GPU parity of libq4k_gemv.so against the CPU oracle (and, through the golden
fixtures, against the reference's own dot product).

Bars (north star): q8_1 quantization and per-sub-block integer sums
bit-exact; fp32 outputs within 1e-4 absolute + 1e-5 relative of the oracle.
Every call goes through the C ABI (ctypes); the oracle is only the checker.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL_ABS, TOL_REL = 1e-4, 1e-5


def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    tol = TOL_ABS + TOL_REL * np.abs(want)
    bad = err > tol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance, worst err/tol {np.max(err / tol):.3g}"


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def dev(q4k, torch_mod):
    assert q4k.lib().q4k_device_supported() == 1, "needs a compute capability 10.0 device"
    return torch_mod.device("cuda", 0)


def to_dev(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def gen(q4k, seed, nrows, K, ncols):
    rng = np.random.default_rng(seed)
    W = q4k.gen_q4k_numpy(rng, nrows, K)
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    return W, x


# ------------------------------------------------------------------ q8_1
@pytest.mark.parametrize("K,Kpad,ncols", [(256, 512, 1), (4096, 4096, 3), (100, 512, 2), (14336, 14336, 8),
                                          (32, 32, 1), (28672, 28672, 1)])
def test_quantize_q8_1_bit_exact(q4k, oracle, torch_mod, dev, K, Kpad, ncols):
    rng = np.random.default_rng(K + ncols)
    x = (rng.standard_normal((ncols, K)) * rng.choice([1e-3, 1.0, 300.0], size=(ncols, 1))).astype(np.float32)
    x[0, : min(32, K)] = 0.0
    got = q4k.quantize_row_q8_1(to_dev(torch_mod, x, dev), Kpad=Kpad).cpu().numpy()
    assert np.array_equal(got, oracle.quantize_q8_1(x, Kpad=Kpad))


def test_quantize_known_answers(q4k, oracle, torch_mod, dev):
    z = np.load(GOLDEN / "q8_1_kat.npz")
    got = q4k.quantize_row_q8_1(to_dev(torch_mod, z["x"], dev), Kpad=int(z["Kpad"])).cpu().numpy()
    assert np.array_equal(got, z["yq"])


# ---------------------------------------------------------- integer sums
def test_subblock_sums_match_reference_golden(q4k, torch_mod, dev):
    z = np.load(GOLDEN / "subblock_sums.npz")
    W = z["W"]  # (n, 144): n super-blocks, each paired with its own 8 q8_1 blocks
    n = W.shape[0]
    # lay the n super-blocks out as one row of K = 256n against one q8_1 column
    Wrow = W.reshape(1, n * 144)
    yq = z["yq"].reshape(1, n * 8 * 36)
    S, T = q4k.debug_subblock_sums(to_dev(torch_mod, Wrow, dev), to_dev(torch_mod, yq, dev), 256 * n)
    assert np.array_equal(S.cpu().numpy().reshape(n, 8), z["S"])
    assert np.array_equal(T.cpu().numpy().reshape(n, 8), z["T"])


@pytest.mark.parametrize("nrows,K,ncols", [(1, 256, 1), (7, 512, 3), (33, 4096, 8), (70, 14336, 2)])
def test_subblock_sums_bit_exact(q4k, oracle, torch_mod, dev, nrows, K, ncols):
    W, x = gen(q4k, nrows * 7 + K, nrows, K, ncols)
    yq = oracle.quantize_q8_1(x)
    S, T = q4k.debug_subblock_sums(to_dev(torch_mod, W, dev), to_dev(torch_mod, yq, dev), K)
    S_ref, T_ref = oracle.subblock_sums(W, K, yq)
    assert np.array_equal(S.cpu().numpy(), S_ref)
    assert np.array_equal(T.cpu().numpy(), T_ref[:, 0, :])


# ------------------------------------------------------------------ GEMV
SHAPES = [(1, 256), (7, 512), (33, 4096), (512, 4096), (31, 14336), (64, 768), (300, 2048)]


@pytest.mark.parametrize("nrows,K", SHAPES)
@pytest.mark.parametrize("ncols", [1, 2, 3, 4, 5, 8])
def test_gemv_q8_1_vs_oracle(q4k, oracle, torch_mod, dev, nrows, K, ncols):
    W, x = gen(q4k, nrows + 13 * K + ncols, nrows, K, ncols)
    yq = oracle.quantize_q8_1(x)
    got = q4k.mul_mat_vec_q8_1(to_dev(torch_mod, W, dev), to_dev(torch_mod, yq, dev), K).cpu().numpy()
    assert_close(got, oracle.gemv_q8_1(W, K, yq), f"{nrows}x{K} ncols={ncols}")


@pytest.mark.parametrize("nrows,K,ncols", [(1, 256, 1), (33, 4096, 2), (100, 14336, 8), (9, 28672, 3),
                                           (4096, 4096, 1), (257, 8192, 6), (40, 1280, 7)])
def test_gemv_f32_fused_vs_oracle(q4k, oracle, torch_mod, dev, nrows, K, ncols):
    W, x = gen(q4k, 3 * nrows + K + ncols, nrows, K, ncols)
    got = q4k.mul_mat_vec_q(to_dev(torch_mod, W, dev), to_dev(torch_mod, x, dev)).cpu().numpy()
    assert_close(got, oracle.gemv_f32(W, x), f"{nrows}x{K} ncols={ncols}")


@pytest.mark.parametrize("path", sorted(p for p in GOLDEN.glob("gemv_*.npz") if not p.stem.startswith("gemv_q6k_")),
                         ids=lambda p: p.stem)
def test_gemv_matches_reference_golden(q4k, torch_mod, dev, path):
    z = np.load(path)
    nrows, K, ncols, _ = (int(v) for v in z["meta"])
    Wd = to_dev(torch_mod, z["W"], dev)
    got_q8 = q4k.mul_mat_vec_q8_1(Wd, to_dev(torch_mod, z["yq"], dev), K).cpu().numpy()
    got_f32 = q4k.mul_mat_vec_q(Wd, to_dev(torch_mod, z["x"], dev)).cpu().numpy()
    assert_close(got_q8, z["y_ref"], "q8_1 entry")
    assert_close(got_f32, z["y_ref"], "fp32 entry")


def test_strided_rows_columns_and_outputs(q4k, oracle, torch_mod, dev):
    torch = torch_mod
    nrows, K, ncols = 45, 1024, 3
    W, x = gen(q4k, 99, nrows, K, ncols)
    Wpad = np.zeros((nrows, (K // 256 + 3) * 144), np.uint8)  # stride_row_x = K/256 + 3
    Wpad[:, : W.shape[1]] = W
    xpad = np.zeros((ncols, K + 64), np.float32)
    xpad[:, :K] = x
    out = torch.full((ncols, nrows + 11), float("nan"), device=dev)
    q4k.mul_mat_vec_q(to_dev(torch, Wpad, dev), to_dev(torch, xpad, dev)[:, :K], out=out)
    o = out.cpu().numpy()
    assert_close(o[:, :nrows], oracle.gemv_f32(W, x))
    assert np.isnan(o[:, nrows:]).all()  # nothing written past nrows


def test_batch_of_tasks_with_shared_activations(q4k, oracle, torch_mod, dev):
    torch = torch_mod
    rng = np.random.default_rng(5)
    ncols = 2
    shapes = [(96, 1024), (32, 1024), (32, 1024), (96, 1024), (200, 1024), (200, 1024), (96, 3584)]
    xs_np = {1024: [rng.standard_normal((ncols, 1024)).astype(np.float32) for _ in range(3)],
             3584: [rng.standard_normal((ncols, 3584)).astype(np.float32)]}
    x_of = [0, 0, 0, 1, 2, 2, 0]  # q, k, v share; o own; gate/up share; down own
    Ws = [q4k.gen_q4k_numpy(rng, r, K) for r, K in shapes]
    Wd = [to_dev(torch, w, dev) for w in Ws]
    xd = {K: [to_dev(torch, a, dev) for a in v] for K, v in xs_np.items()}
    xs = [xd[K][i] for (r, K), i in zip(shapes, x_of)]
    outs = [torch.empty((ncols, r), device=dev) for r, _ in shapes]
    tasks = q4k.make_tasks(Wd, xs, outs)
    ws = q4k.Workspace(q4k.batch_workspace_bytes(tasks, ncols))
    q4k.gemv_batch(tasks, ncols, ws)
    for (r, K), i, W, o in zip(shapes, x_of, Ws, outs):
        assert_close(o.cpu().numpy(), oracle.gemv_f32(W, xs_np[K][i]), f"task {r}x{K}")
    assert ws.status() == 0


def test_op_mul_mat_vec_q_row_slice(q4k, oracle, torch_mod, dev):
    torch = torch_mod
    nrows, K, ncols = 300, 2048, 2
    W, x = gen(q4k, 17, nrows, K, ncols)
    Kp = q4k.kpad(K)
    yq = oracle.quantize_q8_1(x, Kpad=Kp)
    lo, hi = 77, 211
    out = torch.zeros((ncols, hi - lo + 5), device=dev)
    q4k.op_mul_mat_vec_q(to_dev(torch, W[lo:hi], dev), K, to_dev(torch, yq, dev), lo, hi, Kp, out=out,
                         nrows_dst=hi - lo + 5)
    assert_close(out.cpu().numpy()[:, : hi - lo], oracle.gemv_q8_1(W, K, yq)[:, lo:hi])


def test_custom_hook_contract(q4k, oracle, torch_mod, dev):
    torch = torch_mod
    nrows, K, ncols = 130, 4096, 4
    W, x = gen(q4k, 23, nrows, K, ncols)
    yq = oracle.quantize_q8_1(x)
    dst = torch.empty((ncols, nrows), device=dev)
    q4k.custom_q4k_gemv(to_dev(torch, W, dev), to_dev(torch, yq, dev), dst, K // 256, yq.shape[1] // 36, nrows,
                        ncols)
    assert_close(dst.cpu().numpy(), oracle.gemv_q8_1(W, K, yq))


# ------------------------------------------------------------ edge cases
def test_empty_and_degenerate_inputs(q4k, torch_mod, dev):
    torch = torch_mod
    W = torch.zeros((0, 144), dtype=torch.uint8, device=dev)
    x = torch.randn((1, 256), device=dev)
    out = q4k.mul_mat_vec_q(W, x)
    assert out.shape == (1, 0)
    # K = 0: every output is an empty sum
    L = q4k.lib()
    dst = torch.full((2, 5), 7.0, device=dev)
    ws = q4k.Workspace(1 << 20)
    st = L.q4k_mul_mat_vec(ws.ptr, x.data_ptr(), dst.data_ptr(), 0, 5, 2, 0, 0, 5, ws.ptr, ws.nbytes,
                           torch.cuda.current_stream().cuda_stream)
    assert st == 0
    assert (dst.cpu() == 0).all()


def test_bad_workspace_and_alignment(q4k, torch_mod, dev):
    torch = torch_mod
    L = q4k.lib()
    W = torch.zeros((32, 4 * 144 + 16), dtype=torch.uint8, device=dev)
    x = torch.randn((1, 1024), device=dev)
    dst = torch.empty((1, 32), device=dev)
    need = q4k.gemv_workspace_bytes(32, 1024, 1)
    ws = q4k.Workspace(need + 64)
    s = torch.cuda.current_stream().cuda_stream
    assert L.q4k_mul_mat_vec(W.data_ptr(), x.data_ptr(), dst.data_ptr(), 1024, 32, 1, 4, 1024, 32, ws.ptr,
                             need - 1, s) == 5
    assert L.q4k_mul_mat_vec(W.data_ptr(), x.data_ptr(), dst.data_ptr(), 1024, 32, 1, 4, 1024, 32, ws.ptr + 8,
                             need, s) == 5
    assert L.q4k_mul_mat_vec(W.data_ptr() + 8, x.data_ptr(), dst.data_ptr(), 1024, 32, 1, 4, 1024, 32, ws.ptr,
                             need, s) == 1
    assert L.q4k_mul_mat_vec(W.data_ptr(), x.data_ptr(), dst.data_ptr(), 1024, 32, 1, 4, 1024, 32, ws.ptr,
                             need, s) == 0
    assert ws.status() == 0


def test_deterministic_and_graph_capturable(q4k, torch_mod, dev):
    torch = torch_mod
    rng = np.random.default_rng(8)
    W = to_dev(torch, q4k.gen_q4k_numpy(rng, 2048, 4096), dev)
    x = to_dev(torch, rng.standard_normal((3, 4096)).astype(np.float32), dev)
    ws = q4k.Workspace(q4k.gemv_workspace_bytes(2048, 4096, 3))
    a = q4k.mul_mat_vec_q(W, x, ws=ws).clone()
    b = q4k.mul_mat_vec_q(W, x, ws=ws).clone()
    assert torch.equal(a, b)
    out = torch.empty_like(a)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        q4k.mul_mat_vec_q(W, x, out=out, ws=ws, stream=s)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        q4k.mul_mat_vec_q(W, x, out=out, ws=ws, stream=s)
    out.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, a)
    assert ws.status() == 0


# ------------------------------------------- full configuration sizes (sampled)
@pytest.mark.parametrize("nrows,K,ncols", [(4096, 4096, 1), (14336, 4096, 1), (14336, 4096, 2),
                                           (14336, 4096, 3), (14336, 4096, 4), (14336, 4096, 8),
                                           (4096, 14336, 1), (28672, 8192, 1), (8192, 28672, 1),
                                           (128256, 8192, 1), (1024, 4096, 1), (512, 4096, 1)])
def test_full_size_configs_row_sampled(q4k, oracle, torch_mod, dev, nrows, K, ncols):
    """BASELINE shapes at full size on the GPU, checked against the oracle on a
    seeded sample of rows (the oracle needs only those rows)."""
    torch = torch_mod
    g = torch.Generator(device=dev)
    g.manual_seed(nrows + K + ncols)
    Wd = q4k.gen_q4k_torch(nrows, K, generator=g, device=dev)
    xd = torch.randn((ncols, K), device=dev, generator=g)
    out = q4k.mul_mat_vec_q(Wd, xd)
    rows = np.unique(np.concatenate([np.array([0, nrows - 1]),
                                     np.random.default_rng(1).integers(0, nrows, 254)]))
    W_s = Wd[torch.from_numpy(rows).to(dev)].cpu().numpy()
    want = oracle.gemv_f32(W_s, xd.cpu().numpy())
    assert_close(out.cpu().numpy()[:, rows], want, f"{nrows}x{K} ncols={ncols}")

"""Q6_K weights (the other k-quant of Q4_K_M checkpoints): the oracle pinned
against the reference's own vec_dot_q6_K_q8_1 (kernels/vecdotq.cuh:867-890,
golden fixtures from tests/golden/make_golden.py: GEMV outputs in MMVQ order
and exact per-16-weight integer sums) and against gguf-py's Q6_K dequantizer
on the CPU; the CUDA path against the reference's fixtures and the oracle on
the GPU (every row, fp32 bar 1e-4 absolute + 1e-5 relative)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
Q6_GOLDEN = sorted(GOLDEN.glob("gemv_q6k_*.npz"))

TOL_ABS, TOL_REL = 1e-4, 1e-5


def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    bad = np.abs(got - want) > TOL_ABS + TOL_REL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance (first at {np.argwhere(bad)[:3]})"


def test_oracle_q6k_dequant_matches_gguf_py(q4k, oracle):
    import gguf
    rng = np.random.default_rng(1)
    W = q4k.gen_q6k_numpy(rng, 9, 2048)
    assert np.array_equal(oracle.dequant_q6k(W, 2048), gguf.quants.dequantize(W, gguf.GGMLQuantizationType.Q6_K))


def test_q6k_golden_fixtures_present():
    assert len(Q6_GOLDEN) >= 3 and (GOLDEN / "q6k_subblock_sums.npz").exists()


def test_oracle_q6k_subblock_sums_match_reference_golden(oracle):
    """The oracle's 6-bit unpacking (dequantized with d = 1 and unit scales,
    i.e. the signed values q6 - 32) times the q8 quants, summed per 16
    weights, equals the integers read out of the reference's dot product."""
    z = np.load(GOLDEN / "q6k_subblock_sums.npz")
    W, yq, S = z["W"], z["yq"], z["S"]
    for i in range(W.shape[0]):
        h = W[i].copy()
        h[192:208] = 1  # unit int8 scales
        h[208:210] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
        v = oracle.dequant_q6k(h[None, :], 256)[0].astype(np.int64)  # q6 - 32, exactly
        q = yq[i].reshape(8, 36)[:, 4:].view(np.int8).reshape(256).astype(np.int64)
        assert np.array_equal((v * q).reshape(16, 16).sum(axis=1), S[i].astype(np.int64)), f"super-block {i}"


@pytest.mark.parametrize("path", Q6_GOLDEN, ids=lambda p: p.stem)
def test_oracle_q6k_gemv_matches_reference_golden(oracle, path):
    z = np.load(path)
    nrows, K, ncols, _ = (int(v) for v in z["meta"])
    assert np.array_equal(oracle.quantize_q8_1(z["x"]), z["yq"])
    assert_close(oracle.gemv_q6k_q8_1(z["W"], K, z["yq"]), z["y_ref"], path.stem)


def test_oracle_q6k_gemv_is_the_dequantized_product(q4k, oracle):
    rng = np.random.default_rng(2)
    K = 2048
    W = q4k.gen_q6k_numpy(rng, 7, K)
    x = rng.standard_normal((2, K)).astype(np.float32)
    yq = oracle.quantize_q8_1(x)
    blk = yq.reshape(2, -1, 36)
    xq = (blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)[:, :, None] *
          blk[:, :, 4:].view(np.int8).astype(np.float64)).reshape(2, -1)[:, :K]
    want = oracle.dequant_q6k(W, K).astype(np.float64) @ xq.T
    got = oracle.gemv_q6k_q8_1(W, K, yq).astype(np.float64).T
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("nrows,K,ncols", [(8, 2048, 1), (37, 4096, 1), (37, 4096, 2), (300, 8192, 3),
                                           (1000, 14336, 1), (129, 4096, 8), (64, 28672, 5)])
def test_q6k_gemv_vs_oracle(q4k, oracle, nrows, K, ncols):
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(nrows + K + ncols)
    W = q4k.gen_q6k_numpy(rng, nrows, K)
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    Wd, xd = torch.from_numpy(W).to(dev), torch.from_numpy(x).to(dev)
    ws = q4k.Workspace()
    a = q4k.mul_mat_vec_q6_k(Wd, xd, ws=ws).clone()
    b = q4k.mul_mat_vec_q6_k(Wd, xd, ws=ws)
    assert torch.equal(a, b)
    assert ws.status() == 0
    assert_close(a.cpu().numpy(), oracle.gemv_q6k_f32(W, x), f"{nrows}x{K} ncols={ncols}")
    yq = oracle.quantize_q8_1(x)
    c = q4k.mul_mat_vec_q6_k_q8_1(Wd, torch.from_numpy(yq).to(dev), K)
    assert_close(c.cpu().numpy(), oracle.gemv_q6k_q8_1(W, K, yq), "q8_1 entry")


@pytest.mark.gpu
@pytest.mark.parametrize("path", Q6_GOLDEN, ids=lambda p: p.stem)
def test_q6k_gpu_matches_reference_golden(q4k, path):
    """The CUDA path on the reference's own fixtures: the q8_1 entry on the
    fixture's q8_1 blocks and the fp32 entry on its activations, both against
    y_ref from the reference's vec_dot_q6_K_q8_1."""
    import torch
    dev = torch.device("cuda", 0)
    z = np.load(path)
    nrows, K, ncols, _ = (int(v) for v in z["meta"])
    Wd = torch.from_numpy(z["W"]).to(dev)
    c = q4k.mul_mat_vec_q6_k_q8_1(Wd, torch.from_numpy(z["yq"]).to(dev), K)
    assert_close(c.cpu().numpy(), z["y_ref"], f"{path.stem} (q8_1 entry)")
    f = q4k.mul_mat_vec_q6_k(Wd, torch.from_numpy(z["x"]).to(dev))
    assert_close(f.cpu().numpy(), z["y_ref"], f"{path.stem} (fp32 entry)")


@pytest.mark.gpu
def test_q6k_output_head_full_size_all_rows(q4k, oracle):
    """Mistral-7B's Q4_K_M output head is Q6_K: 32000 x 4096, every row."""
    import torch
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    Wd = q4k.gen_q6k_torch(32000, 4096, generator=g, device=dev)
    xd = torch.randn((1, 4096), device=dev, generator=g)
    out = q4k.mul_mat_vec_q6_k(Wd, xd)
    assert_close(out.cpu().numpy(), oracle.gemv_q6k_f32(Wd.cpu().numpy(), xd.cpu().numpy()), "head")


@pytest.mark.gpu
def test_q6k_batch_and_strided_rows(q4k, oracle):
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(4)
    K = 4096
    Wa = q4k.gen_q6k_numpy(rng, 100, K)
    Wb_full = q4k.gen_q6k_numpy(rng, 60, K + 2048)  # stride_row_x = 24 super-blocks (multiple of 8)
    Wb = Wb_full[:, : K // 256 * 210]
    x = rng.standard_normal((2, K)).astype(np.float32)
    Wad = torch.from_numpy(Wa).to(dev)
    Wbd = torch.from_numpy(Wb_full).to(dev)[:, : K // 256 * 210]
    xd = torch.from_numpy(x).to(dev)
    outs = [torch.empty((2, 100), device=dev), torch.empty((2, 60), device=dev)]
    ws = q4k.Workspace()
    q4k.gemv_batch_q6_k(q4k.make_tasks_q6_k([Wad, Wbd], [xd, xd], outs), 2, ws)
    assert ws.status() == 0
    assert_close(outs[0].cpu().numpy(), oracle.gemv_q6k_f32(Wa, x), "a")
    assert_close(outs[1].cpu().numpy(), oracle.gemv_q6k_f32(np.ascontiguousarray(Wb), x), "b (strided rows)")

"""RMSNorm fused into the quantization launch (the rms_norm_f32 -> quantize_q8_1
steps of the reference's decode trace).

The oracle restates the library's reduction order (oracle/q4k_oracle.c,
or_rmsnorm), so the normalized-and-quantized q8_1 bytes must match bit for
bit; GEMVs on normalized activations are checked at the GEMV bar.
"""
from __future__ import annotations

import numpy as np
import pytest

TOL_ABS, TOL_REL = 1e-4, 1e-5


def assert_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    bad = np.abs(got - want) > TOL_ABS + TOL_REL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"


def test_oracle_rmsnorm_matches_definition(oracle):
    """CPU: the oracle's fixed-order RMSNorm is the textbook one to fp32 rounding."""
    rng = np.random.default_rng(0)
    for K in (100, 4096, 14336):
        x = (rng.standard_normal((2, K)) * rng.choice([1e-3, 1.0, 100.0], size=(2, 1))).astype(np.float32)
        w = rng.random(K).astype(np.float32) + 0.5
        y = oracle.rmsnorm(x, w, 1e-5)
        x64 = x.astype(np.float64)
        ref = x64 / np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + 1e-5) * w
        assert np.allclose(y, ref, rtol=1e-6, atol=1e-7), K
        assert np.array_equal(y, oracle.rmsnorm(x, w, 1e-5))  # deterministic


@pytest.mark.gpu
@pytest.mark.parametrize("K,Kpad,ncols,weighted,eps", [(4096, 4096, 1, True, 1e-5), (4096, 4096, 3, False, 1e-6),
                                                       (14336, 14336, 2, True, 1e-5), (100, 512, 2, True, 1e-5),
                                                       (28672, 28672, 1, True, 1e-5), (8192, 8192, 8, True, 1e-6)])
def test_rms_norm_quantize_bit_exact(q4k, oracle, K, Kpad, ncols, weighted, eps):
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(K + ncols)
    x = (rng.standard_normal((ncols, K)) * rng.choice([1e-3, 1.0, 300.0], size=(ncols, 1))).astype(np.float32)
    if ncols > 1:
        x[1] = 0.0  # an all-zero column: scale 1/sqrt(eps), every block quantizes to zeros
    w = (rng.random(K) + 0.5).astype(np.float32) if weighted else None
    got = q4k.rms_norm_quantize_q8_1(torch.from_numpy(x).to(dev), None if w is None else torch.from_numpy(w).to(dev),
                                     eps=eps, Kpad=Kpad).cpu().numpy()
    want = oracle.quantize_q8_1(oracle.rmsnorm(x, w, eps), Kpad=Kpad)
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_batch_with_normalized_activations(q4k, oracle):
    """q, k, v on RMSNorm(x_attn) (one shared normalized quantization), o on the
    raw x_attn (a second, plain quantization of the same buffer), down plain."""
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(9)
    ncols, K = 2, 2048
    shapes = {"q": (256, K), "k": (64, K), "v": (64, K), "o": (256, K), "down": (128, 1024)}
    W = {k: q4k.gen_q4k_numpy(rng, r, kk) for k, (r, kk) in shapes.items()}
    Wd = {k: torch.from_numpy(v).to(dev) for k, v in W.items()}
    x_attn = (rng.standard_normal((ncols, K)) * 3).astype(np.float32)
    x_down = rng.standard_normal((ncols, 1024)).astype(np.float32)
    w_norm = (rng.random(K) + 0.5).astype(np.float32)
    xa, xd, wn = (torch.from_numpy(a).to(dev) for a in (x_attn, x_down, w_norm))
    outs = {k: torch.empty((ncols, r), device=dev) for k, (r, _) in shapes.items()}
    items = [dict(W=Wd[k], x=xa, out=outs[k], rms_norm=True, norm_eps=1e-5, norm_weight=wn) for k in "qkv"]
    items += [dict(W=Wd["o"], x=xa, out=outs["o"]), dict(W=Wd["down"], x=xd, out=outs["down"])]
    ws = q4k.Workspace()
    q4k.gemv_batch_ex(q4k.make_tasks_ex(items), ncols, ws)
    assert ws.status() == 0
    yq = oracle.quantize_q8_1(oracle.rmsnorm(x_attn, w_norm, 1e-5))
    for k in "qkv":
        assert_close(outs[k].cpu().numpy(), oracle.gemv_q8_1(W[k], K, yq), k)
    assert_close(outs["o"].cpu().numpy(), oracle.gemv_f32(W["o"], x_attn), "o (raw x)")
    assert_close(outs["down"].cpu().numpy(), oracle.gemv_f32(W["down"], x_down), "down")

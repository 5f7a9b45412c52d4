"""Fused epilogue (kernels/mmvq.cu:182-227, :309-338): bias and gated linear
unit on the GEMV output, both matrices streamed in one launch.

Reference values: the oracle's GEMVs of the main and the gate matrix (exact
sums of the q8_1 arithmetic) with the op applied in fp64.  Tolerance: the
GEMV bar (1e-4 absolute + 1e-5 relative) on r and g, carried through the op
by its partial derivatives, plus the op's own fp32 evaluation error: 1e-5
relative, and 4x the deviation of an fp32 evaluation of the same formula on
the same inputs from the fp64 one (GEGLU's 1 + tanh(u) cancels for negative
g, in the reference's fp32 formula as in this one).  A plain bar on the
product would demand more than fp32 GEMVs can give: with |r| ~ 1000 and g
near 0, r * silu(g) moves by |r| * 0.5 * dg.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-4, 1e-5


def glu_ref(op, r, g, dtype=np.float64):
    r = np.asarray(r, dtype)
    g = np.asarray(g, dtype)
    c = lambda v: dtype(v)  # noqa: E731
    if op == "swiglu":
        return r * (g / (c(1.0) + np.exp(-g)))
    if op == "geglu":
        u = c(np.sqrt(2.0 / np.pi)) * g * (c(1.0) + c(0.044715) * g * g)
        return r * (c(0.5) * g * (c(1.0) + np.tanh(u)))
    if op == "swiglu_oai":
        a = np.minimum(g, c(7.0))
        b = np.clip(r, c(-7.0), c(7.0))
        return a / (c(1.0) + np.exp(-a * c(1.702))) * (c(1.0) + b)
    if op == "mul":
        return r * g
    return r


def glu_tol(op, r, g):
    r = np.asarray(r, np.float64)
    g = np.asarray(g, np.float64)
    tr, tg = TOL_ABS + TOL_REL * np.abs(r), TOL_ABS + TOL_REL * np.abs(g)
    hr, hg = np.maximum(1e-3, 1e-4 * np.abs(r)), np.maximum(1e-3, 1e-4 * np.abs(g))
    dr = np.abs(glu_ref(op, r + hr, g) - glu_ref(op, r - hr, g)) / (2 * hr)
    dg = np.abs(glu_ref(op, r, g + hg) - glu_ref(op, r, g - hg)) / (2 * hg)
    out = glu_ref(op, r, g)
    with np.errstate(over="ignore"):
        f32 = glu_ref(op, r.astype(np.float32), g.astype(np.float32), np.float32).astype(np.float64)
    return dr * tr + dg * tg + 1e-5 * np.abs(out) + 4 * np.abs(f32 - out) + 1e-6


def check(got, r, g, op, what):
    want = glu_ref(op, r, g)
    tol = glu_tol(op, r, g) if op != "none" else TOL_ABS + TOL_REL * np.abs(want)
    err = np.abs(np.asarray(got, np.float64) - want)
    bad = err > tol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance, worst {np.max(err / tol):.3g}"


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def dev(q4k, torch_mod):
    assert q4k.lib().q4k_device_supported() == 1
    return torch_mod.device("cuda", 0)


def to_dev(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("op", ["swiglu", "geglu", "swiglu_oai", "mul"])
@pytest.mark.parametrize("ncols,biases", [(1, False), (1, True), (3, True)])
def test_fused_glu_vs_oracle(q4k, oracle, torch_mod, dev, op, ncols, biases):
    torch = torch_mod
    rng = np.random.default_rng(ncols * 10 + len(op))
    nrows, K = 200, 2048
    Wu, Wg = q4k.gen_q4k_numpy(rng, nrows, K), q4k.gen_q4k_numpy(rng, nrows, K)
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    if op == "swiglu_oai":
        x *= 0.01  # keep r and g around the clamp limits (|r|, |g| ~ 7)
    xb = (rng.standard_normal((ncols, nrows)) * 3).astype(np.float32) if biases else None
    gb = (rng.standard_normal((ncols, nrows)) * 3).astype(np.float32) if biases else None
    out = q4k.mul_mat_vec_fused(to_dev(torch, Wu, dev), to_dev(torch, Wg, dev), to_dev(torch, x, dev), glu=op,
                                x_bias=None if xb is None else to_dev(torch, xb, dev),
                                gate_bias=None if gb is None else to_dev(torch, gb, dev))
    r = oracle.gemv_f32(Wu, x).astype(np.float64) + (0 if xb is None else xb)
    g = oracle.gemv_f32(Wg, x).astype(np.float64) + (0 if gb is None else gb)
    check(out.cpu().numpy(), r, g, op, f"{op} ncols={ncols} biases={biases}")


def test_fused_q8_1_entry_and_bias_only(q4k, oracle, torch_mod, dev):
    torch = torch_mod
    rng = np.random.default_rng(77)
    nrows, K = 130, 4096
    Wu, Wg = q4k.gen_q4k_numpy(rng, nrows, K), q4k.gen_q4k_numpy(rng, nrows, K)
    x = rng.standard_normal((2, K)).astype(np.float32)
    yq = oracle.quantize_q8_1(x)
    xb = rng.standard_normal((2, nrows)).astype(np.float32)
    Wud, Wgd, yqd, xbd = (to_dev(torch, a, dev) for a in (Wu, Wg, yq, xb))
    out = q4k.mul_mat_vec_q8_1_fused(Wud, Wgd, yqd, K, glu="swiglu", x_bias=xbd)
    r = oracle.gemv_q8_1(Wu, K, yq).astype(np.float64) + xb
    g = oracle.gemv_q8_1(Wg, K, yq).astype(np.float64)
    check(out.cpu().numpy(), r, g, "swiglu", "q8_1 entry")
    # a bias without a gate: r + x_bias
    out2 = q4k.mul_mat_vec_q8_1_fused(Wud, None, yqd, K, glu="none", x_bias=xbd)
    check(out2.cpu().numpy(), r, r, "none", "bias only")


@pytest.mark.parametrize("ncols", [1, 2])
def test_fused_gate_up_full_size_all_rows(q4k, oracle, torch_mod, dev, ncols):
    """Mistral ffn gate/up (2 x 14336x4096): every row, split row groups included."""
    torch = torch_mod
    g_ = torch.Generator(device=dev)
    g_.manual_seed(5 + ncols)
    Wu = q4k.gen_q4k_torch(14336, 4096, generator=g_, device=dev)
    Wg = q4k.gen_q4k_torch(14336, 4096, generator=g_, device=dev)
    x = torch.randn((ncols, 4096), device=dev, generator=g_)
    ws = q4k.Workspace()
    a = q4k.mul_mat_vec_fused(Wu, Wg, x, glu="swiglu", ws=ws).clone()
    b = q4k.mul_mat_vec_fused(Wu, Wg, x, glu="swiglu", ws=ws)
    assert torch.equal(a, b)
    assert ws.status() == 0
    xn = x.cpu().numpy()
    r = oracle.gemv_f32(Wu.cpu().numpy(), xn).astype(np.float64)
    g = oracle.gemv_f32(Wg.cpu().numpy(), xn).astype(np.float64)
    check(a.cpu().numpy(), r, g, "swiglu", f"gate/up ncols={ncols}")


def test_batch_ex_layer_with_fused_ffn(q4k, oracle, torch_mod, dev):
    """A decoder layer's batch with gate+up fused: q, k, v, o, glu(up, gate), down in one launch."""
    torch = torch_mod
    rng = np.random.default_rng(21)
    ncols = 1
    shapes = {"q": (512, 1024), "k": (128, 1024), "v": (128, 1024), "o": (512, 1024), "up": (1792, 1024),
              "gate": (1792, 1024), "down": (512, 1792)}
    W = {k: q4k.gen_q4k_numpy(rng, r, K) for k, (r, K) in shapes.items()}
    Wd = {k: to_dev(torch, v, dev) for k, v in W.items()}
    xs = {n: rng.standard_normal((ncols, K)).astype(np.float32) for n, K in
          (("attn", 1024), ("o", 1024), ("ffn", 1024), ("down", 1792))}
    xd = {k: to_dev(torch, v, dev) for k, v in xs.items()}
    outs = {k: torch.empty((ncols, shapes[k][0]), device=dev) for k in ("q", "k", "v", "o", "up", "down")}
    items = [dict(W=Wd["q"], x=xd["attn"], out=outs["q"]), dict(W=Wd["k"], x=xd["attn"], out=outs["k"]),
             dict(W=Wd["v"], x=xd["attn"], out=outs["v"]), dict(W=Wd["o"], x=xd["o"], out=outs["o"]),
             dict(W=Wd["up"], W_gate=Wd["gate"], x=xd["ffn"], out=outs["up"], glu="swiglu"),
             dict(W=Wd["down"], x=xd["down"], out=outs["down"])]
    tasks = q4k.make_tasks_ex(items)
    ws = q4k.Workspace()
    q4k.gemv_batch_ex(tasks, ncols, ws)
    assert ws.status() == 0
    for name, xname in (("q", "attn"), ("k", "attn"), ("v", "attn"), ("o", "o"), ("down", "down")):
        want = oracle.gemv_f32(W[name], xs[xname]).astype(np.float64)
        check(outs[name].cpu().numpy(), want, want, "none", name)
    r = oracle.gemv_f32(W["up"], xs["ffn"]).astype(np.float64)
    g = oracle.gemv_f32(W["gate"], xs["ffn"]).astype(np.float64)
    check(outs["up"].cpu().numpy(), r, g, "swiglu", "fused ffn")

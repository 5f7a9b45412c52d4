"""The CPU oracle, pinned against the reference's own code and an independent
Q4_K implementation.  No GPU needed.

Pins:
  * tests/golden/*.npz were produced from the reference's vec_dot_q4_K_q8_1
    (kernels/vecdotq.cuh:775-819) compiled on the host (tests/golden/make_golden.py);
  * gguf-py's Q4_K dequantizer (an independent implementation of the same
    format) cross-checks the byte layout and the 6-bit scale unpacking;
  * hand-derived known answers for the q8_1 quantizer.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL_ABS, TOL_REL = 1e-4, 1e-5  # fp32 output tolerance of the north star


def close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.all(np.abs(a - b) <= TOL_ABS + TOL_REL * np.abs(b))


# ---------------------------------------------------------------- half floats
def test_h2f_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.h2f(int(v)) for v in h], dtype=np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(ref)]))


def test_f2h_round_to_nearest_even(oracle):
    rng = np.random.default_rng(0)
    f = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                  2.0 ** -14, 6.1e-5, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32)])
    ref = f.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f2h(float(v)) for v in f], dtype=np.uint16)
    assert np.array_equal(got, ref)


# ------------------------------------------------------------- layout checks
def test_scale_min_matches_gguf(oracle):
    gguf_quants = pytest.importorskip("gguf.quants")
    rng = np.random.default_rng(1)
    scales = rng.integers(0, 256, size=(4096, 12), dtype=np.uint8)
    sc_ref, m_ref = gguf_quants.Q4_K.get_scale_min(scales)
    import ctypes
    L = oracle.lib()
    L.or_scale_min.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_int)]
    sc, m = ctypes.c_int(), ctypes.c_int()
    for i in range(0, 4096, 7):
        row = np.ascontiguousarray(scales[i])
        for s in range(8):
            L.or_scale_min(row.ctypes.data, s, ctypes.byref(sc), ctypes.byref(m))
            assert (sc.value, m.value) == (int(sc_ref[i, s]), int(m_ref[i, s]))


def test_dot_matches_gguf_dequantized_weights(oracle, q4k):
    """Oracle GEMV == fp64 dot of gguf-dequantized weights with d8*q8 activations."""
    gguf_quants = pytest.importorskip("gguf.quants")
    rng = np.random.default_rng(2)
    nrows, K = 12, 1024
    W = q4k.gen_q4k_numpy(rng, nrows, K)
    x = rng.standard_normal((1, K)).astype(np.float32)
    yq = oracle.quantize_q8_1(x)
    deq = gguf_quants.Q4_K.dequantize_blocks(W.reshape(-1, 144)).reshape(nrows, K).astype(np.float64)
    blocks = yq.reshape(-1, 36)[: K // 32]
    d8 = blocks[:, 0:2].copy().view(np.float16).astype(np.float64).reshape(-1)
    q8 = blocks[:, 4:].view(np.int8).astype(np.float64)
    act = (q8 * d8[:, None]).reshape(K)
    expect = deq @ act
    got = oracle.gemv_q8_1(W, K, yq)[0]
    # gguf rounds each weight to fp32 once; allow a few ulp of the row magnitude
    scale = np.abs(deq).sum(axis=1) * np.abs(act).max()
    assert np.all(np.abs(got - expect) <= 1e-6 * scale + 1e-5)


# ------------------------------------------------------------- q8_1 quantizer
def test_q8_1_known_answers(oracle):
    z = np.load(GOLDEN / "q8_1_kat.npz")
    x, Kpad = z["x"], int(z["Kpad"])
    yq = oracle.quantize_q8_1(x, Kpad=Kpad)
    assert np.array_equal(yq, z["yq"])
    b = yq[0].reshape(-1, 36)
    half = lambda blk, o: float(blk[o:o + 2].copy().view(np.float16)[0])
    q = lambda blk: blk[4:].view(np.int8).astype(np.int64)
    # block 0: all zeros -> d = 0, sum = 0, q = 0
    assert half(b[0], 0) == 0.0 and half(b[0], 2) == 0.0 and not q(b[0]).any()
    # block 1: amax = 127 -> d = 1 and q = x exactly (incl. saturation at +-127)
    assert half(b[1], 0) == 1.0
    assert np.array_equal(q(b[1]), x[0, 32:64].astype(np.int64))
    # block 2: amax 63.5 -> d = 0.5, x/d = k + 0.5 exactly -> round half away from zero
    assert half(b[2], 0) == 0.5
    exp = x[0, 64:96] / np.float32(0.5)
    assert np.array_equal(q(b[2]), (np.sign(exp) * np.floor(np.abs(exp) + 0.5)).astype(np.int64))
    # ragged K = 100: block 3 holds 4 real values, blocks 4..15 are zero padding
    assert not q(b[3])[4:].any()
    for k in range(4, Kpad // 32):
        assert not b[k].any()
    # random column: |q| <= 127 and q = roundf(x / d) with d = amax/127
    b1 = yq[1].reshape(-1, 36)
    for k in range(3):
        xs = x[1, 32 * k:32 * k + 32]
        d = np.float32(np.abs(xs).max()) / np.float32(127)
        r = xs / d
        assert np.array_equal(q(b1[k]), (np.sign(r) * np.floor(np.abs(r) + np.float32(0.5))).astype(np.int64))
        assert half(b1[k], 0) == float(np.float16(d))


def test_q8_1_sum_is_butterfly_order(oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((1, 256)) * 100).astype(np.float32)
    yq = oracle.quantize_q8_1(x, Kpad=256).reshape(-1, 36)
    for k in range(8):
        t = x[0, 32 * k:32 * k + 32].copy()
        for off in (16, 8, 4, 2, 1):
            t = (t + t[np.arange(32) ^ off]).astype(np.float32)
        assert yq[k, 2:4].copy().view(np.float16)[0] == np.float16(t[0])


# ------------------------------------------------- pinned against the reference
def test_subblock_sums_match_reference_golden(oracle):
    z = np.load(GOLDEN / "subblock_sums.npz")
    W, yq = z["W"], z["yq"]
    import ctypes
    for i in range(W.shape[0]):
        S = np.zeros(8, np.int32)
        T = np.zeros(8, np.int32)
        sb = np.ascontiguousarray(W[i])
        q8 = np.ascontiguousarray(yq[i])
        oracle.lib().or_subblock_sums_sb(sb.ctypes.data, q8.ctypes.data, S.ctypes.data, T.ctypes.data)
        assert np.array_equal(S, z["S"][i]), i
        assert np.array_equal(T, z["T"][i]), i


@pytest.mark.parametrize("path", sorted(p for p in GOLDEN.glob("gemv_*.npz") if not p.stem.startswith("gemv_q6k_")),
                         ids=lambda p: p.stem)
def test_gemv_matches_reference_golden(oracle, path):
    z = np.load(path)
    nrows, K, ncols, _ = (int(v) for v in z["meta"])
    yq = oracle.quantize_q8_1(z["x"])
    assert np.array_equal(yq, z["yq"])  # quantizer unchanged since the fixture was made
    y = oracle.gemv_q8_1(z["W"], K, yq)
    assert y.shape == (ncols, nrows)
    assert close(y, z["y_ref"])


def test_oracle_vs_reference_random_shapes(oracle, q4k):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    rng = np.random.default_rng(11)
    for nrows, K, ncols in [(3, 256, 1), (17, 768, 5), (40, 4096, 8), (6, 28672, 1)]:
        W = q4k.gen_q4k_numpy(rng, nrows, K)
        x = rng.standard_normal((ncols, K)).astype(np.float32)
        yq = oracle.quantize_q8_1(x)
        assert close(oracle.gemv_q8_1(W, K, yq), oracle.ref_gemv_q8_1(W, K, yq))


def test_gemv_f32_entry_equals_quantize_then_gemv(oracle, q4k):
    rng = np.random.default_rng(12)
    W = q4k.gen_q4k_numpy(rng, 9, 512)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    a = oracle.gemv_f32(W, x)
    b = oracle.gemv_q8_1(W, 512, oracle.quantize_q8_1(x))
    assert np.array_equal(a, b)

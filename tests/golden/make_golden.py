"""Generate the golden fixtures in this directory from the REFERENCE's own code.

Run here, where the reference checkout exists (the fixtures are committed; the
GPU box never needs the reference):

    make -C oracle && python tests/golden/make_golden.py

Outputs (numpy .npz, a few hundred KB in total):

  gemv_<name>.npz  seeded Q4_K weights W, fp32 activations x, their q8_1
                   quantization yq (this project's quantizer: the reference
                   calls upstream quantize_q8_1, which it does not ship), and
                   y_ref = the reference's vec_dot_q4_K_q8_1
                   (kernels/vecdotq.cuh:775-819) summed in upstream MMVQ order
                   (kernels/mmvq.cu:236-301), via oracle/_ref/libq4k_ref.so.
  subblock_sums.npz  exact per-sub-block integer sums S (nibble.q8) and T (sum
                   q8) of seeded super-blocks, read out of the reference's dot
                   product by giving each super-block a one-hot header
                   (d = 1, sc_s = 1 for one s, everything else 0; or d = 0,
                   dmin = -1, m_s = 1): the reference then returns exactly S_s
                   (or T_s), a small integer that fp32 holds exactly.
  q8_1_kat.npz     hand-made q8_1 quantization cases (zeros, saturation,
                   ties, padding) with their expected blocks.
  gemv_q6k_<name>.npz  the same as gemv_<name>.npz for Q6_K weights (210-byte
                   super-blocks), y_ref = the reference's vec_dot_q6_K_q8_1
                   (kernels/vecdotq.cuh:867-890, VDR 1 at :576) in MMVQ order.
  q6k_subblock_sums.npz  exact per-16-weight sums S = sum (q6 - 32) * q8 of
                   seeded Q6_K super-blocks, read out of the reference's dot
                   product with d = 1, one scale = 1 and the others 0, d8 = 1.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402

QK_K, SB = 256, 144


def gen_w(rng, nrows, K):
    nb = K // QK_K
    W = rng.integers(0, 256, size=(nrows, nb, SB), dtype=np.uint8)
    d = (np.abs(rng.standard_normal((nrows, nb, 2))) * 0.01).astype(np.float16)
    W[:, :, 0:4] = d.view(np.uint8).reshape(nrows, nb, 4)
    return W.reshape(nrows, nb * SB)


def pack_scales(sc, m):
    """Inverse of the 6-bit unpacking (kernels/vecdotq.cuh:796-807)."""
    b = np.zeros(12, dtype=np.uint8)
    for s in range(4):
        b[s] = (sc[s] & 63) | ((sc[s + 4] >> 4) << 6)
        b[s + 4] = (m[s] & 63) | ((m[s + 4] >> 4) << 6)
        b[s + 8] = (sc[s + 4] & 15) | ((m[s + 4] & 15) << 4)
    return b


def ref_sb_value(sb, q8):
    """sum over iqs = 0,2,..,30 of the reference's vec_dot (one super-block)."""
    return sum(O.ref_vec_dot(sb, q8, iqs) for iqs in range(0, 32, 2))


def extract_sums(sb, q8):
    """Exact S_s, T_s of one super-block from the reference's dot product."""
    one = np.float16(1.0).view(np.uint16)
    mone = np.float16(-1.0).view(np.uint16)
    q8 = q8.copy().reshape(8, 36)
    q8[:, 0:2] = np.frombuffer(np.uint16(one).tobytes(), dtype=np.uint8)  # d8 = 1
    q8 = q8.reshape(-1)
    S, T = np.zeros(8, np.int32), np.zeros(8, np.int32)
    for s in range(8):
        h = sb.copy()
        h[0:2] = np.frombuffer(np.uint16(one).tobytes(), np.uint8)
        h[2:4] = 0
        sc = np.zeros(8, np.int64); sc[s] = 1
        h[4:16] = pack_scales(sc, np.zeros(8, np.int64))
        v = ref_sb_value(h, q8)
        assert v == int(v)
        S[s] = int(v)
        h = sb.copy()
        h[0:2] = 0
        h[2:4] = np.frombuffer(np.uint16(mone).tobytes(), np.uint8)
        m = np.zeros(8, np.int64); m[s] = 1
        h[4:16] = pack_scales(np.zeros(8, np.int64), m)
        v = ref_sb_value(h, q8)
        assert v == int(v)
        T[s] = int(v)
    return S, T


def gemv_case(name, seed, nrows, K, ncols, full_rows=None):
    rng = np.random.default_rng(seed)
    if full_rows is None:
        W = gen_w(rng, nrows, K)
    else:  # first nrows rows of a full_rows x K matrix drawn with this seed
        W = gen_w(rng, full_rows, K)[:nrows].copy()
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    yq = O.quantize_q8_1(x)
    y_ref = O.ref_gemv_q8_1(W, K, yq)
    np.savez_compressed(HERE / f"gemv_{name}.npz", W=W, x=x, yq=yq, y_ref=y_ref,
                        meta=np.array([nrows, K, ncols, seed], dtype=np.int64))
    return W.nbytes + x.nbytes


def subblock_case(seed=7, nsb=24):
    rng = np.random.default_rng(seed)
    W = gen_w(rng, nsb, QK_K)
    x = rng.standard_normal((1, nsb * QK_K)).astype(np.float32)
    # make some blocks saturate / vanish to cover the extremes
    x[0, 0:32] = 0.0
    x[0, 32:64] = 1000.0
    x[0, 64:96] = -1000.0
    yq = O.quantize_q8_1(x, Kpad=nsb * QK_K).reshape(nsb, 8 * 36)
    W = W.reshape(nsb, SB)
    W[1, 16:] = 0xFF  # all nibbles 15
    W[2, 16:] = 0x00
    S = np.zeros((nsb, 8), np.int32)
    T = np.zeros((nsb, 8), np.int32)
    for i in range(nsb):
        S[i], T[i] = extract_sums(W[i], yq[i])
    np.savez_compressed(HERE / "subblock_sums.npz", W=W, yq=yq, S=S, T=T)


def q8_kat():
    K = 128
    x = np.zeros((2, K), np.float32)
    # block 0: all zero -> d = 0, q = 0
    # block 1: amax 127 -> d = 1, q = x exactly, incl. +-127
    x[0, 32:64] = np.arange(-16, 16, dtype=np.float32) * 8.0 - 1.0
    x[0, 32] = -127.0
    x[0, 63] = 127.0
    # block 2: exact .5 ties after division (amax 63.5 -> d = 0.5): x/d = k + 0.5 for x = (k+.5)/2
    x[0, 64:96] = (np.arange(32, dtype=np.float32) - 16.0 + 0.5) * 0.5
    x[0, 64] = 63.5
    # block 3: tiny values (half subnormal d)
    x[0, 96:128] = np.linspace(-1e-6, 1e-6, 32, dtype=np.float32)
    x[1] = np.random.default_rng(3).standard_normal(K).astype(np.float32) * 5
    Kv = 100  # ragged K: positions 100..511 are padding
    yq = O.quantize_q8_1(x[:, :Kv].copy(), Kpad=512)
    np.savez_compressed(HERE / "q8_1_kat.npz", x=x[:, :Kv].copy(), yq=yq, Kpad=np.int64(512))


Q6 = 210


def gen_w6(rng, nrows, K):
    """Q6_K rows: ql/qh/scales bytes uniform, d = fp16(|N(0,1)|*0.01)."""
    nb = K // QK_K
    W = rng.integers(0, 256, size=(nrows, nb, Q6), dtype=np.uint8)
    d = (np.abs(rng.standard_normal((nrows, nb))) * 0.01).astype(np.float16)
    W[:, :, 208:210] = d.view(np.uint8).reshape(nrows, nb, 2)
    return W.reshape(nrows, nb * Q6)


def gemv_q6k_case(name, seed, nrows, K, ncols):
    rng = np.random.default_rng(seed)
    W = gen_w6(rng, nrows, K)
    x = rng.standard_normal((ncols, K)).astype(np.float32)
    yq = O.quantize_q8_1(x)
    y_ref = O.ref_gemv_q6k_q8_1(W, K, yq)
    np.savez_compressed(HERE / f"gemv_q6k_{name}.npz", W=W, x=x, yq=yq, y_ref=y_ref,
                        meta=np.array([nrows, K, ncols, seed], dtype=np.int64))
    return W.nbytes + x.nbytes


def q6k_subblock_case(seed=11, nsb=12):
    """S[i, s] = sum over the 16 weights of sub-block s of (q6 - 32) * q8, from the
    reference's dot product summed over all 32 threads of a super-block
    (iqs = 0..31, VDR 1): with d = 1, scales = one-hot at s and every q8
    block's d8 = 1 it returns exactly that integer."""
    rng = np.random.default_rng(seed)
    W = gen_w6(rng, nsb, QK_K).reshape(nsb, Q6)
    W[1, 0:192] = 0xFF  # every 6-bit value 63 (+31 after the offset)
    W[2, 0:192] = 0x00  # every value 0 (-32)
    x = rng.standard_normal((1, nsb * QK_K)).astype(np.float32)
    x[0, 32:64] = 1000.0   # a saturating block
    x[0, 64:96] = -1000.0
    yq = O.quantize_q8_1(x, Kpad=nsb * QK_K).reshape(nsb, 8, 36).copy()
    yq[:, :, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)  # d8 = 1
    yq = yq.reshape(nsb, 8 * 36)
    S = np.zeros((nsb, 16), np.int32)
    for i in range(nsb):
        for s in range(16):
            h = W[i].copy()
            h[192:208] = 0
            h[192 + s] = 1
            h[208:210] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
            v = sum(O.ref_vec_dot_q6k(h, yq[i], iqs) for iqs in range(32))
            assert v == int(v)
            S[i, s] = int(v)
    np.savez_compressed(HERE / "q6k_subblock_sums.npz", W=W, yq=yq, S=S)


def main():
    assert O.ref_available(), "oracle/_ref missing: run make -C oracle with the reference present"
    total = 0
    total += gemv_case("k256_r7_c1", 1, 7, 256, 1)
    total += gemv_case("k512_r33_c3", 2, 33, 512, 3)
    total += gemv_case("k2048_r9_c8", 3, 9, 2048, 8)
    total += gemv_case("k4096_r32_c2", 4, 32, 4096, 2)
    total += gemv_case("k14336_r5_c2", 5, 5, 14336, 2)
    # BASELINE config 1 (4096x4096, seed 0, batch 1): its first 16 rows
    total += gemv_case("cfg1_k4096_r16_c1", 0, 16, 4096, 1, full_rows=4096)
    subblock_case()
    q8_kat()
    # Q6_K (K a multiple of 2048, as the GPU path needs): odd row counts, batch 1..8
    total += gemv_q6k_case("k2048_r9_c1", 21, 9, 2048, 1)
    total += gemv_q6k_case("k4096_r17_c2", 22, 17, 4096, 2)
    total += gemv_q6k_case("k8192_r8_c8", 23, 8, 8192, 8)
    q6k_subblock_case()
    print("golden fixtures written; raw payload bytes", total)


if __name__ == "__main__":
    main()

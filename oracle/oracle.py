"""ctypes front-end to the CPU checkers built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's cpu_baseline / --impl reference legs, always as the checker or the
timed CPU baseline, never on the product path.

Two libraries:
  * liboracle_q4k.so  -- this project's C restatement (q4k_oracle.c);
  * _ref/libq4k_ref.so -- the reference's own kernels/vecdotq.cuh compiled for
    the host (present when the reference checkout was available at build time).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle_q4k.so"
REF_SO = HERE / "_ref" / "libq4k_ref.so"

QK_K = 256
QK8_1 = 32
Q4K_BYTES = 144
Q81_BYTES = 36

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p


def reference_dir() -> Path | None:
    """The reference checkout: $Q4K_REFERENCE, else a `reference` directory
    beside this repository's checkout; None when neither exists."""
    env = os.environ.get("Q4K_REFERENCE")
    if env:
        return Path(env)
    sibling = HERE.parent.parent / "reference"
    return sibling if sibling.is_dir() else None


def build(force: bool = False) -> None:
    """Build the checkers (make in oracle/).  Cheap; safe to call repeatedly."""
    if force or not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(HERE), "liboracle_q4k.so"], check=True,
                       stdout=subprocess.DEVNULL)
    ref_dir = reference_dir()
    ref_src = ref_dir / "kernels" / "vecdotq.cuh" if ref_dir is not None else None
    if ref_src is not None and ref_src.exists() and (force or not REF_SO.exists()):
        subprocess.run(["make", "-C", str(HERE), "ref", f"REF={ref_src.parent.parent}"],
                       check=True, stdout=subprocess.DEVNULL)


_lib = None
_ref = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.or_h2f.argtypes = [ctypes.c_uint16]
        L.or_h2f.restype = ctypes.c_float
        L.or_f2h.argtypes = [ctypes.c_float]
        L.or_f2h.restype = ctypes.c_uint16
        L.or_quantize_q8_1.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p]
        L.or_rmsnorm.argtypes = [_c_p, _c_i64, _c_i64, ctypes.c_int, _c_p, ctypes.c_float, _c_p]
        L.or_dequant_q6k.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p]
        L.or_gemv_q6k_q8_1.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int, _c_p, _c_i64,
                                       ctypes.c_int]
        L.or_rmsnorm_scale.argtypes = [_c_p, _c_i64, ctypes.c_float]
        L.or_rmsnorm_scale.restype = ctypes.c_float
        L.or_subblock_sums_sb.argtypes = [_c_p, _c_p, _c_p, _c_p]
        L.or_gemv_q4k_q8_1.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int,
                                       _c_p, _c_i64, ctypes.c_int]
        L.or_gemv_q4k_f32.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int,
                                      _c_p, _c_i64, ctypes.c_int]
        L.or_subblock_sums.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int,
                                       _c_p, _c_p]
        L.or_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    """The reference's own dot product compiled for the host (oracle/_ref)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} missing (build with the reference checkout present)")
        L = ctypes.CDLL(str(REF_SO))
        L.ref_vec_dot_q4_K_q8_1.argtypes = [_c_p, _c_p, ctypes.c_int, ctypes.c_int]
        L.ref_vec_dot_q4_K_q8_1.restype = ctypes.c_float
        L.ref_gemv_q4k_q8_1.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int,
                                        _c_p, _c_i64, ctypes.c_int]
        L.ref_vec_dot_q6_K_q8_1.argtypes = [_c_p, _c_p, ctypes.c_int, ctypes.c_int]
        L.ref_vec_dot_q6_K_q8_1.restype = ctypes.c_float
        L.ref_gemv_q6k_q8_1.argtypes = [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, ctypes.c_int,
                                        _c_p, _c_i64, ctypes.c_int]
        L.ref_max_threads.restype = ctypes.c_int
        _ref = L
    return _ref


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def kpad(K: int) -> int:
    """K rounded up to the q8_1 row padding (kernels/mmvq.cu:728, 512)."""
    return (K + 511) // 512 * 512


def quantize_q8_1(x: np.ndarray, Kpad: int | None = None) -> np.ndarray:
    """x: (ncols, K) float32 -> (ncols, Kpad/32*36) uint8 ggml block_q8_1 rows."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    ncols, K = x.shape
    Kp = kpad(K) if Kpad is None else Kpad
    out = np.zeros((ncols, Kp // QK8_1 * Q81_BYTES), dtype=np.uint8)
    lib().or_quantize_q8_1(_ptr(x), K, K, Kp, ncols, _ptr(out))
    return out


Q6K_BYTES = 210


def dequant_q6k(W: np.ndarray, K: int) -> np.ndarray:
    """Q6_K rows (nrows, K/256*210) uint8 -> (nrows, K) float32."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    out = np.empty((W.shape[0], K), dtype=np.float32)
    lib().or_dequant_q6k(_ptr(W), W.shape[0], K, W.shape[1] // Q6K_BYTES, _ptr(out))
    return out


def gemv_q6k_q8_1(W: np.ndarray, K: int, yq: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """Q6_K rows x q8_1 columns (ncols, Kpad/32*36) -> (ncols, nrows) float32 (exact sums)."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    yq = np.ascontiguousarray(yq, dtype=np.uint8)
    nrows, ncols = W.shape[0], yq.shape[0]
    out = np.empty((ncols, nrows), dtype=np.float32)
    lib().or_gemv_q6k_q8_1(_ptr(W), nrows, K, W.shape[1] // Q6K_BYTES, _ptr(yq), yq.shape[1] // Q81_BYTES, ncols,
                           _ptr(out), nrows, nthreads)
    return out


def gemv_q6k_f32(W: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """fp32 x (ncols, K): q8_1 quantization, then the Q6_K product."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    return gemv_q6k_q8_1(W, x.shape[1], quantize_q8_1(x), nthreads)


def rmsnorm(x: np.ndarray, w: np.ndarray | None = None, eps: float = 1e-5) -> np.ndarray:
    """(ncols, K) float32 -> RMSNorm(x) * w in the library's reduction order (bit-exact)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    ncols, K = x.shape
    y = np.empty_like(x)
    wa = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    lib().or_rmsnorm(_ptr(x), K, K, ncols, None if wa is None else _ptr(wa), eps, _ptr(y))
    return y


def gemv_q8_1(W: np.ndarray, K: int, yq: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """W: (nrows, K/256*144) uint8; yq: (ncols, blocks*36) uint8 -> (ncols, nrows) float32."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    yq = np.ascontiguousarray(yq, dtype=np.uint8)
    nrows = W.shape[0]
    ncols = yq.shape[0]
    out = np.empty((ncols, nrows), dtype=np.float32)
    lib().or_gemv_q4k_q8_1(_ptr(W), nrows, K, W.shape[1] // Q4K_BYTES, _ptr(yq),
                           yq.shape[1] // Q81_BYTES, ncols, _ptr(out), nrows, nthreads)
    return out


def gemv_f32(W: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """fp32 activations (ncols, K): quantize to q8_1 then GEMV -> (ncols, nrows)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    return gemv_q8_1(W, x.shape[1], quantize_q8_1(x), nthreads)


def subblock_sums(W: np.ndarray, K: int, yq: np.ndarray):
    """Exact S (nibble.q8) and T (sum q8) per (col, row, sub-block): int32 (ncols, nrows, K/32)."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    yq = np.ascontiguousarray(yq, dtype=np.uint8)
    nrows, ncols = W.shape[0], yq.shape[0]
    S = np.empty((ncols, nrows, K // QK8_1), dtype=np.int32)
    T = np.empty_like(S)
    lib().or_subblock_sums(_ptr(W), nrows, K, W.shape[1] // Q4K_BYTES, _ptr(yq),
                           yq.shape[1] // Q81_BYTES, ncols, _ptr(S), _ptr(T))
    return S, T


def ref_gemv_q8_1(W: np.ndarray, K: int, yq: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """The reference's own vec_dot_q4_K_q8_1 in upstream MMVQ's summation order."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    yq = np.ascontiguousarray(yq, dtype=np.uint8)
    nrows, ncols = W.shape[0], yq.shape[0]
    out = np.empty((ncols, nrows), dtype=np.float32)
    ref_lib().ref_gemv_q4k_q8_1(_ptr(W), nrows, K, W.shape[1] // Q4K_BYTES, _ptr(yq),
                                yq.shape[1] // Q81_BYTES, ncols, _ptr(out), nrows, nthreads)
    return out


def ref_gemv_q6k_q8_1(W: np.ndarray, K: int, yq: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """The reference's own vec_dot_q6_K_q8_1 (kernels/vecdotq.cuh:867-890) in
    upstream MMVQ's summation order, over Q6_K rows (nrows, K/256*210)."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    yq = np.ascontiguousarray(yq, dtype=np.uint8)
    nrows, ncols = W.shape[0], yq.shape[0]
    out = np.empty((ncols, nrows), dtype=np.float32)
    ref_lib().ref_gemv_q6k_q8_1(_ptr(W), nrows, K, W.shape[1] // Q6K_BYTES, _ptr(yq),
                                yq.shape[1] // Q81_BYTES, ncols, _ptr(out), nrows, nthreads)
    return out


def ref_vec_dot_q6k(sb: np.ndarray, q8: np.ndarray, iqs: int) -> float:
    """Reference vec_dot_q6_K_q8_1 on one super-block (210 B) and its 8 q8_1 blocks."""
    sb = np.ascontiguousarray(sb, dtype=np.uint8)
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    return float(ref_lib().ref_vec_dot_q6_K_q8_1(_ptr(sb), _ptr(q8), 0, iqs))


def ref_vec_dot(sb: np.ndarray, q8: np.ndarray, iqs: int) -> float:
    """Reference vec_dot_q4_K_q8_1 on one super-block (144 B) and its 8 q8_1 blocks."""
    sb = np.ascontiguousarray(sb, dtype=np.uint8)
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    return float(ref_lib().ref_vec_dot_q4_K_q8_1(_ptr(sb), _ptr(q8), 0, iqs))


def h2f(h: int) -> float:
    return float(lib().or_h2f(h))


def f2h(f: float) -> int:
    return int(lib().or_f2h(f))


def max_threads() -> int:
    return int(lib().or_max_threads())

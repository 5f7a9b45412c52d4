"""Python front-end of libq4k_gemv.so, the sm_100a Q4_K x q8_1 decode GEMV.

The library's C ABI (include/q4k_gemv.h) is the drop-in boundary; this module
binds it with ctypes and uses torch only for device memory and streams.  The
function names follow the reference entry points they stand in for
(paths relative to the reference project):

  mul_mat_vec_q        ggml_cuda_mul_mat_vec_q       kernels/mmvq.cu:666-762
  mul_mat_vec_q8_1     mul_mat_vec_q_switch_type Q4_K kernels/mmvq.cu:479-593
  op_mul_mat_vec_q     ggml_cuda_op_mul_mat_vec_q    kernels/mmvq.cu:764-793
  quantize_row_q8_1    quantize_row_q8_1_cuda call   kernels/mmvq.cu:734
  custom_q4k_gemv      custom_q4k_gemv hook launch   kernels/mmvq.cu:10-18, :563-584

Tensor conventions: a Q4_K matrix is a uint8 tensor (nrows, K/256*144);
fp32 activations are (ncols, K) (column j = row j of the tensor, so the ggml
column stride is x.stride(0)); outputs are (ncols, nrows).  There is no CPU
fallback: every call goes to the CUDA library, which must be built
(`make -C gemv-q4_k-optimization_b200`) and fails loudly otherwise.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("Q4K_LIB", str(HERE / "libq4k_gemv.so")))  # Q4K_LIB: another build
HEADER_PATH = HERE.parent / "include" / "q4k_gemv.h"

QK_K = 256
BLOCK_BYTES = 144
QK8_1 = 32
Q8_1_BYTES = 36
ROW_PADDING = 512
MAX_NCOLS = 8
MAX_TASKS = 16

STATUS_NAMES = {0: "Q4K_OK", 1: "Q4K_EINVAL", 2: "Q4K_ECUDA", 3: "Q4K_ETIMEOUT", 4: "Q4K_ENCCL",
                5: "Q4K_EWORKSPACE"}


class Q4KError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


MAX_PEERS = 8


class Gather(ctypes.Structure):
    """struct q4k_gather (include/q4k_gemv.h)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("out_local", ctypes.c_void_p),
                ("out_peer", ctypes.c_void_p * MAX_PEERS), ("flags_peer", ctypes.c_void_p * MAX_PEERS),
                ("epoch", ctypes.c_void_p), ("out_elems", ctypes.c_int64)]


class Task(ctypes.Structure):
    """struct q4k_task (include/q4k_gemv.h)."""
    _fields_ = [("W", ctypes.c_void_p), ("x", ctypes.c_void_p), ("dst", ctypes.c_void_p),
                ("nrows", ctypes.c_int64), ("K", ctypes.c_int64), ("stride_row_x", ctypes.c_int64),
                ("stride_col_x", ctypes.c_int64), ("stride_col_dst", ctypes.c_int64)]


class TaskEx(ctypes.Structure):
    """struct q4k_task_ex (include/q4k_gemv.h): a task with an optional fused epilogue."""
    _fields_ = [("t", Task), ("W_gate", ctypes.c_void_p), ("x_bias", ctypes.c_void_p),
                ("gate_bias", ctypes.c_void_p), ("stride_col_bias", ctypes.c_int64), ("glu_op", ctypes.c_int),
                ("rms_norm", ctypes.c_int), ("norm_eps", ctypes.c_float), ("norm_weight", ctypes.c_void_p)]


# Q4K_GLU_* (include/q4k_gemv.h)
GLU_NONE, GLU_SWIGLU, GLU_GEGLU, GLU_SWIGLU_OAI, GLU_MUL = 0, 1, 2, 3, 4
GLU_OPS = {"none": GLU_NONE, "swiglu": GLU_SWIGLU, "geglu": GLU_GEGLU, "swiglu_oai": GLU_SWIGLU_OAI,
           "mul": GLU_MUL}

_lib = None
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_SZ = ctypes.c_size_t


def build() -> None:
    """Compile libq4k_gemv.so for sm_100a in-tree (nvcc cross-compiles without a GPU)."""
    import subprocess
    subprocess.run(["make", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build the CUDA library first "
                               f"(make -C {HERE})")
        L = ctypes.CDLL(str(LIB_PATH))
        TP, GP, TXP = ctypes.POINTER(Task), ctypes.POINTER(Gather), ctypes.POINTER(TaskEx)
        sigs = {  # name: (restype, argtypes); restype None = int status
            "q4k_status_string": (ctypes.c_char_p, [_I]),
            "q4k_last_error": (ctypes.c_char_p, []),
            "q4k_version": (_I, []),
            "q4k_device_supported": (_I, []),
            "q4k_row_bytes": (_SZ, [_I64]),
            "q4k_q8_1_bytes": (_SZ, [_I64, _I]),
            "q4k_gemv_workspace_bytes": (_SZ, [_I64, _I64, _I]),
            "q4k_batch_workspace_bytes": (_SZ, [TP, _I, _I]),
            "q4k_quantize_q8_1": (None, [_P, _I64, _I64, _I64, _I, _P, _P]),
            "q4k_mul_mat_vec_q8_1": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _SZ, _P]),
            "q4k_mul_mat_vec": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _SZ, _P]),
            "q4k_op_mul_mat_vec_q": (None, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
            "q4k_custom_q4k_gemv": (None, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
            "q4k_gemv_batch": (None, [TP, _I, _I, _P, _SZ, _P]),
            "q4k_debug_subblock_sums": (None, [_P, _P, _I64, _I64, _I, _I64, _I64, _P, _P, _P, _SZ, _P]),
            "q4k_workspace_status": (None, [_P, ctypes.POINTER(_I), _P]),
            "q4k_mul_mat_vec_noalloc": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P]),
            "q4k_noalloc_scratch_bytes": (_SZ, []),
            "q4k_sharded_workspace_bytes": (_SZ, [_I64, _I64, _I, _I]),
            "q4k_gemv_sharded": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _I, _I, _P, _SZ, _P]),
            "q4k_gemv_batch_allgather": (None, [TP, _I, _I, GP, _P, _SZ, _P]),
            "q4k_gather_wait": (None, [GP, _P, _SZ, _P]),
            "q4k_workspace_init": (None, [_P, _SZ, _P]),
            "q4k_gemv_batch_persistent": (None, [TP, _I, _I, GP, _P, _SZ, _P]),
            "q4k_batch_ex_workspace_bytes": (_SZ, [TXP, _I, _I]),
            "q4k_gemv_batch_ex": (None, [TXP, _I, _I, _P, _SZ, _P]),
            "q4k_gemv_fused_workspace_bytes": (_SZ, [_I64, _I64, _I]),
            "q4k_mul_mat_vec_q8_1_fused": (None, [_P, _P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _P, _I,
                                                  _P, _SZ, _P]),
            "q4k_mul_mat_vec_fused": (None, [_P, _P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _P, _I,
                                             _P, _SZ, _P]),
            "q4k_rms_norm_quantize_q8_1": (None, [_P, _I64, _I64, _I64, _I, _P, ctypes.c_float, _P, _P]),
            "q4k_q6_k_workspace_bytes": (_SZ, [_I64, _I64, _I]),
            "q4k_mul_mat_vec_q6_k": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _SZ, _P]),
            "q4k_mul_mat_vec_q6_k_q8_1": (None, [_P, _P, _P, _I64, _I64, _I, _I64, _I64, _I64, _P, _SZ, _P]),
            "q4k_batch_q6_k_workspace_bytes": (_SZ, [TP, _I, _I]),
            "q4k_gemv_batch_q6_k": (None, [TP, _I, _I, _P, _SZ, _P]),
            "q4k_ipc_alloc": (None, [_SZ, ctypes.POINTER(ctypes.c_void_p)]),
            "q4k_ipc_free": (None, [_P]),
            "q4k_ipc_handle": (None, [_P, ctypes.c_char_p]),
            "q4k_ipc_open": (None, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
            "q4k_ipc_close": (None, [_P]),
            "q4k_batch_ex_kernel": (_I, [TXP, _I, _I, _I]),
            "q4k_batch_persistent_kernel": (_I, [TP, _I, _I, _I]),
            "q4k_timeline_bytes": (_SZ, []),
            "q4k_timeline_read": (None, [_P, _SZ, ctypes.POINTER(_I)]),
            "q4k_timeline_reset": (None, []),
        }
        overridden = "Q4K_LIB" in os.environ
        for name, (res, args) in sigs.items():
            fn = getattr(L, name, None) if overridden else getattr(L, name)  # the in-tree build must have all
            if fn is None:
                continue
            fn.restype = res if res is not None else _I
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    """Entry points declared in include/q4k_gemv.h."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"^Q4K_API\s+[\w\s\*]*?\b(q4k_\w+)\s*\(", text, flags=re.M)))


def _check(status: int) -> None:
    if status != 0:
        msg = lib().q4k_last_error().decode(errors="replace")
        raise Q4KError(status, msg)


def _stream(stream) -> int:
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def kpad(K: int) -> int:
    return (K + ROW_PADDING - 1) // ROW_PADDING * ROW_PADDING


def row_bytes(K: int) -> int:
    return int(lib().q4k_row_bytes(K))


# ---------------------------------------------------------------------------
# workspace
# ---------------------------------------------------------------------------
class Workspace:
    """Device scratch owned by the caller (the library never allocates).

    Grows on demand; one Workspace must not serve two calls that can overlap
    on the GPU (e.g. on two streams)."""

    def __init__(self, nbytes: int = 0, device=None):
        import torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=self.device)
        self.zeroed = False  # control words zero (q4k_workspace_init ran on this buffer)

    def ensure(self, nbytes: int) -> "Workspace":
        import torch
        if nbytes > self.buf.numel():
            self.buf = torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)
            self.zeroed = False
        return self

    def init(self, stream=None) -> "Workspace":
        """Zero the whole buffer (q4k_workspace_init), as the single-launch path needs."""
        _check(lib().q4k_workspace_init(self.ptr, self.nbytes, _stream(stream)))
        self.zeroed = True
        return self

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    @property
    def nbytes(self) -> int:
        return self.buf.numel()

    def status(self, stream=None) -> int:
        v = ctypes.c_int(0)
        _check(lib().q4k_workspace_status(self.ptr, ctypes.byref(v), _stream(stream)))
        return v.value


_default_ws: dict = {}


def _ws_for(nbytes: int, ws: Workspace | None, device) -> Workspace:
    if ws is not None:
        return ws.ensure(nbytes)
    key = str(device)
    w = _default_ws.get(key)
    if w is None:
        w = _default_ws[key] = Workspace(nbytes, device)
    return w.ensure(nbytes)


def gemv_workspace_bytes(nrows: int, K: int, ncols: int) -> int:
    return int(lib().q4k_gemv_workspace_bytes(nrows, K, ncols))


# ---------------------------------------------------------------------------
# entry points
# ---------------------------------------------------------------------------
def quantize_row_q8_1(x, Kpad: int | None = None, out=None, stream=None):
    """fp32 (ncols, K) -> ggml q8_1 (ncols, Kpad/32*36) uint8 on the device."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    assert x.dtype == torch.float32 and x.is_cuda and x.stride(1) == 1
    ncols, K = x.shape
    Kp = kpad(K) if Kpad is None else int(Kpad)
    if out is None:
        out = torch.empty((ncols, Kp // QK8_1 * Q8_1_BYTES), dtype=torch.uint8, device=x.device)
    _check(lib().q4k_quantize_q8_1(x.data_ptr(), K, x.stride(0), Kp, ncols, out.data_ptr(), _stream(stream)))
    return out


def mul_mat_vec_q(W, x, out=None, ws: Workspace | None = None, stream=None):
    """y = W @ x with fp32 activations x (ncols, K); returns (ncols, nrows) fp32."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    assert W.dtype == torch.uint8 and W.is_cuda and x.is_cuda and x.dtype == torch.float32
    assert x.stride(1) == 1 and W.stride(1) == 1
    ncols, K = x.shape
    nrows = W.shape[0]
    if W.stride(0) % BLOCK_BYTES:
        raise Q4KError(1, "W row stride is not a whole number of super-blocks")
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=x.device)
    w = _ws_for(gemv_workspace_bytes(nrows, K, ncols), ws, x.device)
    _check(lib().q4k_mul_mat_vec(W.data_ptr(), x.data_ptr(), out.data_ptr(), K, nrows, ncols,
                                 W.stride(0) // BLOCK_BYTES, x.stride(0), out.stride(0),
                                 w.ptr, w.nbytes, _stream(stream)))
    return out


def mul_mat_vec_q_noalloc(W, x, out=None, stream=None):
    """mul_mat_vec_q for callers that cannot allocate device scratch: the library
    uses its own built-in array (q4k_noalloc_scratch_bytes(); shared by all such
    calls on a device, so calls that may overlap on the GPU race)."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    ncols, K = x.shape
    nrows = W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=x.device)
    _check(lib().q4k_mul_mat_vec_noalloc(W.data_ptr(), x.data_ptr(), out.data_ptr(), K, nrows, ncols,
                                         W.stride(0) // BLOCK_BYTES, x.stride(0), out.stride(0), _stream(stream)))
    return out


def sharded_workspace_bytes(nrows: int, K: int, ncols: int, world: int) -> int:
    return int(lib().q4k_sharded_workspace_bytes(nrows, K, ncols, world))


def gemv_sharded(W_shard, x, nrows: int, nccl_comm: int, rank: int, world: int, out=None,
                 ws: Workspace | None = None, stream=None):
    """Row-sharded y = W @ x gathered over an NCCL communicator (its ncclComm_t
    as an integer): this rank's rows W_shard (shard_rows(nrows, rank, world)),
    the same fp32 x (ncols, K) on every rank; returns all (ncols, nrows) rows."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    assert x.is_cuda and x.dtype == torch.float32 and x.stride(1) == 1
    ncols, K = x.shape
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=x.device)
    w = _ws_for(sharded_workspace_bytes(nrows, K, ncols, world), ws, x.device)
    wptr = W_shard.data_ptr() if W_shard is not None and W_shard.numel() else None
    rs = W_shard.stride(0) // BLOCK_BYTES if W_shard is not None and W_shard.dim() == 2 else K // QK_K
    _check(lib().q4k_gemv_sharded(wptr, x.data_ptr(), out.data_ptr(), K, nrows, ncols, rs, x.stride(0),
                                  out.stride(0), nccl_comm, rank, world, w.ptr, w.nbytes, _stream(stream)))
    return out


def mul_mat_vec_q8_1(W, yq, K: int, out=None, ws: Workspace | None = None, stream=None):
    """y = W @ q8_1 activations yq (ncols, blocks*36 uint8); returns (ncols, nrows)."""
    import torch
    if yq.dim() == 1:
        yq = yq.unsqueeze(0)
    ncols = yq.shape[0]
    nrows = W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=W.device)
    w = _ws_for(gemv_workspace_bytes(nrows, K, ncols), ws, W.device)
    _check(lib().q4k_mul_mat_vec_q8_1(W.data_ptr(), yq.data_ptr(), out.data_ptr(), K, nrows, ncols,
                                      W.stride(0) // BLOCK_BYTES, yq.stride(0) // Q8_1_BYTES, out.stride(0),
                                      w.ptr, w.nbytes, _stream(stream)))
    return out


def op_mul_mat_vec_q(W_slice, K: int, yq, row_low: int, row_high: int, src1_padded_row_size: int,
                     out=None, nrows_dst: int | None = None, ws: Workspace | None = None, stream=None):
    """Row-split slice: rows [row_low, row_high) of the matrix, src1 pre-quantized."""
    import torch
    ncols = yq.shape[0]
    rows = row_high - row_low
    nd = rows if nrows_dst is None else nrows_dst
    if out is None:
        out = torch.empty((ncols, nd), dtype=torch.float32, device=W_slice.device)
    w = _ws_for(gemv_workspace_bytes(rows, K, ncols), ws, W_slice.device)
    _check(lib().q4k_op_mul_mat_vec_q(W_slice.data_ptr(), K, yq.data_ptr(), out.data_ptr(), row_low, row_high,
                                      ncols, src1_padded_row_size, nd, w.ptr, w.nbytes, _stream(stream)))
    return out


def custom_q4k_gemv(vx, vy, dst, num_blocks_total: int, stride_col_y_blocks: int, stride_col_dst: int,
                    ncols_dst: int, ws: Workspace | None = None, stream=None):
    """The reference hook's 6-argument launch contract (+ ncols and workspace)."""
    w = _ws_for(gemv_workspace_bytes(stride_col_dst, num_blocks_total * QK_K, ncols_dst), ws, dst.device)
    _check(lib().q4k_custom_q4k_gemv(vx.data_ptr(), vy.data_ptr(), dst.data_ptr(), num_blocks_total,
                                     stride_col_y_blocks, stride_col_dst, ncols_dst, w.ptr, w.nbytes,
                                     _stream(stream)))
    return dst


def make_tasks(mats: Sequence, xs: Sequence, outs: Sequence):
    """ctypes task array for gemv_batch from (W, x, out) tensor triples."""
    n = len(mats)
    arr = (Task * n)()
    for i, (W, x, o) in enumerate(zip(mats, xs, outs)):
        if x.dim() == 1:
            x = x.unsqueeze(0)
        arr[i].W = W.data_ptr()
        arr[i].x = x.data_ptr()
        arr[i].dst = o.data_ptr()
        arr[i].nrows = W.shape[0]
        arr[i].K = x.shape[1]
        arr[i].stride_row_x = W.stride(0) // BLOCK_BYTES
        arr[i].stride_col_x = x.stride(0)
        arr[i].stride_col_dst = o.stride(0) if o.dim() > 1 else W.shape[0]
    return arr


def batch_workspace_bytes(tasks, ncols: int) -> int:
    return int(lib().q4k_batch_workspace_bytes(tasks, len(tasks), ncols))


def _sized_call(fn, tasks, ncols: int, ws: Workspace, stream, size_fn) -> None:
    """Call a batch entry with the workspace as it is; only when the library
    answers Q4K_EWORKSPACE is the size asked for, the buffer grown and the call
    repeated (what a refused call did, zeroing the outputs of K = 0 tasks, is
    idempotent), so steady-state calls pay one library call, not two."""
    s = _stream(stream)
    st = fn(tasks, len(tasks), ncols, ws.ptr, ws.nbytes, s)
    if st == 5:
        need = int(size_fn(tasks, len(tasks), ncols))
        if need > ws.nbytes:
            ws.ensure(need)
            st = fn(tasks, len(tasks), ncols, ws.ptr, ws.nbytes, s)
    _check(st)


def gemv_batch(tasks, ncols: int, ws: Workspace, stream=None) -> None:
    """Every task's GEMV in one prep + one persistent GEMV launch."""
    L = lib()
    _sized_call(L.q4k_gemv_batch, tasks, ncols, ws, stream, L.q4k_batch_workspace_bytes)


def _ptr_or_none(t):
    return None if t is None else t.data_ptr()


def make_tasks_ex(items):
    """ctypes q4k_task_ex array from dicts with keys W, x, out and optionally
    W_gate, x_bias, gate_bias (tensors; biases (ncols, nrows) or (nrows,)) and
    glu ("swiglu", "geglu", "swiglu_oai", "mul" or "none"), and rms_norm (bool), norm_eps,
    norm_weight (K fp32) for RMSNorm of x inside the quantization launch."""
    arr = (TaskEx * len(items))()
    for i, it in enumerate(items):
        base = make_tasks([it["W"]], [it["x"]], [it["out"]])[0]
        arr[i].t = base
        arr[i].W_gate = _ptr_or_none(it.get("W_gate"))
        xb, gb = it.get("x_bias"), it.get("gate_bias")
        arr[i].x_bias = _ptr_or_none(xb)
        arr[i].gate_bias = _ptr_or_none(gb)
        b = xb if xb is not None else gb
        arr[i].stride_col_bias = b.stride(0) if (b is not None and b.dim() > 1) else 0
        arr[i].glu_op = GLU_OPS[it.get("glu", "swiglu" if it.get("W_gate") is not None else "none")]
        if it.get("rms_norm"):
            arr[i].rms_norm = 1
            arr[i].norm_eps = float(it.get("norm_eps", 1e-5))
            arr[i].norm_weight = _ptr_or_none(it.get("norm_weight"))
    return arr


def rms_norm_quantize_q8_1(x, norm_weight=None, eps: float = 1e-5, Kpad: int | None = None, stream=None):
    """ggml q8_1 blocks of RMSNorm(x) * norm_weight: (ncols, Kpad/32*36) uint8 (one launch)."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    ncols, K = x.shape
    Kp = kpad(K) if Kpad is None else Kpad
    y = torch.zeros((ncols, Kp // QK8_1 * Q8_1_BYTES), dtype=torch.uint8, device=x.device)
    _check(lib().q4k_rms_norm_quantize_q8_1(x.data_ptr(), K, x.stride(0), Kp, ncols, _ptr_or_none(norm_weight),
                                            eps, y.data_ptr(), _stream(stream)))
    return y


def batch_ex_workspace_bytes(tasks, ncols: int) -> int:
    return int(lib().q4k_batch_ex_workspace_bytes(tasks, len(tasks), ncols))


KERNEL_NAMES = {0: "k_gemv", 2: "k_gemv (epilogue)", 3: "k_gemv (two rows per lane)", 5: "k_gemv_dyn",
                6: "k_gemv_dyn (epilogue)", 7: "k_gemv (single launch)",
                8: "k_gemv (two rows per lane, int8 MMA)"}


def batch_kernel(tasks, ncols: int, num_sms: int | None = None) -> str:
    """Name of the GEMV kernel a batch call with these tasks (q4k_task or
    q4k_task_ex array) runs on a device with num_sms SMs (default: the
    current device's); touches no device memory."""
    if num_sms is None:
        import torch
        num_sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    if len(tasks) and isinstance(tasks[0], Task):
        ex = (TaskEx * len(tasks))()
        for i, t in enumerate(tasks):
            ex[i].t = t
        tasks = ex
    k = int(lib().q4k_batch_ex_kernel(tasks, len(tasks), ncols, num_sms))
    if k < 0:
        _check(1)
    return KERNEL_NAMES.get(k, str(k))


def batch_persistent_kernel(tasks, ncols: int, num_sms: int | None = None) -> str:
    """Name of the GEMV kernel gemv_batch_persistent runs for these q4k_task
    tasks: "k_gemv (single launch)", or its two-launch fallback's kernel."""
    if num_sms is None:
        import torch
        num_sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    k = int(lib().q4k_batch_persistent_kernel(tasks, len(tasks), ncols, num_sms))
    if k < 0:
        _check(1)
    return KERNEL_NAMES.get(k, str(k))


def gemv_batch_ex(tasks, ncols: int, ws: Workspace, stream=None) -> None:
    """Batched launch of tasks with optional fused bias/gate epilogues."""
    L = lib()
    _sized_call(L.q4k_gemv_batch_ex, tasks, ncols, ws, stream, L.q4k_batch_ex_workspace_bytes)


def mul_mat_vec_fused(W, W_gate, x, glu: str = "swiglu", x_bias=None, gate_bias=None, out=None,
                      ws: Workspace | None = None, stream=None):
    """glu(W.x + x_bias, W_gate.x + gate_bias) through q4k_mul_mat_vec_fused.
    x: (ncols, K) fp32; biases: (ncols, nrows) with the output's column stride, or None."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    ncols, K = x.shape
    nrows = W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=x.device)
    for b in (x_bias, gate_bias):
        if b is not None and ncols > 1:
            assert b.stride(0) == out.stride(0), "bias column stride must equal the output's"
    w = _ws_for(int(lib().q4k_gemv_fused_workspace_bytes(nrows, K, ncols)), ws, x.device)
    _check(lib().q4k_mul_mat_vec_fused(W.data_ptr(), _ptr_or_none(W_gate), x.data_ptr(), out.data_ptr(), K, nrows,
                                       ncols, W.stride(0) // BLOCK_BYTES, x.stride(0), out.stride(0),
                                       _ptr_or_none(x_bias), _ptr_or_none(gate_bias), GLU_OPS[glu],
                                       w.ptr, w.nbytes, _stream(stream)))
    return out


def mul_mat_vec_q8_1_fused(W, W_gate, yq, K: int, glu: str = "swiglu", x_bias=None, gate_bias=None, out=None,
                           ws: Workspace | None = None, stream=None):
    """The q8_1-input fused entry (q4k_mul_mat_vec_q8_1_fused).  yq: (ncols, Kpad/32*36) uint8."""
    import torch
    ncols, nrows = yq.shape[0], W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=yq.device)
    w = _ws_for(int(lib().q4k_gemv_fused_workspace_bytes(nrows, K, ncols)), ws, yq.device)
    _check(lib().q4k_mul_mat_vec_q8_1_fused(W.data_ptr(), _ptr_or_none(W_gate), yq.data_ptr(), out.data_ptr(), K,
                                            nrows, ncols, W.stride(0) // BLOCK_BYTES, yq.stride(0) // Q8_1_BYTES,
                                            out.stride(0), _ptr_or_none(x_bias), _ptr_or_none(gate_bias),
                                            GLU_OPS[glu], w.ptr, w.nbytes, _stream(stream)))
    return out


def gemv_batch_persistent(tasks, ncols: int, ws: Workspace, stream=None, gather=None) -> None:
    """q4k_gemv_batch in a single launch (each CTA quantizes its activations
    into shared memory) where the tasks allow it, else the two-launch sequence.

    ws is zeroed on first use (and whenever it grows); afterwards every
    completed call leaves its control words zero.  gather: a PeerGather for
    the fused all-gather, or None."""
    ws.ensure(batch_workspace_bytes(tasks, ncols))
    if not ws.zeroed:
        ws.init(stream)
    g = ctypes.byref(gather.desc) if gather is not None else None
    _check(lib().q4k_gemv_batch_persistent(tasks, len(tasks), ncols, g, ws.ptr, ws.nbytes, _stream(stream)))


def debug_subblock_sums(W, yq, K: int, ws: Workspace | None = None, stream=None):
    """Exact (S, T) as the kernels form them: S (ncols, nrows, K/32), T (ncols, K/32) int32."""
    import torch
    ncols, nrows = yq.shape[0], W.shape[0]
    S = torch.empty((ncols, nrows, K // QK8_1), dtype=torch.int32, device=W.device)
    T = torch.empty((ncols, K // QK8_1), dtype=torch.int32, device=W.device)
    w = _ws_for(gemv_workspace_bytes(nrows, K, ncols), ws, W.device)
    _check(lib().q4k_debug_subblock_sums(W.data_ptr(), yq.data_ptr(), K, nrows, ncols,
                                         W.stride(0) // BLOCK_BYTES, yq.stride(0) // Q8_1_BYTES,
                                         S.data_ptr(), T.data_ptr(), w.ptr, w.nbytes, _stream(stream)))
    return S, T


# ---------------------------------------------------------------------------
# synthetic data with the benchmark's value distributions
# ---------------------------------------------------------------------------
Q6K_BYTES = 210


def mul_mat_vec_q6_k(W, x, out=None, ws: Workspace | None = None, stream=None):
    """y = W @ x for Q6_K rows W (nrows, K/256*210) uint8 and fp32 x (ncols, K)."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    ncols, K = x.shape
    nrows = W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=x.device)
    w = _ws_for(int(lib().q4k_q6_k_workspace_bytes(nrows, K, ncols)), ws, x.device)
    _check(lib().q4k_mul_mat_vec_q6_k(W.data_ptr(), x.data_ptr(), out.data_ptr(), K, nrows, ncols,
                                      W.stride(0) // Q6K_BYTES, x.stride(0), out.stride(0), w.ptr, w.nbytes,
                                      _stream(stream)))
    return out


def mul_mat_vec_q6_k_q8_1(W, yq, K: int, out=None, ws: Workspace | None = None, stream=None):
    """The q8_1-input Q6_K entry.  yq: (ncols, Kpad/32*36) uint8."""
    import torch
    ncols, nrows = yq.shape[0], W.shape[0]
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=yq.device)
    w = _ws_for(int(lib().q4k_q6_k_workspace_bytes(nrows, K, ncols)), ws, yq.device)
    _check(lib().q4k_mul_mat_vec_q6_k_q8_1(W.data_ptr(), yq.data_ptr(), out.data_ptr(), K, nrows, ncols,
                                           W.stride(0) // Q6K_BYTES, yq.stride(0) // Q8_1_BYTES, out.stride(0),
                                           w.ptr, w.nbytes, _stream(stream)))
    return out


def make_tasks_q6_k(mats: Sequence, xs: Sequence, outs: Sequence):
    """Task array for gemv_batch_q6_k (W: Q6_K rows)."""
    arr = make_tasks(mats, xs, outs)
    for i, W in enumerate(mats):
        arr[i].stride_row_x = W.stride(0) // Q6K_BYTES
    return arr


def gemv_batch_q6_k(tasks, ncols: int, ws: Workspace, stream=None) -> None:
    L = lib()
    _sized_call(L.q4k_gemv_batch_q6_k, tasks, ncols, ws, stream, L.q4k_batch_q6_k_workspace_bytes)


def gen_q6k_numpy(rng: np.random.Generator, nrows: int, K: int) -> np.ndarray:
    """Q6_K matrix (nrows, K/256*210) uint8: d = fp16(|N(0,1)|*0.01), int8 scales and the
    6-bit quants uniform."""
    nb = K // QK_K
    W = rng.integers(0, 256, size=(nrows, nb, Q6K_BYTES), dtype=np.uint8)
    d = (np.abs(rng.standard_normal((nrows, nb))) * 0.01).astype(np.float16)
    W[:, :, 208:210] = d.view(np.uint8).reshape(nrows, nb, 2)
    return W.reshape(nrows, nb * Q6K_BYTES)


def gen_q6k_torch(nrows: int, K: int, generator=None, device="cuda"):
    """Same distributions as gen_q6k_numpy, generated on the device."""
    import torch
    nb = K // QK_K
    W = torch.randint(0, 256, (nrows, nb, Q6K_BYTES), dtype=torch.uint8, device=device, generator=generator)
    d = (torch.randn((nrows, nb), device=device, generator=generator).abs_() * 0.01).to(torch.float16)
    W[:, :, 208:210] = d.view(torch.uint8).reshape(nrows, nb, 2)
    return W.view(nrows, nb * Q6K_BYTES)


def gen_q4k_numpy(rng: np.random.Generator, nrows: int, K: int) -> np.ndarray:
    """Q4_K matrix (nrows, K/256*144) uint8: d, dmin = fp16(|N(0,1)|*0.01); scale/min
    bytes uniform (so every 6-bit scale and min is uniform on 0..63); nibbles uniform."""
    nb = K // QK_K
    W = rng.integers(0, 256, size=(nrows, nb, BLOCK_BYTES), dtype=np.uint8)
    d = (np.abs(rng.standard_normal((nrows, nb, 2))) * 0.01).astype(np.float16)
    W[:, :, 0:4] = d.view(np.uint8).reshape(nrows, nb, 4)
    return W.reshape(nrows, nb * BLOCK_BYTES)


def gen_q4k_torch(nrows: int, K: int, generator=None, device="cuda"):
    """Same distributions as gen_q4k_numpy, generated on the device (large matrices)."""
    import torch
    nb = K // QK_K
    W = torch.randint(0, 256, (nrows, nb, BLOCK_BYTES), dtype=torch.uint8, device=device, generator=generator)
    d = (torch.randn((nrows, nb, 2), device=device, generator=generator).abs_() * 0.01).to(torch.float16)
    W[:, :, 0:4] = d.view(torch.uint8).reshape(nrows, nb, 4)
    return W.view(nrows, nb * BLOCK_BYTES)


# ---------------------------------------------------------------------------
# row-sharded multi-GPU (one process per GPU)
# ---------------------------------------------------------------------------
def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int, int]:
    """Contiguous ceil-split rows [lo, hi) of rank, and the per-rank capacity.

    The reference's row split gives each device a contiguous row range
    (kernels/mmvq.cu:764-793); trailing ranks may get fewer (or no) rows."""
    per = (rows + world - 1) // world
    lo = min(rows, rank * per)
    return lo, min(rows, lo + per), per


class DeviceBuffer:
    """A torch view of device memory the library allocated (for IPC)."""

    def __init__(self, ptr: int, nbytes: int, device):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device = device

    def tensor(self):
        import torch
        return torch.as_tensor(self, device=self.device)


class PeerGather:
    """Full-output buffers shared by all ranks for q4k_gemv_batch_allgather.

    Collective over the default torch.distributed group: every rank allocates
    `out_elems` fp32 outputs + its flag words + its epoch word with
    q4k_ipc_alloc, the 64-byte IPC handles are exchanged with all_gather_object,
    and every peer's buffers are mapped with q4k_ipc_open.  `out` is this rank's
    full output as a float32 tensor; outputs of this rank's shard of a matrix
    go at its own row offset inside it, and every launch fills all rows."""

    def __init__(self, out_elems: int):
        import torch
        import torch.distributed as dist
        L = lib()
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        if self.world > MAX_PEERS:
            raise Q4KError(1, f"world size {self.world} > {MAX_PEERS}")
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._own = []
        self._opened = []

        def alloc(nbytes):
            p = ctypes.c_void_p()
            _check(L.q4k_ipc_alloc(nbytes, ctypes.byref(p)))
            self._own.append(p.value)
            return p.value

        out_bytes = (out_elems * 4 + 255) // 256 * 256
        out_ptr = alloc(out_bytes)
        flags_ptr = alloc(256)
        epoch_ptr = alloc(256)

        def handle(ptr):
            h = ctypes.create_string_buffer(64)
            _check(L.q4k_ipc_handle(ptr, h))
            return h.raw

        mine = (handle(out_ptr), handle(flags_ptr))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine)
        g = Gather()
        g.world, g.rank = self.world, self.rank
        g.out_local = out_ptr
        g.out_elems = out_elems
        g.epoch = epoch_ptr
        for q in range(self.world):
            if q == self.rank:
                g.out_peer[q], g.flags_peer[q] = out_ptr, flags_ptr
                continue
            ptrs = []
            for h in allh[q]:
                p = ctypes.c_void_p()
                _check(L.q4k_ipc_open(h, ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
            g.out_peer[q], g.flags_peer[q] = ptrs
        self.desc = g
        self.out = DeviceBuffer(out_ptr, out_elems * 4, self.device).tensor().view(torch.float32)
        dist.barrier()

    def close(self):
        """Unmap the peers' buffers, wait until every rank has done the same
        (collective), then free this rank's own buffers: no rank frees memory
        that another still has mapped."""
        import torch.distributed as dist
        L = lib()
        for p in self._opened:
            L.q4k_ipc_close(p)
        self._opened = []
        if dist.is_initialized():
            dist.barrier()
        for p in self._own:
            L.q4k_ipc_free(p)
        self._own = []


def gemv_batch_allgather(tasks, ncols: int, gather: PeerGather, ws: Workspace, stream=None) -> None:
    """q4k_gemv_batch on this rank's row shards, outputs gathered into every rank's buffer
    (complete once gather_wait has run on the stream)."""
    ws.ensure(batch_workspace_bytes(tasks, ncols))
    _check(lib().q4k_gemv_batch_allgather(tasks, len(tasks), ncols, ctypes.byref(gather.desc), ws.ptr, ws.nbytes,
                                          _stream(stream)))


def gather_wait(gather: PeerGather, ws: Workspace, stream=None) -> None:
    """q4k_gather_wait: the peers' rows of the last gathering call are in this rank's buffer
    once this stream-ordered wait has run (a wait that gives up sets the status word)."""
    _check(lib().q4k_gather_wait(ctypes.byref(gather.desc), ws.ptr, ws.nbytes, _stream(stream)))


# ---------------------------------------------------------------------------
# launch timeline (diagnostic library built with -DQ4K_TIMELINE=1)
# ---------------------------------------------------------------------------
TIMELINE_LIB = HERE / "libq4k_gemv_timeline.so"  # load it with Q4K_LIB=<this path>
TL_SLOTS, TL_CTAS, TL_PREP_CTAS = 64, 256, 4096  # Q4K_TIMELINE_* in include/q4k_gemv.h


def timeline_reset() -> None:
    _check(lib().q4k_timeline_reset())


def timeline_read():
    """(gemv, prep, ncalls) from a timeline build: gemv u64[slot][CTA][warp][8]
    = {start, wait return, end, atoms, SM, worker, first atom, end atom} and
    prep u64[slot][CTA][4] = {start, wait return, end, 1}, in %globaltimer ns;
    slot = call index since the last reset, modulo TL_SLOTS."""
    L = lib()
    nb = int(L.q4k_timeline_bytes())
    if nb == 0:
        raise Q4KError(1, f"{LIB_PATH.name} is built without Q4K_TIMELINE (set Q4K_LIB={TIMELINE_LIB})")
    buf = np.zeros(nb // 8, np.uint64)
    n = ctypes.c_int(0)
    _check(L.q4k_timeline_read(buf.ctypes.data, nb, ctypes.byref(n)))
    ng = TL_SLOTS * TL_CTAS * 16 * 8
    return (buf[:ng].reshape(TL_SLOTS, TL_CTAS, 16, 8).astype(np.int64),
            buf[ng:].reshape(TL_SLOTS, TL_PREP_CTAS, 4).astype(np.int64), n.value)

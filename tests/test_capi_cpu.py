"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, sizes buffers, and rejects bad arguments with Q4K_EINVAL
before touching a device."""
from __future__ import annotations

import ctypes
import subprocess

import pytest

EINVAL, EWORKSPACE = 1, 5


def test_library_loads_and_exports_header_symbols(q4k):
    L = q4k.lib()
    declared = q4k.declared_symbols()
    assert len(declared) >= 16
    for name in declared:
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(q4k.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported
    # nothing else of the library's internals leaks out
    assert all(e.startswith("q4k_") for e in exported)


def test_sizes(q4k):
    L = q4k.lib()
    assert L.q4k_row_bytes(4096) == 16 * 144
    assert L.q4k_row_bytes(100) == 0
    assert L.q4k_q8_1_bytes(4608, 3) == 4608 // 32 * 36 * 3
    ws1 = q4k.gemv_workspace_bytes(4096, 4096, 1)
    ws8 = q4k.gemv_workspace_bytes(4096, 4096, 8)
    assert 0 < ws1 < ws8
    assert ws8 >= 8 * 16 * 320  # the activation pack
    assert L.q4k_version() >= 100
    assert L.q4k_status_string(1) == b"Q4K_EINVAL"


def _call(L, W=256, x=512, dst=1024, K=4096, nrows=8, ncols=1, srx=None, scx=None, scd=None, ws=4096,
          wsb=1 << 30):
    srx = K // 256 if srx is None else srx
    scx = K if scx is None else scx
    scd = nrows if scd is None else scd
    return L.q4k_mul_mat_vec(W, x, dst, K, nrows, ncols, srx, scx, scd, ws, wsb, None)


@pytest.mark.parametrize("kw", [
    dict(K=100), dict(K=-256), dict(ncols=0), dict(ncols=9), dict(nrows=-1),
    dict(W=258), dict(W=0), dict(x=0), dict(dst=0), dict(srx=15),
    dict(ncols=2, scx=4000), dict(ncols=2, scd=4),
])
def test_invalid_arguments_rejected_without_gpu(q4k, kw):
    L = q4k.lib()
    assert _call(L, **kw) == EINVAL
    assert len(L.q4k_last_error()) > 0


def test_workspace_checks(q4k):
    L = q4k.lib()
    # size and alignment are checked after the device is known; without a GPU the
    # call reports the CUDA failure instead, never a crash
    st = _call(L, ws=0)
    assert st in (EWORKSPACE, 2)


def test_batch_rejects_bad_task_count(q4k):
    L = q4k.lib()
    tasks = (q4k.Task * 17)()
    assert L.q4k_gemv_batch(tasks, 17, 1, None, 0, None) == EINVAL
    assert L.q4k_gemv_batch(tasks, 0, 1, None, 0, None) == EINVAL


def test_quantize_rejects_bad_padding(q4k):
    L = q4k.lib()
    assert L.q4k_quantize_q8_1(256, 100, 100, 96, 1, 512, None) == EINVAL   # Kpad < K
    assert L.q4k_quantize_q8_1(256, 100, 100, 120, 1, 512, None) == EINVAL  # Kpad % 32
    assert L.q4k_quantize_q8_1(256, 100, 100, 128, 9, 512, None) == EINVAL  # ncols


def test_op_mul_mat_vec_q_rejects_bad_rows(q4k):
    L = q4k.lib()
    assert L.q4k_op_mul_mat_vec_q(256, 4096, 512, 1024, 10, 5, 1, 4096, 16, None, 0, None) == EINVAL
    assert L.q4k_op_mul_mat_vec_q(256, 4096, 512, 1024, 0, 32, 1, 4096, 16, None, 0, None) == EINVAL
    assert L.q4k_op_mul_mat_vec_q(256, 4096, 512, 1024, 0, 8, 1, 4000, 16, None, 0, None) == EINVAL


def test_persistent_path_argument_checks(q4k):
    L = q4k.lib()
    tasks = (q4k.Task * 17)()
    assert L.q4k_gemv_batch_persistent(tasks, 17, 1, None, None, 0, None) == EINVAL
    assert L.q4k_gemv_batch_persistent(None, 1, 1, None, None, 0, None) == EINVAL
    t = (q4k.Task * 1)()
    t[0].W, t[0].x, t[0].dst, t[0].nrows, t[0].K, t[0].stride_row_x = 256, 512, 1024, 32, 300, 2
    assert L.q4k_gemv_batch_persistent(t, 1, 1, None, None, 0, None) == EINVAL  # K % 256
    g = q4k.Gather()
    g.world = 9
    t[0].K = 256
    assert L.q4k_gemv_batch_persistent(t, 1, 1, ctypes.byref(g), None, 0, None) == EINVAL
    assert L.q4k_workspace_init(None, 256, None) == EWORKSPACE
    assert L.q4k_workspace_init(4097, 256, None) == EWORKSPACE  # not 16-byte aligned


def test_fused_epilogue_argument_checks(q4k):
    L = q4k.lib()
    # glu op without a gate, gate without an op, gate_bias without a gate, bad op: all rejected before the GPU
    assert L.q4k_mul_mat_vec_fused(256, None, 512, 1024, 256, 32, 1, 1, 256, 32, None, None, 1, None, 0,
                                   None) == EINVAL
    assert L.q4k_mul_mat_vec_fused(256, 768, 512, 1024, 256, 32, 1, 1, 256, 32, None, None, 0, None, 0,
                                   None) == EINVAL
    assert L.q4k_mul_mat_vec_fused(256, None, 512, 1024, 256, 32, 1, 1, 256, 32, None, 2048, 0, None, 0,
                                   None) == EINVAL
    assert L.q4k_mul_mat_vec_fused(256, 768, 512, 1024, 256, 32, 1, 1, 256, 32, None, None, 9, None, 0,
                                   None) == EINVAL
    assert L.q4k_mul_mat_vec_fused(256, 776, 512, 1024, 256, 32, 1, 1, 256, 32, None, None, 1, None, 0,
                                   None) == EINVAL  # gate not 16-byte aligned
    assert L.q4k_mul_mat_vec_fused(256, 768, 512, 1024, 0, 32, 1, 0, 0, 32, None, None, 1, None, 0,
                                   None) == EINVAL  # K = 0 with a fused epilogue
    assert "glu_op" in L.q4k_last_error().decode() or "K > 0" in L.q4k_last_error().decode()
    # the fused launch keeps two partial slots (main and gate sums) per CTA:
    # counters of its 448 row groups plus 2 x 256 (the SM bound) x 2 x 32 floats
    assert q4k.lib().q4k_gemv_fused_workspace_bytes(14336, 4096, 1) >= 448 * 4 + 2 * 256 * 2 * 32 * 4


def test_rms_norm_quantize_argument_checks(q4k):
    L = q4k.lib()
    assert L.q4k_rms_norm_quantize_q8_1(256, 0, 0, 32, 1, None, 1e-5, 512, None) == EINVAL       # K = 0
    assert L.q4k_rms_norm_quantize_q8_1(256, 100, 100, 96, 1, None, 1e-5, 512, None) == EINVAL   # Kpad < K
    assert L.q4k_rms_norm_quantize_q8_1(256, 64, 64, 64, 9, None, 1e-5, 512, None) == EINVAL     # ncols
    assert L.q4k_rms_norm_quantize_q8_1(256, 64, 64, 64, 1, None, -1.0, 512, None) == EINVAL     # eps
    assert L.q4k_rms_norm_quantize_q8_1(None, 64, 64, 64, 1, None, 1e-5, 512, None) == EINVAL    # null x


def test_q6k_argument_checks(q4k):
    L = q4k.lib()
    # K not a multiple of 2048, row stride not a multiple of 8 super-blocks
    assert L.q4k_mul_mat_vec_q6_k(256, 512, 1024, 1024, 8, 1, 4, 1024, 8, None, 0, None) == EINVAL
    assert L.q4k_mul_mat_vec_q6_k(256, 512, 1024, 2048, 8, 1, 9, 2048, 8, None, 0, None) == EINVAL
    assert "2048" in L.q4k_last_error().decode() or "% 8" in L.q4k_last_error().decode()
    assert q4k.lib().q4k_q6_k_workspace_bytes(32000, 4096, 1) > 0


def test_timeline_entry_points(q4k):
    """The product library carries the timeline API but no stamps; the
    diagnostic build (make timeline) sizes its record ring."""
    L = q4k.lib()
    assert L.q4k_timeline_bytes() == 0
    n = ctypes.c_int(-1)
    buf = ctypes.create_string_buffer(64)
    assert L.q4k_timeline_read(buf, 64, ctypes.byref(n)) == EINVAL
    assert L.q4k_timeline_reset() == EINVAL
    tl_path = q4k.TIMELINE_LIB
    if not tl_path.exists():
        pytest.skip("timeline library not built")
    T = ctypes.CDLL(str(tl_path))
    T.q4k_timeline_bytes.restype = ctypes.c_size_t
    want = (q4k.TL_SLOTS * q4k.TL_CTAS * 16 * 8 + q4k.TL_SLOTS * q4k.TL_PREP_CTAS * 4) * 8
    assert T.q4k_timeline_bytes() == want
    T.q4k_timeline_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int)]
    assert T.q4k_timeline_read(None, 8, ctypes.byref(n)) == EINVAL  # null destination


def _tasks_ex(q4k, specs):
    """TaskEx array from (rows, K, x_id, gated) with made-up aligned addresses
    (the kernel-choice query reads shapes only)."""
    arr = (q4k.TaskEx * len(specs))()
    base = 1 << 32
    for i, (rows, K, x_id, gated) in enumerate(specs):
        t = arr[i].t
        t.W, t.x, t.dst = base * (i + 1), base * (100 + x_id), base * (200 + i)
        t.nrows, t.K, t.stride_row_x, t.stride_col_x, t.stride_col_dst = rows, K, K // 256, K, rows
        if gated:
            arr[i].W_gate = base * (300 + i)
            arr[i].glu_op = q4k.GLU_SWIGLU
    return arr


MISTRAL_SPECS = [(4096, 4096, 0, False), (1024, 4096, 0, False), (1024, 4096, 0, False), (4096, 4096, 1, False),
                 (14336, 4096, 2, False), (14336, 4096, 2, False), (4096, 14336, 3, False)]


@pytest.mark.parametrize("specs,ncols,want", [
    (MISTRAL_SPECS, 1, "k_gemv"),                              # a whole layer: long static streams
    (MISTRAL_SPECS, 3, "k_gemv (two rows per lane)"),
    ([(14336, 4096, 0, False)], 1, "k_gemv_dyn"),             # one matrix, spread thinly: dynamic
    ([(14336, 4096, 0, False)], 2, "k_gemv_dyn"),
    ([(14336, 4096, 0, False)], 4, "k_gemv (two rows per lane, int8 MMA)"),
    ([(4096, 4096, 0, False)], 1, "k_gemv"),                  # too few row groups for the queue
    ([(14336, 4096, 0, True)], 1, "k_gemv (epilogue)"),        # fused gate/up: K run over both matrices
    (MISTRAL_SPECS[:4] + [(14336, 4096, 2, True)] + MISTRAL_SPECS[6:], 1, "k_gemv (epilogue)"),  # a layer
    ([(14336, 4096, 0, True)], 4, "k_gemv (epilogue)"),        # no two-row variant with an epilogue
    ([(14336, 2048, 0, True)], 1, "k_gemv_dyn (epilogue)"),    # fused, spread
])
def test_kernel_choice(q4k, specs, ncols, want):
    if "Q4K_LIB" in __import__("os").environ:
        pytest.skip("another build of the library (it may force one kernel)")
    assert q4k.batch_kernel(_tasks_ex(q4k, specs), ncols, num_sms=148) == want


def test_kernel_choice_rejects_bad_tasks(q4k):
    L = q4k.lib()
    assert L.q4k_batch_ex_kernel(None, 0, 1, 148) == -1
    bad = _tasks_ex(q4k, [(100, 300, 0, False)])  # K not a multiple of 256
    assert L.q4k_batch_ex_kernel(bad, 1, 1, 148) == -1
    assert b"K" in L.q4k_last_error()
    with pytest.raises(q4k.Q4KError):
        q4k.batch_kernel(bad, 1, num_sms=148)


def test_sharded_argument_checks(q4k):
    """q4k_gemv_sharded refuses bad ranks, communicators, shapes and
    workspaces before it touches NCCL or a device."""
    L = q4k.lib()
    assert L.q4k_sharded_workspace_bytes(100, 4096, 1, 0) == 0
    assert L.q4k_sharded_workspace_bytes(0, 4096, 1, 2) == 0
    assert L.q4k_sharded_workspace_bytes(100, 100, 1, 2) == 0  # K % 256
    # staging for 4 ranks x 2 columns x ceil(100 / 4) rows beside the shard's GEMV workspace
    assert L.q4k_sharded_workspace_bytes(100, 4096, 2, 4) >= q4k.gemv_workspace_bytes(25, 4096, 2) + 4 * 2 * 25 * 4

    def call(W=256, x=512, y=1024, K=4096, nrows=100, ncols=1, srx=16, scx=4096, scy=100, comm=4096, rank=0,
             world=2, ws=4096, wsb=1 << 30):
        return L.q4k_gemv_sharded(W, x, y, K, nrows, ncols, srx, scx, scy, comm, rank, world, ws, wsb, None)

    for kw in [dict(world=0), dict(world=1025), dict(rank=2), dict(rank=-1), dict(comm=None), dict(ncols=0),
               dict(ncols=9), dict(nrows=0), dict(y=None), dict(x=None), dict(ncols=2, scy=99), dict(K=100)]:
        assert call(**kw) == EINVAL, kw
        assert len(L.q4k_last_error()) > 0
    assert call(ws=None) == EWORKSPACE
    assert call(wsb=64) == EWORKSPACE
    assert call(ws=4096 + 16) == EWORKSPACE  # not 256-byte aligned

"""q4k_mul_mat_vec_noalloc: the GEMV for callers that cannot allocate device memory.

Such callers (runtimes that plan every device buffer ahead and forbid
cudaMalloc on the decode path; host applications that own the GPU memory
budget) cannot hand the library a workspace, so this entry point uses a
scratch array built into the library.  The test calls it through the C ABI
twice in a row -- different shapes, so the second call runs on whatever the
first left in the shared array -- and compares each result with the regular
workspace-taking entry point and with the CPU oracle, within the tolerance of
the other parity tests.
It lives in its own file, collected last, and needs nothing from other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-4, 1e-5


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row(q4k, oracle):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = q4k.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(2024)
    for nrows, K, ncols in [(1000, 4096, 3), (4096, 14336, 1)]:
        W = torch.from_numpy(q4k.gen_q4k_numpy(rng, nrows, K)).to(dev)
        x = torch.from_numpy(rng.standard_normal((ncols, K)).astype(np.float32)).to(dev)
        want = q4k.mul_mat_vec_q(W, x)  # regular entry point, caller workspace
        got = torch.full((ncols, nrows), float("nan"), device=dev)
        st = L.q4k_mul_mat_vec_noalloc(W.data_ptr(), x.data_ptr(), got.data_ptr(), K, nrows, ncols,
                                       W.stride(0) // 144, x.stride(0), got.stride(0), stream)
        assert st == 0, L.q4k_last_error()
        torch.cuda.synchronize()
        g, w = got.cpu().numpy().astype(np.float64), want.cpu().numpy().astype(np.float64)
        assert np.all(np.abs(g - w) <= TOL_ABS + TOL_REL * np.abs(w)), f"{nrows}x{K} ncols={ncols}"
        o = oracle.gemv_f32(W.cpu().numpy(), x.cpu().numpy()).astype(np.float64)
        assert np.all(np.abs(g - o) <= TOL_ABS + TOL_REL * np.abs(o)), f"{nrows}x{K} ncols={ncols} vs oracle"


def test_noalloc_rejects_calls_larger_than_its_array(q4k):
    import torch

    L = q4k.lib()
    cap = L.q4k_noalloc_scratch_bytes()
    assert cap == 4 << 20
    # 8 columns of K = 2^20 need 8 * 4096 * 320 B of packed activations alone (> 4 MiB)
    K, nrows, ncols = 1 << 20, 32, 8
    assert q4k.gemv_workspace_bytes(nrows, K, ncols) > cap
    st = L.q4k_mul_mat_vec_noalloc(256, 512, 1024, K, nrows, ncols, K // 256, K, nrows,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 1
    assert b"built-in array" in L.q4k_last_error()

"""Failure path of the fused all-gather, on one GPU and without a fault: a
"peer" that never signals.  The gather descriptor names a second rank whose
buffers are ordinary local memory and whose flag nothing ever sets.  The
gathering call itself does not wait for its peers: it stores this rank's
rows locally and into the silent peer's buffer, raises its flag there and
returns.  The consumer-side wait (q4k_gather_wait, and the next gathering
call before it reads its activations) must then give up after its bounded
2 s, record Q4K_ETIMEOUT in the workspace status word and return; the
context stays usable."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_and_reports_status(q4k):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(3)
    nrows, K = 64, 512
    W = torch.from_numpy(q4k.gen_q4k_numpy(rng, nrows, K)).to(dev)
    x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).to(dev)
    out_local = torch.zeros(nrows * 2, device=dev)       # this rank's full buffer (2 ranks x 64 rows)
    out_fake_peer = torch.zeros(nrows * 2, device=dev)   # the silent peer's buffer (local memory)
    flags_local = torch.zeros(64, dtype=torch.int32, device=dev)
    flags_fake_peer = torch.zeros(64, dtype=torch.int32, device=dev)
    epoch = torch.zeros(64, dtype=torch.int32, device=dev)

    g = q4k.Gather()
    g.world, g.rank = 2, 0
    g.out_local = out_local.data_ptr()
    g.out_elems = out_local.numel()
    g.out_peer[0], g.out_peer[1] = out_local.data_ptr(), out_fake_peer.data_ptr()
    g.flags_peer[0], g.flags_peer[1] = flags_local.data_ptr(), flags_fake_peer.data_ptr()
    g.epoch = epoch.data_ptr()
    dst = out_local[:nrows].view(1, nrows)  # rank 0 owns rows [0, 64) of a 128-row matrix
    tasks = q4k.make_tasks([W], [x], [dst])
    tasks[0].stride_col_dst = 2 * nrows
    ws = q4k.Workspace(q4k.batch_workspace_bytes(tasks, 1))
    s = torch.cuda.current_stream()
    L = q4k.lib()

    # the producer returns without waiting for the silent peer
    t0 = time.time()
    st = L.q4k_gemv_batch_allgather(tasks, 1, 1, ctypes.byref(g), ws.ptr, ws.nbytes, s.cuda_stream)
    assert st == 0, L.q4k_last_error()
    status = ws.status(s)  # synchronises
    assert status == 0, f"the gathering call itself must not wait (status {status})"
    assert time.time() - t0 < 1.5
    want = q4k.mul_mat_vec_q(W, x)
    assert torch.allclose(out_local[:nrows], want[0], rtol=1e-5, atol=1e-4)
    assert torch.allclose(out_fake_peer[:nrows], want[0], rtol=1e-5, atol=1e-4)
    assert int(flags_fake_peer[0]) == 1 and int(epoch[0]) == 1

    # the consumer's wait gives up after its bound and says so
    t0 = time.time()
    assert L.q4k_gather_wait(ctypes.byref(g), ws.ptr, ws.nbytes, s.cuda_stream) == 0
    status = ws.status(s)
    waited = time.time() - t0
    assert status == 3, f"expected Q4K_ETIMEOUT (3), got {status}"
    assert 1.5 < waited < 30.0

    # so does the next gathering call, before it reads its activations
    t0 = time.time()
    st = L.q4k_gemv_batch_allgather(tasks, 1, 1, ctypes.byref(g), ws.ptr, ws.nbytes, s.cuda_stream)
    assert st == 0, L.q4k_last_error()
    status = ws.status(s)
    assert status == 3 and 1.5 < time.time() - t0 < 30.0
    assert int(flags_fake_peer[0]) == 2 and int(epoch[0]) == 2

    # the context is still usable
    again = q4k.mul_mat_vec_q(W, x)
    torch.cuda.synchronize()
    assert torch.equal(again, want)

"""The two-row kernel's two ways of forming the integer sub-block sums give
the same result bit for bit.

At 3 columns the sums come from dp4a, from 4 columns on from int8
tensor-core MMAs (mma.m16n8k32 u8 x s8, eight columns per MMA, padding
included); the fp32 combination after them is the same code path, and a
column's result does not depend on the other columns.  So column j of a
4-column call must equal column j of a 3-column call on the same matrix and
activations exactly, on matrices with ragged row counts and on a batch of
several matrices (same worker partition at 3 and 4 columns).  The oracle
comparison of both widths is in tests/test_gpu_parity.py.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nrows,K", [(4096, 4096), (1000, 14336), (77, 256)])
def test_mma_and_dp4a_sums_agree_bitwise(q4k, nrows, K):
    import torch

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(nrows + K)
    W = torch.from_numpy(q4k.gen_q4k_numpy(rng, nrows, K)).to(dev)
    x = torch.from_numpy(rng.standard_normal((4, K)).astype(np.float32)).to(dev)
    y3 = q4k.mul_mat_vec_q(W, x[:3].contiguous())   # dp4a
    y4 = q4k.mul_mat_vec_q(W, x)                    # int8 MMA
    torch.cuda.synchronize()
    assert torch.equal(y3, y4[:3])


def test_mma_and_dp4a_agree_on_a_batch(q4k):
    import torch

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(5)
    shapes = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]
    Ws = [torch.from_numpy(q4k.gen_q4k_numpy(rng, r, K)).to(dev) for r, K in shapes]
    xs = [torch.from_numpy(rng.standard_normal((4, K)).astype(np.float32)).to(dev) for _, K in shapes]
    outs = {}
    for nc in (3, 4):
        ys = [torch.empty((nc, r), device=dev) for r, _ in shapes]
        tasks = q4k.make_tasks(Ws, [x[:nc].contiguous() for x in xs], ys)
        ws = q4k.Workspace(q4k.batch_workspace_bytes(tasks, nc), dev)
        q4k.gemv_batch(tasks, nc, ws)
        torch.cuda.synchronize()
        outs[nc] = ys
    for a, b in zip(outs[3], outs[4]):
        assert torch.equal(a, b[:3])

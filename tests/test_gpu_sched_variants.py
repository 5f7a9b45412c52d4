"""The GEMV kernels chosen by Q4K_SCHED, each against the oracle.

The library reads Q4K_SCHED once per process, so every variant runs in a
child process: "static" (the statically partitioned kernel only), "dynamic"
(the dynamically scheduled kernel wherever it can run: here a layer-sized
plain batch and a fused gate/up batch) and "mixed" (static prefix +
dynamic tail).  Each child computes the same seeded batches; the parent
checks every row against the oracle at the parity bar (1e-4 absolute +
1e-5 relative; the fused rows at the GLU tolerance of test_gpu_glu) and
that repeated calls in one child are bit-identical.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from test_gpu_glu import check

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
# 2 x 14336x4096 + 4096x14336: 10752 atoms, enough for the static prefix of
# the mixed kernel (4 atoms per warp) and for the dynamic kernel's groups
SHAPES = [(14336, 4096), (14336, 4096), (4096, 14336)]
X_OF = [0, 0, 1]

CHILD = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from conftest import load_package
q4k = load_package()
out_path, ncols = sys.argv[2], int(sys.argv[3])
shapes = [(14336, 4096), (14336, 4096), (4096, 14336)]
x_of = [0, 0, 1]
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev); g.manual_seed(321)
W = [q4k.gen_q4k_torch(r, K, generator=g, device=dev) for r, K in shapes]
xs = {0: torch.randn((ncols, 4096), device=dev, generator=g), 1: torch.randn((ncols, 14336), device=dev, generator=g)}
ws = q4k.Workspace()
runs = []
for _ in range(2):
    outs = [torch.empty((ncols, r), device=dev) for r, _ in shapes]
    q4k.gemv_batch(q4k.make_tasks(W, [xs[i] for i in x_of], outs), ncols, ws)
    runs.append([o.cpu().numpy() for o in outs])
fused = torch.empty((ncols, shapes[0][0]), device=dev)
q4k.gemv_batch_ex(q4k.make_tasks_ex([dict(W=W[1], W_gate=W[0], x=xs[0], out=fused, glu="swiglu")]), ncols, ws)
assert ws.status() == 0
np.savez(out_path, W0=W[0].cpu().numpy(), W1=W[1].cpu().numpy(), W2=W[2].cpu().numpy(),
         x0=xs[0].cpu().numpy(), x1=xs[1].cpu().numpy(), fused=fused.cpu().numpy(),
         **{f"r{k}_{i}": o for k, run in enumerate(runs) for i, o in enumerate(run)})
'''


@pytest.mark.parametrize("sched,ncols", [("static", 1), ("dynamic", 1), ("dynamic", 2), ("mixed", 1)])
def test_schedule_variant_vs_oracle(q4k, oracle, tmp_path, sched, ncols):
    out = tmp_path / f"{sched}_{ncols}.npz"
    env = {**os.environ, "Q4K_SCHED": sched}
    p = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(out), str(ncols)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    z = np.load(out)
    Ws = [z["W0"], z["W1"], z["W2"]]
    xs = [z["x0"], z["x1"]]
    for i in range(len(SHAPES)):
        assert np.array_equal(z[f"r0_{i}"], z[f"r1_{i}"]), f"{sched}: task {i} differs between calls"
        want = oracle.gemv_f32(Ws[i], xs[X_OF[i]]).astype(np.float64)
        check(z[f"r0_{i}"], want, want, "none", f"{sched} ncols={ncols} task {i}")
    r = oracle.gemv_f32(Ws[1], xs[0]).astype(np.float64)
    gate = oracle.gemv_f32(Ws[0], xs[0]).astype(np.float64)
    check(z["fused"], r, gate, "swiglu", f"{sched} ncols={ncols} fused gate/up")

"""The GEMV kernel variants, each against the oracle.

Every variant runs in a child process that loads one build of the library
(Q4K_LIB): "static" is the release build, whose measured choice for these
layer-sized launches is the statically partitioned kernel; "dynamic" is
libq4k_gemv_dyn.so (built with -DQ4K_SCHED_FORCE=2), which runs the
dynamically scheduled kernel wherever it can run (here a layer-sized plain
batch and a fused gate/up batch).  Each child computes the same seeded batches; the parent
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
# 2 x 14336x4096 + 4096x14336: 10752 atoms, enough row groups for the
# dynamic kernel's queue
SHAPES = [(14336, 4096), (14336, 4096), (4096, 14336)]
X_OF = [0, 0, 1]

CHILD = r'''
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from conftest import load_package
q4k = load_package()
out_path, ncols, want_kernel = sys.argv[2], int(sys.argv[3]), sys.argv[4]
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
    tasks = q4k.make_tasks(W, [xs[i] for i in x_of], outs)
    assert q4k.batch_kernel(tasks, ncols) == want_kernel, q4k.batch_kernel(tasks, ncols)
    q4k.gemv_batch(tasks, ncols, ws)
    runs.append([o.cpu().numpy() for o in outs])
fused = torch.empty((ncols, shapes[0][0]), device=dev)
q4k.gemv_batch_ex(q4k.make_tasks_ex([dict(W=W[1], W_gate=W[0], x=xs[0], out=fused, glu="swiglu")]), ncols, ws)
assert ws.status() == 0
np.savez(out_path, W0=W[0].cpu().numpy(), W1=W[1].cpu().numpy(), W2=W[2].cpu().numpy(),
         x0=xs[0].cpu().numpy(), x1=xs[1].cpu().numpy(), fused=fused.cpu().numpy(),
         **{f"r{k}_{i}": o for k, run in enumerate(runs) for i, o in enumerate(run)})
'''


VARIANTS = {"static": ("libq4k_gemv.so", "k_gemv"), "dynamic": ("libq4k_gemv_dyn.so", "k_gemv_dyn")}


@pytest.mark.parametrize("sched,ncols", [("static", 1), ("dynamic", 1), ("dynamic", 2)])
def test_schedule_variant_vs_oracle(q4k, oracle, tmp_path, sched, ncols):
    so, kernel = VARIANTS[sched]
    if not (q4k.HERE / so).exists():
        pytest.skip(f"{so} not built (make -C gemv-q4_k-optimization_b200 variants)")
    out = tmp_path / f"{sched}_{ncols}.npz"
    env = {**os.environ, "Q4K_LIB": str(q4k.HERE / so)}
    p = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(out), str(ncols), kernel], env=env,
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

"""The launch-timeline diagnostic (tests/timeline_driver.py
over the Q4K_TIMELINE build): one small chained workload, recorded from a CUDA
graph replay, gives a sane record for every launch."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


def test_timeline_records_every_launch(q4k):
    if not q4k.TIMELINE_LIB.exists():
        pytest.skip("timeline library not built (make -C gemv-q4_k-optimization_b200 timeline)")
    script = Path(__file__).resolve().parent / "timeline_driver.py"
    env = {"Q4K_LIB": str(q4k.TIMELINE_LIB)}
    import os
    env = {**os.environ, **env}
    out = subprocess.run([sys.executable, str(script), "--config", "1", "--json"], capture_output=True,
                         text=True, env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["launches"] == 48
    m = d["mean_us"]
    # a 4096x4096 launch streams 9.4 MB: a period of microseconds, workers
    # ending after their release, the quantization launch in between
    assert 1.0 < m["period"] < 100.0
    assert 0.0 < m["end_p10"] <= m["end_p50"] <= m["end_p90"] <= m["end_max"] < m["period"] + 5
    assert 0.0 <= m["prep_run"] < m["period"]
    assert len(d["ring_mean_end_us"]) >= 1 and len(d["cta_mean_end_us"]) >= 1


def test_timeline_fused_launch_records(q4k):
    """Launches with a fused gate/up task run the queue variant: besides the
    compute warps' records, each CTA's flushing warp (which writes the rows)
    leaves one, ending after most compute warps and within the launch."""
    if not q4k.TIMELINE_LIB.exists():
        pytest.skip("timeline library not built (make -C gemv-q4_k-optimization_b200 timeline)")
    import os
    script = Path(__file__).resolve().parent / "timeline_driver.py"
    env = {**os.environ, "Q4K_LIB": str(q4k.TIMELINE_LIB)}
    out = subprocess.run([sys.executable, str(script), "--config", "ffn", "--json"], capture_output=True,
                         text=True, env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["launches"] == 16
    m = d["mean_us"]
    assert 1.0 < m["period"] < 200.0
    assert m["end_p10"] <= m["fold_end_max"] < m["period"] + 5


def test_timeline_single_launch_records(q4k):
    """The same diagnostic over the single-launch mode: every launch planned
    and quantized its activations after its release and before its warps
    ended."""
    if not q4k.TIMELINE_LIB.exists():
        pytest.skip("timeline library not built (make -C gemv-q4_k-optimization_b200 timeline)")
    import os
    script = Path(__file__).resolve().parent / "timeline_driver.py"
    env = {**os.environ, "Q4K_LIB": str(q4k.TIMELINE_LIB)}
    out = subprocess.run([sys.executable, str(script), "--config", "1", "--single", "--json"], capture_output=True,
                         text=True, env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["launches"] == 48 and d["single"]
    m = d["mean_us"]
    assert 1.0 < m["period"] < 100.0
    assert 0.0 <= m["quant_p50"] <= m["quant_max"] <= m["end_max"]
    assert m["plan_max"] >= 0.0

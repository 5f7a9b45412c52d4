#!/usr/bin/env python
"""Q4_K x q8_1 decode-GEMV benchmark on B200.

Default workload ("mistral-7b-decode-gemv-set"): one decode
step's Q4_K GEMVs of Mistral-7B at batch 1 -- 32 layers x {q 4096x4096, k
1024x4096, v 1024x4096, o 4096x4096, gate 14336x4096, up 14336x4096, down
4096x14336} plus the 32000x4096 output head, synthetic seeded weights with
the BASELINE value distributions (d, dmin = fp16(|N(0,1)|*0.01), uniform 6-bit
scales/mins, uniform nibbles; generated on the device) and x ~ N(0,1) (q/k/v
share one activation, gate/up share one).  One prep + persistent GEMV launch
pair per layer.  The 4.0 GB of weights per step exceed the 126 MB L2, so
every step streams from HBM.  Other BASELINE configs: --config 1/3/4/5/5t.

Metric: achieved algorithmic HBM bandwidth of the whole job (TB/s, all
ranks) with bytes = rows*K*0.5625 + ncols*K*4 per distinct activation +
ncols*rows*4; also us per GEMV launch.

  python bench.py [--gpus N --steps K --warmup W --ncols C --config 2]
  python bench.py --impl reference    # the reference's CPU path, timed on the host

N > 1 (torchrun, one rank per GPU): every matrix is row-sharded across the
ranks; by default each launch also all-gathers the output rows into every
rank's buffer over NVLink peer stores (--gather nccl: NCCL all_gather per
launch instead).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "gemv-q4_k-optimization_b200"
PROFILES = ROOT / "profiles"
METRIC = "Q4_K GEMV achieved HBM TB/s (algorithmic bytes), us per GEMV launch"

# A launch group is one q4k_gemv_batch launch: (name, rows, K, activation group
# [, glu op]).  An entry with a glu op is a gate/up pair fused in one task
# (two matrices of rows x K, one output: op(up.x, gate.x)).
MISTRAL_LAYER = [("q", 4096, 4096, "attn"), ("k", 1024, 4096, "attn"), ("v", 1024, 4096, "attn"),
                 ("o", 4096, 4096, "o"), ("gate", 14336, 4096, "ffn"), ("up", 14336, 4096, "ffn"),
                 ("down", 4096, 14336, "down")]
LLAMA70B_LAYER = [("q", 8192, 8192, "attn"), ("k", 1024, 8192, "attn"), ("v", 1024, 8192, "attn"),
                  ("o", 8192, 8192, "o"), ("gate", 28672, 8192, "ffn"), ("up", 28672, 8192, "ffn"),
                  ("down", 8192, 28672, "down")]
MISTRAL_LAYER_FUSED = [e for e in MISTRAL_LAYER if e[0] not in ("gate", "up")]
MISTRAL_LAYER_FUSED.insert(4, ("gate_up", 14336, 4096, "ffn", "swiglu"))
# BASELINE config -> (workload name, repeated launch group, default repeats, trailing groups)
WORKLOADS = {
    "2": ("mistral-7b-decode-gemv-set", MISTRAL_LAYER, 32, [[("head", 32000, 4096, "head")]]),
    "1": ("single-4096x4096", [("attn_q", 4096, 4096, "x")], 48, []),
    "3": ("ffn-up-14336x4096", [("ffn_up", 14336, 4096, "x")], 16, []),
    "4": ("llama-3-70b-layer-gemvs", LLAMA70B_LAYER, 8, []),
    "5": ("head-128256x8192", [("head", 128256, 8192, "x")], 6, []),
    "5t": ("tiny-1024x4096-and-512x4096", [("tiny_1024", 1024, 4096, "x")], 256, []),
    # next-row workloads: the fused gate+up+SwiGLU epilogue
    "2f": ("mistral-7b-decode-gemv-set-ffn-gate-up-swiglu-fused", MISTRAL_LAYER_FUSED, 32,
           [[("head", 32000, 4096, "head")]]),
    "ffn": ("ffn-gate-up-swiglu-2x14336x4096", [("gate_up", 14336, 4096, "x", "swiglu")], 16, []),
    # Q6_K weights (the output heads of Q4_K_M checkpoints)
    "q6": ("mistral-7b-q6_k-head-32000x4096", [("head_q6", 32000, 4096, "x", "q6")], 16, []),
    "q6l": ("llama-3-q6_k-head-128256x8192", [("head_q6", 128256, 8192, "x", "q6")], 6, []),
}


def ent(e):
    """(name, rows, K, activation group, glu op or None) of a group entry ("q6": Q6_K weights)."""
    return (e[0], e[1], e[2], e[3], e[4] if len(e) > 4 else None)


def wbytes(r, K, glu):
    """Weight bytes of an entry: Q4_K 0.5625 B/weight (two matrices when fused), Q6_K 0.8203."""
    if glu == "q6":
        return r * K * 210 // 256
    return r * K * 9 // 16 * (2 if glu else 1)


def build_groups(cfg: str, repeats: int):
    name, group, _, tail = WORKLOADS[cfg]
    groups = [list(group) for _ in range(repeats)]
    if cfg == "5t":  # alternate the two tiny shapes, one launch each
        groups = [[("tiny_1024", 1024, 4096, "x")] if i % 2 == 0 else [("tiny_512", 512, 4096, "x")]
                  for i in range(repeats)]
    return name, groups + [list(t) for t in tail]


def group_bytes(group, ncols: int, world: int = 1) -> int:
    """Algorithmic bytes of one launch group, all ranks (every rank reads the whole x)."""
    acts = {}
    for _, r, K, a, _ in map(ent, group):
        acts[a] = K
    w = sum(wbytes(r, K, glu) for _, r, K, _, glu in map(ent, group))
    x = sum(ncols * K * 4 for K in acts.values()) * world
    y = sum(ncols * r * 4 for _, r, _, _, _ in map(ent, group))
    return w + x + y


def load_package():
    if "q4k_b200" in sys.modules:
        return sys.modules["q4k_b200"]
    spec = importlib.util.spec_from_file_location("q4k_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["q4k_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    O.build()
    return O


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = str(uuid or "").lower()
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)  # let the sampler catch the end of the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        rows = []
        for ln in self.lines:
            f = [c.strip() for c in ln.split(",")]
            if len(f) < 10:
                continue
            if self.uuid and self.uuid not in f[1].lower():
                continue
            rows.append(f)
        sm = [float(f[2].split()[0]) for f in rows if f[2].split()[0].replace(".", "").isdigit()]
        smax = [float(f[3].split()[0]) for f in rows if f[3].split()[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for f in rows for n, v in zip(names, f[6:10]) if v.lower() == "active"})
        loaded = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows),
                "window": "untimed soak of step replays (~0.8 s) + warm-up + timed steps"}


# ---------------------------------------------------------------------------
# CPU legs (the oracle and the reference's own dot product; checkers only)
# ---------------------------------------------------------------------------
def host_group(q4k, group, ncols, rng):
    """Host matrices (W, K, activation group, Q6_K?) of one launch group, and its activations."""
    mats = []
    for _, r, K, a, glu in map(ent, group):
        if glu == "q6":
            mats.append((q4k.gen_q6k_numpy(rng, r, K), K, a, True))
        else:
            mats += [(q4k.gen_q4k_numpy(rng, r, K), K, a, False) for _ in range(2 if glu else 1)]
    xs = {a: rng.standard_normal((ncols, K)).astype(np.float32) for _, _, K, a, _ in map(ent, group)}
    return mats, xs


def run_reference(args) -> None:
    """The reference's CPU implementation of the path (its vec_dot_q4_K_q8_1
    compiled for the host, oracle/_ref), all host threads, one launch group
    per step (a decoder layer for config 2)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    O = load_oracle()
    q4k = load_package()
    name, groups = build_groups(args.config, 1)
    group = groups[0]
    ncols = args.ncols
    mats, xs = host_group(q4k, group, ncols, np.random.default_rng(0))
    # the reference's compiled dot product covers Q4_K; Q6_K runs on the port
    kind = "reference" if O.ref_available() and not any(m[3] for m in mats) else "port"
    threads = O.max_threads() if kind == "port" else O.ref_lib().ref_max_threads()

    def one_step():
        for W, K, a, is_q6 in mats:
            yq = O.quantize_q8_1(xs[a])
            if is_q6:
                O.gemv_q6k_q8_1(W, K, yq, nthreads=threads)
            elif kind == "reference":
                O.ref_gemv_q8_1(W, K, yq, nthreads=threads)
            else:
                O.gemv_q8_1(W, K, yq, nthreads=threads)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = (time.perf_counter() - t0) / args.steps
    tbs = group_bytes(group, ncols) / dt / 1e12
    sample = (f"one launch group of {name} per step ({len(group)} Q4_K GEMVs, "
              f"{group_bytes(group, ncols) / 1e6:.1f} MB algorithmic), q8_1 quantization included; "
              f"{'the reference vec_dot_q4_K_q8_1 in MMVQ order' if kind == 'reference' else 'the C oracle'}")
    line = {
        "impl": "reference", "metric": METRIC, "value": tbs, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": name, "ncols": ncols, "sample": "one launch group per step"},
        "cpu_baseline": {"value": tbs, "unit": "TB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": tbs, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(O, mats, group, ncols, budget_s: float = 12.0) -> dict:
    """The oracle (all host threads) on the first launch group, repeated for ~budget_s."""
    rng = np.random.default_rng(1)
    xs = {a: rng.standard_normal((ncols, K)).astype(np.float32) for _, _, K, a, _ in map(ent, group)}
    threads = O.max_threads()

    def timed(nthreads, budget):
        n, t0 = 0, time.perf_counter()
        while True:
            for W, K, a, is_q6 in mats:
                (O.gemv_q6k_f32 if is_q6 else O.gemv_f32)(W, xs[a], nthreads=nthreads)
            n += 1
            el = time.perf_counter() - t0
            if el > budget:
                return n, el

    n, el = timed(threads, budget_s)
    n1, el1 = timed(1, budget_s / 3)
    return {"value": group_bytes(group, ncols) * n / el / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
            "value_1thread": group_bytes(group, ncols) * n1 / el1 / 1e12,
            "sample": f"{n} x the first launch group ({len(group)} Q4_K GEMVs, fp32 x, q8_1 quantization "
                      f"included) = {el:.1f} s on the host with {threads} threads; value_1thread: {n1} x the "
                      f"same group = {el1:.1f} s on one thread"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--ncols", type=int, default=1)
    ap.add_argument("--config", default="2", choices=sorted(WORKLOADS), help="BASELINE config (default 2)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=None,
                    help="repeats of the workload's launch group (default: the workload's; profiling: fewer)")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying CUDA graphs")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: fused peer-store all-gather in the GEMV (default) or NCCL all_gather per launch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    q4k = load_package()
    q4k.lib()
    ncols = args.ncols
    reps = args.layers if args.layers is not None else WORKLOADS[args.config][2]
    wname, groups = build_groups(args.config, reps)
    full_run = args.layers is None or args.layers == WORKLOADS[args.config][2]

    # ---- weights (row shards), activations, outputs -------------------------
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    peer = world > 1 and args.gather == "peer"
    full_elems = sum(r * ncols for grp in groups for _, r, _, _, _ in map(ent, grp))
    q6 = any(glu == "q6" for grp in groups for *_, glu in map(ent, grp))
    fused = not q6 and any(glu for grp in groups for *_, glu in map(ent, grp))
    if (fused or q6) and world > 1:
        raise SystemExit(f"config {args.config} (fused epilogue / Q6_K) runs on one GPU")
    pg = q4k.PeerGather(full_elems) if peer else None
    # Every step's activations live in one device buffer and its local outputs
    # in another, so that the end-to-end leg moves each with one copy.
    x_tot = sum(ncols * K for grp in groups for K in {a: K for _, _, K, a, _ in map(ent, grp)}.values())
    x_all = torch.empty((x_tot,), device=dev)
    x_off = 0
    y_tot = 0
    if not peer:
        for grp in groups:
            y_tot += -(-sum(q4k.shard_rows(r, rank, world)[2] for _, r, _, _, _ in map(ent, grp)) * ncols // 64) * 64
    y_all = torch.zeros((max(y_tot, 1),), device=dev)
    y_off = 0
    L = []
    base = 0
    for grp in groups:
        xs = {}
        for _, _, K, a, _ in map(ent, grp):
            if a not in xs:
                xs[a] = x_all[x_off: x_off + ncols * K].view(ncols, K).normal_(generator=g)
                x_off += ncols * K
        ents = []
        for name, rows, K, a, glu in map(ent, grp):
            lo, hi, per = q4k.shard_rows(rows, rank, world)
            if glu == "q6":
                W, Wg = q4k.gen_q6k_torch(hi - lo, K, generator=g, device=dev), None
            else:
                W = q4k.gen_q4k_torch(hi - lo, K, generator=g, device=dev)
                Wg = q4k.gen_q4k_torch(hi - lo, K, generator=g, device=dev) if glu else None
            ents.append(dict(name=name, W=W, W_gate=Wg, glu=glu, x=xs[a], rows=rows, K=K, lo=lo, n=hi - lo,
                             per=per))
        if peer:
            # full outputs live in the shared buffer; each rank writes its rows
            # there and the kernel stores them into every peer's buffer too
            outs, ybuf0 = [], base
            for e in ents:
                full = pg.out[base: base + e["rows"] * ncols].view(ncols, e["rows"])
                outs.append(full[:, e["lo"]: e["lo"] + e["n"]])
                e["stride"] = e["rows"]
                base += e["rows"] * ncols
            ybuf, gath = pg.out[ybuf0: base], None
        else:
            per_tot = sum(e["per"] for e in ents)
            ybuf = y_all[y_off: y_off + per_tot * ncols]
            y_off += -(-per_tot * ncols // 64) * 64
            outs, off = [], 0
            for e in ents:
                outs.append(ybuf[off: off + e["per"] * ncols].view(ncols, e["per"])[:, : e["n"]])
                e["stride"] = e["per"]
                off += e["per"] * ncols
            gath = torch.empty((per_tot * ncols * world,), device=dev) if world > 1 else None
        if q6:
            tasks = q4k.make_tasks_q6_k([e["W"] for e in ents], [e["x"] for e in ents], outs)
            for i, e in enumerate(ents):
                tasks[i].stride_col_dst = e["stride"]
        elif fused:
            tasks = q4k.make_tasks_ex([dict(W=e["W"], W_gate=e["W_gate"], x=e["x"], out=o,
                                            glu=e["glu"] or "none") for e, o in zip(ents, outs)])
            for i, e in enumerate(ents):
                tasks[i].t.stride_col_dst = e["stride"]
        else:
            tasks = q4k.make_tasks([e["W"] for e in ents], [e["x"] for e in ents], outs)
            for i, e in enumerate(ents):
                tasks[i].stride_col_dst = e["stride"]
        L.append(dict(xs=xs, ents=ents, ybuf=ybuf, tasks=tasks, gath=gath))

    wsb = (q4k.batch_ex_workspace_bytes if fused else
           (lambda t, n: int(q4k.lib().q4k_batch_q6_k_workspace_bytes(t, len(t), n))) if q6 else
           q4k.batch_workspace_bytes)
    ws = q4k.Workspace(max(wsb(G["tasks"], ncols) for G in L), dev)
    stream = torch.cuda.Stream(device=dev)

    def gemv(tasks):
        if peer:
            q4k.gemv_batch_allgather(tasks, ncols, pg, ws, stream=stream)
        elif fused:
            q4k.gemv_batch_ex(tasks, ncols, ws, stream=stream)
        elif q6:
            q4k.gemv_batch_q6_k(tasks, ncols, ws, stream=stream)
        else:
            q4k.gemv_batch(tasks, ncols, ws, stream=stream)

    def run_step(ev=None):
        for gi, G in enumerate(L):
            if ev is not None:
                ev[gi][0].record(stream)
            gemv(G["tasks"])
            if ev is not None:
                ev[gi][1].record(stream)
            if world > 1 and not peer:
                dist.all_gather_into_tensor(G["gath"], G["ybuf"])

    # ---- one untimed step: checks the device status word before timing ------
    with torch.cuda.stream(stream):
        run_step()
    stream.synchronize()
    assert ws.status(stream) == 0, "device status word reports an error"

    # ---- capture the step: launches chained back to back (no events between
    # them, which would break the programmatic-dependency overlap) -----------
    use_graph = not args.no_graph
    step_graph = None
    if use_graph:
        try:
            with torch.cuda.stream(stream):
                step_graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(step_graph, stream=stream):
                    run_step()
        except Exception as e:  # capture unsupported: time eagerly
            print(f"# graph capture failed ({e!r}); timing eager launches", file=sys.stderr)
            use_graph, step_graph = False, None

    def replay():
        with torch.cuda.stream(stream):  # replay() launches on the current stream
            if use_graph:
                step_graph.replay()
            else:
                run_step()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except AttributeError:
        pass
    sampler = ClockSampler(uuid) if rank == 0 else None

    # Clock samples (every 200 ms) need load around the short timed region:
    # the sampler runs from an untimed soak of step replays (~0.8 s) through
    # the warm-up and the timed steps.  Every rank replays the same number of
    # soak steps (rank 0's count).
    if sampler:
        sampler.start()
    nsoak, t_soak = 0, time.perf_counter()
    while time.perf_counter() - t_soak < 0.8 and nsoak < 4000:
        for _ in range(10):
            replay()
        nsoak += 10
        torch.cuda.synchronize(dev)
    if world > 1:
        t = torch.tensor([nsoak], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        for _ in range(int(t[0]) - nsoak):
            replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
    for _ in range(args.warmup):
        replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        replay()
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop() if sampler else None
    ms = t_start.elapsed_time(t_end) / args.steps

    # ---- isolated launches (events between launches serialize them) ---------
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in L]
    with torch.cuda.stream(stream):
        run_step(ev)
    torch.cuda.synchronize(dev)
    nrep = len(groups) - len(WORKLOADS[args.config][3])  # the repeated group only
    iso_ms = float(np.mean([a.elapsed_time(b) for a, b in ev[: max(1, nrep)]]))
    if world > 1:
        t = torch.tensor([ms, iso_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, iso_ms = float(t[0]), float(t[1])

    step_total = sum(group_bytes(G, ncols, world) for G in groups)
    value = step_total / (ms * 1e-3) / 1e12
    peak, peak_kind = measured_peaks()
    nlaunch = len(groups)
    launch_us = ms * 1e3 / nlaunch
    # Every launch of the timed step is k_gemv (with its programmatic-dependent
    # prep): its average duration in the chained step is step time / launches;
    # achieved bandwidth per rank = the rank's step bytes / step time.
    achieved = step_total / world / (ms * 1e-3) / 1e9
    g0 = groups[0]
    if world == 1:
        launch_bytes = group_bytes(g0, ncols)
    else:  # this rank's share of the first launch group
        launch_bytes = (sum(wbytes(e["n"], e["K"], e["glu"]) + ncols * e["n"] * 4 for e in L[0]["ents"]) +
                        sum(ncols * x.shape[1] * 4 for x in L[0]["xs"].values()))

    # ---- e2e: public C-ABI calls with host buffers ------------------------------
    e2e = None
    if not args.no_e2e:
        xs_all = [x_all]
        ys_all = [pg.out] if peer else [y_all]
        h_x = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs_all]
        for h, d in zip(h_x, xs_all):
            h.copy_(d)
        h_y = [torch.empty(y.shape, dtype=y.dtype, pin_memory=True) for y in ys_all]
        h2d = sum(h.numel() * 4 for h in h_x)
        d2h = sum(h.numel() * 4 for h in h_y)

        def e2e_step():
            with torch.cuda.stream(stream):
                for h, d in zip(h_x, xs_all):
                    d.copy_(h, non_blocking=True)
                run_step()
                for h, d in zip(h_y, ys_all):
                    h.copy_(d, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        e_ms = a.elapsed_time(b) / args.steps
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t[0])
        e2e = {"value": step_total / (e_ms * 1e-3) / 1e12, "unit": "TB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "path": "q4k_gemv_batch C-ABI calls (ctypes), one per launch group, eager (no graph); every "
                       "step one copy of all its activations pinned host -> device before the calls and one "
                       "copy of all its outputs device -> pinned host after them"}

    # the GEMV kernel each distinct launch group runs (the library's own choice)
    try:
        kernels = "k_gemv (Q6_K)" if q6 else (
            "k_gemv (gather epilogue)" if peer else sorted({q4k.batch_kernel(G["tasks"], ncols) for G in L}))
    except Exception as e:  # a report, never a reason to lose the measurement
        kernels = f"unknown ({e!r})"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O = load_oracle()
        mats = [(M.cpu().numpy(), e["K"], a, e["glu"] == "q6")
                for e, (_, _, _, a, _) in zip(L[0]["ents"], map(ent, g0))
                for M in (e["W"], e["W_gate"]) if M is not None]
        cpu = cpu_baseline(O, mats, g0, ncols)

    traffic = None
    tf = PROFILES / "gemv_layer_traffic.json"
    if tf.exists() and world == 1 and args.config == "2":
        d = json.loads(tf.read_text())
        if d.get("ncols") == ncols:
            traffic = d.get("dram_bytes_per_launch")

    if rank == 0:
        shapes = sorted({f"{r}x{K}" for grp in groups for _, r, K, _, _ in map(ent, grp)})
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded, generated on the device)",
            "config": {"workload": wname if full_run else f"{wname} (profiling subset)",
                       "baseline_config": args.config, "launch_groups": nlaunch, "shapes": shapes,
                       "ncols": ncols, "gemv_kernels": kernels,
                       "launches": "per group: prep (q8_1 quantization) + persistent GEMV over the group's "
                                   "matrices, chained with programmatic dependencies" + (
                                       "; ffn gate+up as one task with the SwiGLU epilogue" if fused else ""),
                       "timing": "one CUDA graph per step, CUDA events on the launch stream around all timed steps",
                       "l2": "inputs larger than L2 (weights per step >= 3x the 126 MB L2), no flush needed",
                       "parallelism": "single GPU" if world == 1 else (
                           f"row-shard x{world}, outputs all-gathered inside the GEMV over NVLink peer stores"
                           if peer else f"row-shard x{world} + NCCL all-gather per launch")},
            "us_per_call": launch_us,
            "us_per_launch_isolated": iso_ms * 1e3,
            "pct_hbm_peak": 100.0 * value * 1e3 / world / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": f"{', '.join(kernels) if isinstance(kernels, list) else kernels}: "
                                   "every launch of the step, each with its programmatic-dependent prep "
                                   "launch; achieved = step bytes per rank / step time",
                         "algorithmic_bytes_per_launch": launch_bytes,
                         "launch_isolated_gbs": launch_bytes / (iso_ms * 1e-3) / 1e9},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": args.steps * nlaunch * 2,
            "graph": use_graph,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        step_graph = None
        torch.cuda.synchronize(dev)
        dist.barrier()
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Q4_K x q8_1 decode-GEMV benchmark on B200.

Headline workload ("mistral-7b-decode-gemv-set"): one
decode step's Q4_K GEMVs of Mistral-7B at batch 1 -- 32 layers x {q 4096x4096,
k 1024x4096, v 1024x4096, o 4096x4096, gate 14336x4096, up 14336x4096, down
4096x14336} plus the 32000x4096 output head, synthetic seeded weights with the
BASELINE value distributions (d, dmin = fp16(|N(0,1)|*0.01), uniform 6-bit
scales/mins, uniform nibbles; generated on the device) and x ~ N(0,1) (q/k/v
share one activation, gate/up share one).  One launch sequence per layer.
The 4.0 GB of weights per step exceed the 126 MB L2, so every step streams
from HBM.

Every other BASELINE config is measured in the same run and reported under
"per_config": at one GPU configs 1 (4096x4096), 3 (ffn_up 14336x4096 at
ncols 1, 2, 3, 4, 8), 4 (Llama-3-70B layer), 5 (the 128256x8192 head) and 5t
(the tiny 1024x4096 / 512x4096 pair); at N > 1 GPUs the row-sharded configs
4 and 5.  Each entry: ms per step, us per launch, TB/s, fraction of the
measured HBM peak and the clocks seen during its timed region.

Metric: achieved algorithmic HBM bandwidth of the whole job (TB/s, all
ranks) with bytes = rows*K*0.5625 + ncols*K*4 per distinct activation +
ncols*rows*4; also us per GEMV launch.

  python bench.py [--gpus N --steps K --warmup W --ncols C --config 2]
  python bench.py --impl reference    # the reference's CPU path, timed on the host

N > 1 (torchrun, one rank per GPU): every matrix is row-sharded across the
ranks (contiguous ceil-split, the reference's row-split mode); each launch
stores its output rows into every rank's full output buffer over NVLink
(--gather nccl: NCCL all_gather per launch instead).  Before timing, every
rank checks a seeded sample of 256 gathered rows per matrix against the CPU
oracle ("parity": "ok" | "fail").
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

# A launch group is one batch launch: (name, rows, K, activation group
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
# The other BASELINE configs measured beside the headline: (config, ncols).
PER_CONFIG_1GPU = [("1", 1), ("3", 1), ("3", 2), ("3", 3), ("3", 4), ("3", 8), ("4", 1), ("5", 1), ("5t", 1)]
PER_CONFIG_SHARDED = [("4", 1), ("5", 1)]


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


def host_cores() -> int:
    """Host threads this process may run on (affinity-aware)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
    """nvidia-smi samples every 200 ms, each stamped with the host clock, so
    that any timed window can be summarised."""
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = str(uuid or "").lower()
        self.proc = None
        self.rows: list[tuple[float, list[str]]] = []
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
            f = [c.strip() for c in ln.strip().split(",")]
            if len(f) < 10 or (self.uuid and self.uuid not in f[1].lower()):
                continue
            self.rows.append((time.perf_counter(), f))

    def stop(self):
        if self.proc is None:
            return
        time.sleep(0.25)  # let the sampler catch the end of the last timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)

    def summary(self, t0: float, t1: float, window: str) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [f for t, f in self.rows if t0 - 0.2 <= t <= t1 + 0.2]

        def num(v):
            v = v.split()[0] if v.split() else ""
            return float(v) if v.replace(".", "").isdigit() else None

        sm = [v for v in (num(f[2]) for f in rows) if v is not None]
        smax = [v for v in (num(f[3]) for f in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for f in rows for n, v in zip(names, f[6:10]) if v.lower() == "active"})
        loaded = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows),
                "window": window}


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
    compiled for the host, oracle/_ref), on all host cores, over the same
    step as our arm: every launch group of the config (for config 2: 32
    decoder layers and the output head).  One host copy of each distinct
    launch group's weights serves all its repeats (each group far exceeds the
    CPU caches, so the repeats stream from memory as distinct copies would)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    O = load_oracle()
    q4k = load_package()
    ncols = args.ncols
    reps = args.layers if args.layers is not None else WORKLOADS[args.config][2]
    name, groups = build_groups(args.config, reps)
    rng = np.random.default_rng(0)
    distinct = {}
    for grp in groups:
        key = tuple(grp)
        if key not in distinct:
            distinct[key] = host_group(q4k, grp, ncols, rng)
    # the reference's compiled dot product covers Q4_K; Q6_K runs on the port
    any_q6 = any(m[3] for mats, _ in distinct.values() for m in mats)
    kind = "reference" if O.ref_available() and not any_q6 else "port"
    threads = host_cores()  # explicit: torchrun sets OMP_NUM_THREADS=1 in the environment

    def one_step():
        for grp in groups:
            mats, xs = distinct[tuple(grp)]
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
    step_bytes = sum(group_bytes(g, ncols) for g in groups)
    tbs = step_bytes / dt / 1e12
    sample = (f"the whole step of {name}: {len(groups)} launch groups, "
              f"{sum(len(g) for g in groups)} GEMVs, {step_bytes / 1e9:.2f} GB algorithmic, q8_1 quantization "
              f"included, {threads} host threads; "
              f"{'the reference vec_dot_q4_K_q8_1 in MMVQ order' if kind == 'reference' else 'the C oracle'}")
    line = {
        "impl": "reference", "metric": METRIC, "value": tbs, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": name, "baseline_config": args.config, "ncols": ncols,
                   "launch_groups": len(groups), "sample": "the whole step, every launch group"},
        "cpu_baseline": {"value": tbs, "unit": "TB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": tbs, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(O, mats, group, ncols, budget_s: float = 12.0) -> dict:
    """The oracle (all host cores) on the first launch group, repeated for ~budget_s."""
    rng = np.random.default_rng(1)
    xs = {a: rng.standard_normal((ncols, K)).astype(np.float32) for _, _, K, a, _ in map(ent, group)}
    threads = host_cores()

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
class Ctx:
    """What every workload of one run shares: process layout, device, library."""

    def __init__(self, args, torch, dist, q4k):
        self.args, self.torch, self.dist, self.q4k = args, torch, dist, q4k
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = torch.device("cuda", self.local)
        self.peer = self.world > 1 and args.gather == "peer"

    def barrier(self):
        if self.world > 1:
            self.torch.cuda.synchronize(self.dev)
            self.dist.barrier()

    def max_over_ranks(self, vals):
        if self.world == 1:
            return [float(v) for v in vals]
        t = self.torch.tensor([float(v) for v in vals], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def all_ok(self, ok: bool) -> bool:
        if self.world == 1:
            return ok
        t = self.torch.tensor([1 if ok else 0], device=self.dev, dtype=self.torch.int32)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN)
        return bool(int(t[0]))


class Workload:
    """One config's device buffers, tasks and launch sequence on this rank."""

    def __init__(self, C: Ctx, cfg: str, ncols: int, reps: int | None, pg=None):
        torch, q4k = C.torch, C.q4k
        self.C, self.cfg, self.ncols = C, cfg, ncols
        rank, world, dev = C.rank, C.world, C.dev
        self.reps = reps if reps is not None else WORKLOADS[cfg][2]
        self.name, self.groups = build_groups(cfg, self.reps)
        self.full_run = self.reps == WORKLOADS[cfg][2]
        # weights: this rank's row shards (rank-specific stream); activations:
        # replicated, the same on every rank (row split shares x)
        gw = torch.Generator(device=dev)
        gw.manual_seed(1234 + 7919 * rank + 104729 * int.from_bytes(cfg.encode(), "little") + ncols)
        gx = torch.Generator(device=dev)
        gx.manual_seed(4321 + ncols)
        peer = C.peer
        full_elems = sum(r * ncols for grp in self.groups for _, r, _, _, _ in map(ent, grp))
        self.q6 = any(glu == "q6" for grp in self.groups for *_, glu in map(ent, grp))
        self.fused = not self.q6 and any(glu for grp in self.groups for *_, glu in map(ent, grp))
        if (self.fused or self.q6) and world > 1:
            raise SystemExit(f"config {cfg} (fused epilogue / Q6_K) runs on one GPU")
        # row-sharded runs share one gather buffer (allocated once per run)
        self.pg = pg if peer else None
        self.full_elems = full_elems
        if peer and (pg is None or pg.out.numel() < full_elems):
            raise SystemExit("the gather buffer is smaller than this workload's outputs")
        # Every step's activations live in one device buffer and its local
        # outputs in another, so that the end-to-end leg moves each with one copy.
        x_tot = sum(ncols * K for grp in self.groups for K in {a: K for _, _, K, a, _ in map(ent, grp)}.values())
        self.x_all = torch.empty((x_tot,), device=dev)
        x_off = 0
        y_tot = 0
        if not peer:
            for grp in self.groups:
                y_tot += -(-sum(q4k.shard_rows(r, rank, world)[2] for _, r, _, _, _ in map(ent, grp)) * ncols
                           // 64) * 64
        self.y_all = torch.zeros((max(y_tot, 1),), device=dev)
        y_off = 0
        self.L = []
        base = 0
        for grp in self.groups:
            xs = {}
            for _, _, K, a, _ in map(ent, grp):
                if a not in xs:
                    xs[a] = self.x_all[x_off: x_off + ncols * K].view(ncols, K).normal_(generator=gx)
                    x_off += ncols * K
            ents = []
            for name, rows, K, a, glu in map(ent, grp):
                lo, hi, per = q4k.shard_rows(rows, rank, world)
                if glu == "q6":
                    W, Wg = q4k.gen_q6k_torch(hi - lo, K, generator=gw, device=dev), None
                else:
                    W = q4k.gen_q4k_torch(hi - lo, K, generator=gw, device=dev)
                    Wg = q4k.gen_q4k_torch(hi - lo, K, generator=gw, device=dev) if glu else None
                ents.append(dict(name=name, W=W, W_gate=Wg, glu=glu, x=xs[a], a=a, rows=rows, K=K, lo=lo,
                                 n=hi - lo, per=per))
            if peer:
                # full outputs live in the shared buffer; each rank writes its rows
                # there and the kernel stores them into every peer's buffer too
                outs, ybuf0 = [], base
                for e in ents:
                    full = self.pg.out[base: base + e["rows"] * ncols].view(ncols, e["rows"])
                    e["full"] = full
                    outs.append(full[:, e["lo"]: e["lo"] + e["n"]])
                    e["stride"] = e["rows"]
                    base += e["rows"] * ncols
                ybuf, gath = self.pg.out[ybuf0: base], None
            else:
                per_tot = sum(e["per"] for e in ents)
                ybuf = self.y_all[y_off: y_off + per_tot * ncols]
                y_off += -(-per_tot * ncols // 64) * 64
                outs, off = [], 0
                for e in ents:
                    outs.append(ybuf[off: off + e["per"] * ncols].view(ncols, e["per"])[:, : e["n"]])
                    e["stride"] = e["per"]
                    off += e["per"] * ncols
                gath = torch.empty((per_tot * ncols * world,), device=dev) if world > 1 else None
            for e, o in zip(ents, outs):
                e["out"] = o
            if self.q6:
                tasks = q4k.make_tasks_q6_k([e["W"] for e in ents], [e["x"] for e in ents], outs)
                for i, e in enumerate(ents):
                    tasks[i].stride_col_dst = e["stride"]
            elif self.fused:
                tasks = q4k.make_tasks_ex([dict(W=e["W"], W_gate=e["W_gate"], x=e["x"], out=o,
                                                glu=e["glu"] or "none") for e, o in zip(ents, outs)])
                for i, e in enumerate(ents):
                    tasks[i].t.stride_col_dst = e["stride"]
            else:
                tasks = q4k.make_tasks([e["W"] for e in ents], [e["x"] for e in ents], outs)
                for i, e in enumerate(ents):
                    tasks[i].stride_col_dst = e["stride"]
            self.L.append(dict(xs=xs, ents=ents, ybuf=ybuf, tasks=tasks, gath=gath))
        wsb = (q4k.batch_ex_workspace_bytes if self.fused else
               (lambda t, n: int(q4k.lib().q4k_batch_q6_k_workspace_bytes(t, len(t), n))) if self.q6 else
               q4k.batch_workspace_bytes)
        self.ws = q4k.Workspace(max(wsb(G["tasks"], ncols) for G in self.L), dev)
        self.stream = torch.cuda.Stream(device=dev)
        if peer:
            # every rank's buffer starts as NaN, so that no value left from an
            # earlier workload can pass the parity check
            pg.out[:full_elems].fill_(float("nan"))
        # The weights and activations were generated on the default stream; the
        # launches run on self.stream: everything generated (and, row-sharded,
        # every rank's fill) is complete before any launch.
        torch.cuda.synchronize(dev)
        C.barrier()
        self.graph = None
        self.use_graph = not C.args.no_graph
        self.single = C.args.path == "single"
        if self.single and not (self.fused or self.q6):
            self.ws.init(self.stream)  # the single-launch calls need zeroed control words once

    # -- launches ---------------------------------------------------------------
    def gemv(self, tasks):
        q4k, C, ws, s = self.C.q4k, self.C, self.ws, self.stream
        if self.single and not (self.fused or self.q6):
            # one launch per group where the tasks allow it (else two)
            q4k.gemv_batch_persistent(tasks, self.ncols, ws, stream=s, gather=self.pg if C.peer else None)
        elif C.peer:
            q4k.gemv_batch_allgather(tasks, self.ncols, self.pg, ws, stream=s)
        elif self.fused:
            q4k.gemv_batch_ex(tasks, self.ncols, ws, stream=s)
        elif self.q6:
            q4k.gemv_batch_q6_k(tasks, self.ncols, ws, stream=s)
        else:
            q4k.gemv_batch(tasks, self.ncols, ws, stream=s)

    def run_step(self, ev=None):
        C = self.C
        for gi, G in enumerate(self.L):
            if ev is not None:
                ev[gi][0].record(self.stream)
            self.gemv(G["tasks"])
            if ev is not None:
                ev[gi][1].record(self.stream)
            if C.world > 1 and not C.peer:
                C.dist.all_gather_into_tensor(G["gath"], G["ybuf"])
        if C.peer:
            # the step's gathered outputs are complete once this wait has run
            C.q4k.gather_wait(self.pg, self.ws, stream=self.stream)

    def capture(self):
        torch = self.C.torch
        if not self.use_graph:
            return
        try:
            with torch.cuda.stream(self.stream):
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph, stream=self.stream):
                    self.run_step()
        except Exception as e:  # capture unsupported: time eagerly
            print(f"# graph capture failed ({e!r}); timing eager launches", file=sys.stderr)
            self.use_graph, self.graph = False, None

    def replay(self):
        torch = self.C.torch
        with torch.cuda.stream(self.stream):  # replay() launches on the current stream
            if self.use_graph:
                self.graph.replay()
            else:
                self.run_step()

    def status(self) -> int:
        return self.ws.status(self.stream)

    # -- checks -------------------------------------------------------------------
    def parity_check(self, O, nsample: int = 256) -> dict:
        """Row-sharded runs: a seeded sample of nsample rows of every matrix of
        the first and the last launch group, read from this rank's gathered
        output, against the CPU oracle on the same rows.  The sampled rows'
        weights are assembled on every rank from their owners' shards (NCCL
        all-reduce MAX of zero-padded bytes); the oracle is the checker only."""
        C, torch, q4k = self.C, self.C.torch, self.C.q4k
        worst, bad, checked = 0.0, 0, 0
        bad_by_owner = [0] * C.world
        examples = []
        idx_groups = sorted({0, len(self.L) - 1})
        for gi in idx_groups:
            G = self.L[gi]
            for e in G["ents"]:
                rows, K = e["rows"], e["K"]
                rng = np.random.default_rng(rows * 31 + K + gi)
                sel = np.sort(rng.choice(rows, size=min(nsample, rows), replace=False))
                rb = e["W"].shape[1] if e["W"].dim() > 1 else K // 256 * 144
                buf = torch.zeros((len(sel), rb), dtype=torch.uint8, device=C.dev)
                mine = [(i, r - e["lo"]) for i, r in enumerate(sel) if e["lo"] <= r < e["lo"] + e["n"]]
                if mine:
                    ii = torch.tensor([i for i, _ in mine], device=C.dev)
                    rr = torch.tensor([r for _, r in mine], device=C.dev)
                    buf[ii] = e["W"][rr]
                C.dist.all_reduce(buf, op=C.dist.ReduceOp.MAX)
                x = e["x"].cpu().numpy()
                want = O.gemv_f32(buf.cpu().numpy(), x).astype(np.float64)  # (ncols, nsample)
                if C.peer:
                    got = e["full"][:, torch.from_numpy(sel).to(C.dev)].cpu().numpy().astype(np.float64)
                else:  # NCCL gather: rank q's slice at q * per_tot in the gathered buffer
                    per_tot = sum(f["per"] for f in G["ents"])
                    off = 0
                    for f in G["ents"]:
                        if f is e:
                            break
                        off += f["per"] * self.ncols
                    gath = G["gath"].view(C.world, per_tot * self.ncols)
                    got = np.empty((self.ncols, len(sel)))
                    for k, r in enumerate(sel):
                        q, lr = r // e["per"], r % e["per"]
                        part = gath[q, off: off + e["per"] * self.ncols].view(self.ncols, e["per"])
                        got[:, k] = part[:, lr].cpu().numpy()
                err = np.abs(got - want)
                tol = 1e-4 + 1e-5 * np.abs(want)
                nbad = err > tol  # NaN (never written) counts as bad
                nbad |= ~np.isfinite(got)
                bad += int(nbad.sum())
                worst = max(worst, float(np.nanmax(np.where(np.isfinite(got), err / tol, np.inf))))
                checked += err.size
                for j, k in zip(*np.nonzero(nbad)):
                    owner = int(sel[k] // e["per"])
                    bad_by_owner[min(owner, C.world - 1)] += 1
                    if len(examples) < 6:
                        examples.append({"group": gi, "matrix": e["name"], "row": int(sel[k]), "col": int(j),
                                         "owner": owner, "got": float(got[j, k]), "want": float(want[j, k])})
        ok = C.all_ok(bad == 0)
        mine = {"rank": C.rank, "bad": bad, "bad_by_owner_rank": bad_by_owner, "worst_err_over_tol": worst,
                "examples": examples}
        ranks = [mine]
        if C.world > 1:
            ranks = [None] * C.world
            C.dist.all_gather_object(ranks, mine)
        return {"parity": "ok" if ok else "fail", "values_checked_per_rank": checked,
                "groups_checked": idx_groups, "ranks": ranks,
                "bar": "1e-4 abs + 1e-5 rel vs the CPU oracle, 256 seeded rows per matrix"}

    # -- timing -------------------------------------------------------------------
    def time_steps(self, soak_s: float) -> dict:
        """Soak (untimed), warm-up, then the timed steps between CUDA events on
        the launch stream; then one step with events between the launches
        (serialising them) for the isolated-launch time.  Max over ranks."""
        C, torch, args = self.C, self.C.torch, self.C.args
        dev = C.dev
        hs = time.perf_counter()
        if C.world == 1:
            nsoak, t_soak = 0, hs
            while time.perf_counter() - t_soak < soak_s and nsoak < 4000:
                for _ in range(10):
                    self.replay()
                nsoak += 10
                torch.cuda.synchronize(dev)
        elif soak_s > 0:
            # Every rank must replay exactly as many steps as the others: each
            # gathering launch waits (bounded) for its peers' previous launch,
            # so a rank that ran one step more would wait for launches that
            # never come.  The count comes from one timed step, max over ranks.
            C.barrier()
            t0 = time.perf_counter()
            self.replay()
            torch.cuda.synchronize(dev)
            t_one = C.max_over_ranks([time.perf_counter() - t0])[0]
            n = int(min(4000, max(1, soak_s / max(t_one, 1e-6))))
            for i in range(n):
                self.replay()
                if i % 10 == 9:
                    torch.cuda.synchronize(dev)
            torch.cuda.synchronize(dev)
        C.barrier()
        for _ in range(args.warmup):
            self.replay()
        torch.cuda.synchronize(dev)
        C.barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        h0 = time.perf_counter()
        t_start.record(self.stream)
        for _ in range(args.steps):
            self.replay()
        t_end.record(self.stream)
        torch.cuda.synchronize(dev)
        h1 = time.perf_counter()
        C.barrier()
        ms = t_start.elapsed_time(t_end) / args.steps
        # isolated launches (events between launches serialize them); every
        # rank enters together
        C.barrier()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in self.L]
        with torch.cuda.stream(self.stream):
            self.run_step(ev)
        torch.cuda.synchronize(dev)
        st = self.status()
        nrep = len(self.groups) - len(WORKLOADS[self.cfg][3])  # the repeated group only
        iso_ms = float(np.mean([a.elapsed_time(b) for a, b in ev[: max(1, nrep)]]))
        ms, iso_ms, bad = C.max_over_ranks([ms, iso_ms, 1 if st != 0 else 0])
        if bad:
            raise SystemExit(f"device status word reports an error after the timed steps (config {self.cfg})")
        return {"ms": ms, "iso_ms": iso_ms, "hs": hs, "h0": h0, "h1": h1}

    def step_bytes(self) -> int:
        return sum(group_bytes(G, self.ncols, self.C.world) for G in self.groups)

    def kernels(self):
        q4k = self.C.q4k
        try:
            if self.q6:
                return "k_gemv (Q6_K)"
            if self.single and not self.fused:
                ks = sorted({q4k.batch_persistent_kernel(G["tasks"], self.ncols) for G in self.L})
                return [k + (" + gather epilogue" if self.C.peer else "") for k in ks]
            if self.C.peer:
                return "k_gemv (gather epilogue)"
            return sorted({q4k.batch_kernel(G["tasks"], self.ncols) for G in self.L})
        except Exception as e:  # a report, never a reason to lose the measurement
            return f"unknown ({e!r})"

    def free(self):
        C = self.C
        self.graph = None
        C.torch.cuda.synchronize(C.dev)
        C.barrier()
        self.pg = None  # (the run's gather buffer outlives the workload)
        self.L = []
        self.ws = None
        C.torch.cuda.empty_cache()


def summarize(W: Workload, t: dict, peak: float) -> dict:
    world = W.C.world
    total = W.step_bytes()
    nl = len(W.groups)
    return {"workload": W.name, "ncols": W.ncols, "launch_groups": nl, "ms_per_step": t["ms"],
            "us_per_launch": t["ms"] * 1e3 / nl, "us_per_launch_isolated": t["iso_ms"] * 1e3,
            "tbs": total / (t["ms"] * 1e-3) / 1e12,
            "frac": total / world / (t["ms"] * 1e-3) / 1e9 / peak,
            "bytes_per_step": total, "gemv_kernels": W.kernels(), "window": (t["hs"], t["h1"])}


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
    ap.add_argument("--no-per-config", action="store_true", help="measure the headline config only")
    ap.add_argument("--soak-s", type=float, default=0.8,
                    help="untimed replays before the warm-up, seconds (clock sampling window; 0 for profiling runs)")
    ap.add_argument("--path", default="auto", choices=["auto", "single", "two"],
                    help="single: q4k_gemv_batch_persistent (one launch per group where the tasks allow it, "
                         "else two); two: q4k_gemv_batch (quantization launch + GEMV launch); auto (default): "
                         "the one measured faster for the headline, two at one GPU, single row-sharded")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return
    if args.path == "auto":
        args.path = "two" if args.gpus == 1 else "single"

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=120))
    q4k = load_package()
    q4k.lib()
    C = Ctx(args, torch, dist, q4k)
    rank = C.rank
    peak, peak_kind = measured_peaks()
    O = load_oracle() if (world > 1 or (rank == 0 and not args.no_cpu_baseline)) else None

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(C.dev).uuid)
    except AttributeError:
        pass
    sampler = ClockSampler(uuid) if rank == 0 else None
    if sampler:
        sampler.start()

    # ---- one gather buffer for every row-sharded workload of the run ---------
    todo = []
    if not args.no_per_config and args.layers is None:
        todo = [(cfg, nc) for cfg, nc in (PER_CONFIG_1GPU if world == 1 else PER_CONFIG_SHARDED)
                if not (cfg == args.config and nc == args.ncols)]
    pg = None
    if C.peer:
        def outs(cfg, nc, reps):
            _, grps = build_groups(cfg, reps if reps is not None else WORKLOADS[cfg][2])
            return sum(r * nc for grp in grps for _, r, _, _, _ in map(ent, grp))
        pg = q4k.PeerGather(max([outs(args.config, args.ncols, args.layers)] +
                                [outs(cfg, nc, None) for cfg, nc in todo]))

    # ---- headline ------------------------------------------------------------
    W = Workload(C, args.config, args.ncols, args.layers, pg)
    with torch.cuda.stream(W.stream):
        W.run_step()  # one untimed step: checks the device status word before timing
    W.stream.synchronize()
    if int(C.max_over_ranks([1 if W.status() != 0 else 0])[0]):
        raise SystemExit("device status word reports an error")
    parity = W.parity_check(O) if world > 1 else None
    W.capture()
    t = W.time_steps(soak_s=args.soak_s)
    head = summarize(W, t, peak)
    ms = t["ms"]
    ncols = args.ncols
    step_total = W.step_bytes()
    nlaunch = len(W.groups)
    achieved = step_total / world / (ms * 1e-3) / 1e9
    if world == 1:
        launch_bytes = group_bytes(W.groups[0], ncols)
    else:  # this rank's share of the first launch group
        launch_bytes = (sum(wbytes(e["n"], e["K"], e["glu"]) + ncols * e["n"] * 4 for e in W.L[0]["ents"]) +
                        sum(ncols * x.shape[1] * 4 for x in W.L[0]["xs"].values()))

    # ---- e2e: public C-ABI calls with host buffers ---------------------------
    e2e = None
    if not args.no_e2e:
        xs_all = [W.x_all]
        ys_all = [W.pg.out[:W.full_elems]] if C.peer else [W.y_all]
        h_x = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs_all]
        for h, d in zip(h_x, xs_all):
            h.copy_(d)
        h_y = [torch.empty(y.shape, dtype=y.dtype, pin_memory=True) for y in ys_all]
        h2d = sum(h.numel() * 4 for h in h_x)
        d2h = sum(h.numel() * 4 for h in h_y)

        # One GPU: the copies run on a second stream, overlapped with the
        # launches: the activations arrive in three chunks of launch groups
        # (the first group's alone, so the first launch starts after a
        # ~100 KB copy), and the outputs leave in three chunks as their groups
        # complete; the step ends when its last outputs are on the host.
        pipelined = world == 1 and not C.peer and len(W.L) >= 4
        cs = torch.cuda.Stream(device=C.dev)

        def group_range(t0, t1, key):
            """[lo, hi) element range of x_all / y_all used by groups t0..t1-1."""
            views = [v for G in W.L[t0:t1] for v in (G["xs"].values() if key == "x" else [G["ybuf"]])]
            return (min(v.storage_offset() for v in views),
                    max(v.storage_offset() + v.numel() for v in views))

        ng = len(W.L)
        x_chunks = [(a, b) for a, b in [(0, 1), (1, 4), (4, ng)] if a < b]
        y_chunks = [(a, b) for a, b in [(0, ng // 2), (ng // 2, ng - 2), (ng - 2, ng)] if a < b]
        x_rng = [group_range(a, b, "x") for a, b in x_chunks] if pipelined else []
        y_rng = [group_range(a, b, "y") for a, b in y_chunks] if pipelined else []
        if pipelined:  # the bytes the chunks move (the outputs without the buffer's tail padding)
            h2d = sum(hi - lo for lo, hi in x_rng) * 4
            d2h = sum(hi - lo for lo, hi in y_rng) * 4
        ev_x = [torch.cuda.Event() for _ in x_chunks]
        ev_y = [torch.cuda.Event() for _ in y_chunks]

        def e2e_step():
            if not pipelined:
                with torch.cuda.stream(W.stream):
                    for h, d in zip(h_x, xs_all):
                        d.copy_(h, non_blocking=True)
                    W.run_step()
                    for h, d in zip(h_y, ys_all):
                        h.copy_(d, non_blocking=True)
                return
            x_dev, x_host, y_dev, y_host = xs_all[0], h_x[0], ys_all[0], h_y[0]
            cs.wait_stream(W.stream)  # the previous step (launches and copies) is done
            with torch.cuda.stream(cs):
                for (lo, hi), e in zip(x_rng, ev_x):
                    x_dev[lo:hi].copy_(x_host[lo:hi], non_blocking=True)
                    e.record(cs)
            with torch.cuda.stream(W.stream):
                for (a, b), e in zip(x_chunks, ev_x):
                    W.stream.wait_event(e)
                    for gi in range(a, b):
                        W.gemv(W.L[gi]["tasks"])
                        for (ya, yb), (lo, hi), ey in zip(y_chunks, y_rng, ev_y):
                            if gi + 1 == yb:
                                ey.record(W.stream)
                                cs.wait_event(ey)
                                with torch.cuda.stream(cs):
                                    y_host[lo:hi].copy_(y_dev[lo:hi], non_blocking=True)
            W.stream.wait_stream(cs)  # the step ends with its outputs on the host

        for _ in range(args.warmup):
            e2e_step()
        C.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(W.stream)
        for _ in range(args.steps):
            e2e_step()
        b.record(W.stream)
        torch.cuda.synchronize(C.dev)
        e_ms = C.max_over_ranks([a.elapsed_time(b) / args.steps])[0]
        e2e = {"value": step_total / (e_ms * 1e-3) / 1e12, "unit": "TB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "path": ("batch C-ABI calls (ctypes), one per launch group, eager (no graph); every step all its "
                        "activations copied pinned host -> device in 3 chunks of launch groups on a copy stream "
                        "(group 0, groups 1-3, the rest), each chunk before its groups' calls, and all its outputs "
                        "copied device -> pinned host in 3 chunks as their groups complete; the step ends when the "
                        "last outputs are on the host" if pipelined else
                        "batch C-ABI calls (ctypes), one per launch group, eager (no graph); every step one copy "
                        "of all its activations pinned host -> device before the calls and one copy of all its "
                        "outputs device -> pinned host after them" +
                        ("; the gather wait before the copy back" if C.peer else ""))}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        g0 = W.groups[0]
        mats = [(M.cpu().numpy(), e["K"], a, e["glu"] == "q6")
                for e, (_, _, _, a, _) in zip(W.L[0]["ents"], map(ent, g0))
                for M in (e["W"], e["W_gate"]) if M is not None]
        cpu = cpu_baseline(O, mats, g0, ncols)
    kernels = W.kernels()
    wname, full_run, shapes = W.name, W.full_run, sorted({f"{r}x{K}" for grp in W.groups
                                                          for _, r, K, _, _ in map(ent, grp)})
    fused, peer = W.fused, C.peer
    single_all = isinstance(kernels, list) and all("single launch" in k for k in kernels)
    W.free()
    del W

    # ---- the other BASELINE configs ------------------------------------------
    per_config = {}
    if todo:
        for cfg, nc in todo:
            key = f"{cfg}" if cfg != "3" else f"3/ncols={nc}"
            try:
                Wc = Workload(C, cfg, nc, None, pg)
                with torch.cuda.stream(Wc.stream):
                    Wc.run_step()
                Wc.stream.synchronize()
                if int(C.max_over_ranks([1 if Wc.status() != 0 else 0])[0]):
                    raise RuntimeError("device status word reports an error")
                par = Wc.parity_check(O) if world > 1 else None
                Wc.capture()
                tc = Wc.time_steps(soak_s=min(0.3, args.soak_s))
                per_config[key] = summarize(Wc, tc, peak)
                if par is not None:
                    per_config[key]["parity"] = par
                Wc.free()
                del Wc
            except Exception as e:  # one config's failure must not lose the headline
                per_config[key] = {"error": repr(e)[:300]}
                torch.cuda.synchronize(C.dev)

    if sampler:
        sampler.stop()
    win = "untimed soak of step replays + warm-up + timed steps"
    clocks = sampler.summary(t["hs"], t["h1"], win) if sampler else None
    for v in per_config.values():
        w = v.pop("window", None)
        if w is not None:
            v["clocks"] = sampler.summary(w[0], w[1], win) if sampler else None
    if rank == 0:
        traffic = None
        tf = PROFILES / "gemv_layer_traffic.json"
        if tf.exists() and world == 1 and args.config == "2":
            d = json.loads(tf.read_text())
            if d.get("ncols") == ncols:
                traffic = d.get("dram_bytes_per_launch")
        line = {
            "metric": METRIC, "value": head["tbs"], "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded, generated on the device)",
            "config": {"workload": wname if full_run else f"{wname} (profiling subset)",
                       "baseline_config": args.config, "launch_groups": nlaunch, "shapes": shapes,
                       "ncols": ncols, "gemv_kernels": kernels,
                       "path": args.path,
                       "launches": ("per group: one persistent GEMV launch over the group's matrices whose CTAs "
                                    "quantize the activations into shared memory (two launches where that mode "
                                    "does not apply)" if args.path == "single" else
                                    "per group: q8_1 quantization launch + persistent GEMV launch over the group's "
                                    "matrices") + ", chained with programmatic dependencies" + (
                                       "; ffn gate+up as one task with the SwiGLU epilogue" if fused else ""),
                       "timing": "one CUDA graph per step, CUDA events on the launch stream around all timed steps",
                       "l2": "inputs larger than L2 (weights per step >= 3x the 126 MB L2), no flush needed",
                       "parallelism": "single GPU" if world == 1 else (
                           f"row-shard x{world}, outputs stored into every rank's buffer inside the GEMV over "
                           f"NVLink peer stores" if peer else f"row-shard x{world} + NCCL all-gather per launch")},
            "us_per_call": ms * 1e3 / nlaunch,
            "us_per_launch_isolated": head["us_per_launch_isolated"],
            "pct_hbm_peak": 100.0 * achieved / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": f"{', '.join(kernels) if isinstance(kernels, list) else kernels}: "
                                   "every launch of the step, each with its quantization step; "
                                   "achieved = step bytes per rank / step time",
                         "algorithmic_bytes_per_launch": launch_bytes,
                         "launch_isolated_gbs": launch_bytes / (head["us_per_launch_isolated"] * 1e-6) / 1e9},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": args.steps * nlaunch * (1 if single_all else 2) + (args.steps if peer else 0),
            "graph": not args.no_graph,
            "per_config": per_config,
        }
        if parity is not None:
            line["parity"] = parity["parity"]
            line["parity_detail"] = parity
        print(json.dumps(line), flush=True)

    if world > 1:
        torch.cuda.synchronize(C.dev)
        dist.barrier()
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Launch timeline of a decode step: where the time between the weight
streams goes.

Runs one of bench.py's Q4_K workloads through q4k_gemv_batch with the
timeline build of the library (libq4k_gemv_timeline.so, `make timeline`),
captured in one CUDA graph and replayed, and summarises the device-clock
stamps every launch leaves (include/q4k_gemv.h, q4k_timeline_*):

  per launch   quantization launch: release after the previous GEMV's end,
               run time; GEMV: release after the quantization launch, the
               spread of the workers' end times after the release
  per ring     mean end of the workers of each ring slot of a CTA
  per CTA      mean end by CTA index (CTAs are dispatched in index order)

    python tests/timeline_driver.py --config 2 [--ncols N] [--reverse] [--json] [--save F.npz]

A diagnostic driver kept beside the test that checks its output
(tests/test_gpu_timeline.py); not part of the library.

The reference's own tracing was Nsight plus in-kernel clock64 probes left
commented out (w_tile.cu:76-122); this is the same question asked of the
persistent launch chain.  Q4_K batches (the quantization launch and
k_gemv; groups with a fused gate/up entry through q4k_gemv_batch_ex);
numbers are from the timeline build, whose stamps cost a few stores per
warp.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
HERE = ROOT / "gemv-q4_k-optimization_b200"
os.environ.setdefault("Q4K_LIB", str(HERE / "libq4k_gemv_timeline.so"))
sys.path.insert(0, str(ROOT))


def build_step(q4k, bench, torch, cfg: str, ncols: int, reverse: bool, dev):
    """The workload's launches; a group with a fused gate/up entry becomes a
    q4k_gemv_batch_ex launch (fused=True)."""
    _, groups = bench.build_groups(cfg, bench.WORKLOADS[cfg][2])
    if any(glu == "q6" for grp in groups for *_, glu in map(bench.ent, grp)):
        raise SystemExit(f"config {cfg}: Q4_K batches only")
    if reverse:
        groups = [list(reversed(g)) for g in groups]
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    launches = []
    for grp in groups:
        xs, items = {}, []
        for _, rows, K, a, glu in map(bench.ent, grp):
            if a not in xs:
                xs[a] = torch.randn((ncols, K), device=dev, generator=g)
            W = q4k.gen_q4k_torch(rows, K, generator=g, device=dev)
            Wg = q4k.gen_q4k_torch(rows, K, generator=g, device=dev) if glu else None
            items.append(dict(W=W, W_gate=Wg, x=xs[a], out=torch.empty((ncols, rows), device=dev),
                              glu=glu or "none"))
        fused = any(it["W_gate"] is not None for it in items)
        tasks = (q4k.make_tasks_ex(items) if fused else
                 q4k.make_tasks([it["W"] for it in items], [it["x"] for it in items], [it["out"] for it in items]))
        launches.append(dict(tasks=tasks, fused=fused, keep=(items, xs), names=[e[0] for e in grp]))
    return launches


def summarize(G, Pr, n, single=False):
    """Per-launch and aggregate figures (us) from the records of slots 0..n-1.
    single: launches of the single-launch mode (no quantization launch; words
    6 and 7 of a warp's record hold its quantization end and plan time)."""
    per = []
    for i in range(n):
        # worker records: word 3 (atoms computed) > 0; records 15 and 14 of a
        # CTA are its folding and flushing warps (word 3 = 0); the flushing
        # warp writes the last row groups
        cta, warp = np.nonzero(G[i][:, :, 3] > 0)
        w = G[i][cta, warp]
        fold = G[i][:, 14]
        fold = fold[(fold[:, 0] > 0) & (fold[:, 3] == 0)]
        p = Pr[i][Pr[i][:, 3] == 1]
        if len(w) == 0 or (len(p) == 0 and not single):
            raise SystemExit(f"launch {i}: no records (was the timeline library loaded?)")
        rel = w[:, 1].min()
        end_all = max(w[:, 2].max(), fold[:, 2].max()) if len(fold) else w[:, 2].max()
        d = dict(gemv_release=rel, gemv_end=end_all, ends=np.sort(w[:, 2] - rel) / 1e3,
                 end=(w[:, 2] - rel) / 1e3, cta=cta, warp=warp, start_min=w[:, 0].min(),
                 fold_end=(fold[:, 2] - rel) / 1e3 if len(fold) else None)
        if single:
            d.update(quant=(w[:, 6] - w[:, 1]) / 1e3, plan=(w[:, 7] - w[:, 0]) / 1e3)
            # phases in the records of warp + 8 (warps 0..5): plan barrier,
            # status barrier, quantizer end
            m = warp < 6
            dd = G[i][cta[m], warp[m] + 8]
            if m.any() and dd[:, 0].min() > 0:
                wm = w[m]
                d.update(ph_sync1=(dd[:, 0] - wm[:, 1]) / 1e3, ph_sync2=(dd[:, 1] - dd[:, 0]) / 1e3,
                         ph_quant=(dd[:, 2] - dd[:, 1]) / 1e3, ph_sync3=(wm[:, 6] - dd[:, 2]) / 1e3)
        else:
            d.update(prep_release=p[:, 1].min(), prep_end=p[:, 2].max())
        per.append(d)
    rows = []
    for i in range(1, n):
        a, b = per[i - 1], per[i]
        r = dict(launch=i, period=(b["gemv_end"] - a["gemv_end"]) / 1e3)
        if single:
            r.update(prev_end_to_release=(b["gemv_release"] - a["gemv_end"]) / 1e3,
                     quant_p50=float(np.percentile(b["quant"], 50)), quant_max=float(b["quant"].max()),
                     plan_max=float(b["plan"].max()))
            for k in ("ph_sync1", "ph_sync2", "ph_quant", "ph_sync3"):
                if k in b:
                    r[k + "_p50"] = float(np.percentile(b[k], 50))
                    r[k + "_max"] = float(b[k].max())
        else:
            r.update(prev_end_to_prep_release=(b["prep_release"] - a["gemv_end"]) / 1e3,
                     prep_run=(b["prep_end"] - b["prep_release"]) / 1e3,
                     prep_end_to_gemv_release=(b["gemv_release"] - b["prep_end"]) / 1e3)
        r.update(end_p10=float(np.percentile(b["ends"], 10)), end_p50=float(np.percentile(b["ends"], 50)),
                 end_p90=float(np.percentile(b["ends"], 90)), end_max=float(b["ends"][-1]))
        if b["fold_end"] is not None:
            r.update(fold_end_p50=float(np.percentile(b["fold_end"], 50)), fold_end_max=float(b["fold_end"].max()))
        rows.append(r)
    # (launches of a mixed workload differ in their keys: the flushing warp's
    # end exists for the launches with a fused task only)
    keys = [k for k in dict.fromkeys(k for r in rows for k in r) if k != "launch"]
    mean = {k: float(np.mean([r[k] for r in rows if k in r])) for k in keys}
    # worker end times by warp (ring slot of the CTA) and by CTA index, launches 1..n-1
    end = np.concatenate([r["end"] for r in per[1:]])
    warp = np.concatenate([r["warp"] for r in per[1:]])
    cta = np.concatenate([r["cta"] for r in per[1:]])
    ring = {int(k): float(end[warp == k].mean()) for k in np.unique(warp)}
    ncta = int(cta.max()) + 1
    bins = {}
    for lo in range(0, ncta, 16):
        m = (cta >= lo) & (cta < lo + 16)
        bins[f"{lo}-{min(lo + 16, ncta) - 1}"] = float(end[m].mean())
    return rows, mean, ring, bins


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="2")
    ap.add_argument("--ncols", type=int, default=1)
    ap.add_argument("--reverse", action="store_true", help="reverse the task order inside each launch")
    ap.add_argument("--replays", type=int, default=3)
    ap.add_argument("--json", action="store_true", help="print one JSON line instead of tables")
    ap.add_argument("--save", default=None, help="also write the raw records of the step (.npz)")
    ap.add_argument("--single", action="store_true",
                    help="q4k_gemv_batch_persistent (single-launch mode) instead of the two-launch calls")
    args = ap.parse_args()

    import torch
    import bench
    q4k = bench.load_package()
    if q4k.lib().q4k_timeline_bytes() == 0:
        raise SystemExit(f"{q4k.LIB_PATH} is not a timeline build (make -C {HERE} timeline)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    launches = build_step(q4k, bench, torch, args.config, args.ncols, args.reverse, dev)
    if len(launches) > q4k.TL_SLOTS:
        raise SystemExit(f"{len(launches)} launches per step > {q4k.TL_SLOTS} timeline slots")
    if args.single and any(L["fused"] for L in launches):
        raise SystemExit("--single: plain Q4_K batches only")
    ws = q4k.Workspace(max((q4k.batch_ex_workspace_bytes if L["fused"] else q4k.batch_workspace_bytes)(
        L["tasks"], args.ncols) for L in launches), dev)
    stream = torch.cuda.Stream(device=dev)

    if args.single:
        ws.init(stream)

    def step():
        for L in launches:
            if args.single:
                q4k.gemv_batch_persistent(L["tasks"], args.ncols, ws, stream=stream)
            elif L["fused"]:
                q4k.gemv_batch_ex(L["tasks"], args.ncols, ws, stream=stream)
            else:
                q4k.gemv_batch(L["tasks"], args.ncols, ws, stream=stream)

    for _ in range(3):
        step()
    torch.cuda.synchronize(dev)
    q4k.timeline_reset()  # the graph's launches take slots 0..n-1
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.replays):
        graph.replay()
    torch.cuda.synchronize(dev)
    G, Pr, ncalls = q4k.timeline_read()
    n = len(launches)
    if args.save:
        np.savez_compressed(args.save, gemv=G[:n], prep=Pr[:n])
    rows, mean, ring, cta = summarize(G, Pr, n, args.single)
    out = {"config": args.config, "ncols": args.ncols, "reverse": args.reverse, "single": args.single,
           "launches": n,
           "mean_us": {k: round(v, 3) for k, v in mean.items()},
           "ring_mean_end_us": {k: round(v, 3) for k, v in ring.items()},
           "cta_mean_end_us": {k: round(v, 3) for k, v in cta.items()}}
    if args.json:
        print(json.dumps(out))
        return
    print(f"config {args.config}, ncols {args.ncols}, {n} launches per step, graph replay; us")
    keys = list(mean)
    print("launch  " + "  ".join(keys))
    for r in rows:
        print(f"{r['launch']:6d} " + "  ".join(f"{r[k]:7.2f}" if k in r else "      -" for k in keys))
    print("mean   " + "  ".join(f"{k} {v:.2f}" for k, v in mean.items()))
    print("mean worker end by ring slot: " + "  ".join(f"{k}:{v:.2f}" for k, v in ring.items()))
    print("mean worker end by CTA index: " + "  ".join(f"{k}:{v:.2f}" for k, v in cta.items()))


if __name__ == "__main__":
    main()

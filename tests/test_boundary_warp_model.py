"""CPU model of the boundary warp's hand-off rule (plain and single-launch
k_gemv variants).

A compute warp walks its atom range [a0, a1) (odd workers backwards) and
flushes each row group when its cursor leaves it.  A flushed group that
other workers share is a "split" group; if one of those workers is in
another CTA (or the launch is not packed CTA-major) the group needs a
device-scope arrival.  The compute warp hands such a group to the CTA's
boundary warp when it flushes it before its last atom (slot 0: the group it
began inside; slot 1: the group it ends inside); its last group it flushes
itself.  The boundary warp never sees the compute warp's walk: it derives
from the atom ranges alone which (ring, slot) entries will come and after
how many of the warp's atoms, and waits for them in that order, each on its
own mbarrier.  If the two sides disagreed, an expected entry that never
comes would end in the 2 s bounded wait (Q4K_ETIMEOUT), and an entry that is
not expected would leave its row group without its last arrival.

This test runs both sides of the rule (restated from
gemv-q4_k-optimization_b200/csrc/q4k_kernels.cu: worker_begin, worker_of,
locate_atom, walks_back, flush_values' slot and locality, the boundary
warp's expectation) over random task lists and partitions, and checks that
they agree entry for entry, key for key.
"""
from __future__ import annotations

import random


def worker_begin(natoms, nworkers, w):
    return natoms * w // nworkers


def worker_of(natoms, nworkers, a):
    return ((a + 1) * nworkers - 1) // natoms


def group_of(tasks, a):
    """(start, end) atoms of the row group holding atom a (locate_atom)."""
    t = 0
    while t + 1 < len(tasks) and a >= tasks[t + 1][0]:
        t += 1
    base, apr = tasks[t]
    g = (a - base) // apr
    return base + g * apr, base + (g + 1) * apr


def compute_warp_handoffs(tasks, natoms, nworkers, wk, cta_w0, cta_w1, packed):
    """What the compute warp hands over: {slot: atoms processed when flushed}."""
    a0, a1 = worker_begin(natoms, nworkers, wk), worker_begin(natoms, nworkers, wk + 1)
    back = (wk & 1) == 1
    order = range(a1 - 1, a0 - 1, -1) if back else range(a0, a1)
    flushes, cur, done = [], None, 0
    for a in order:
        grp = group_of(tasks, a)
        if cur is not None and grp != cur:
            flushes.append((cur, done))  # flushed when the cursor leaves it
        cur = grp
        done += 1
    if cur is not None:
        flushes.append((cur, None))      # the last group: flushed by the warp itself
    out = {}
    for (sg, eg), at in flushes:
        if sg >= a0 and eg <= a1:
            continue                     # whole group in this worker: no hand-off
        slot = 0 if a0 > sg else 1
        w1, w2 = worker_of(natoms, nworkers, sg), worker_of(natoms, nworkers, eg - 1)
        local = packed and w1 >= cta_w0 and w2 <= cta_w1
        if at is not None and not local:
            assert slot not in out, "two entries in one slot"
            out[slot] = at
    return out


def boundary_expects(tasks, natoms, nworkers, wk, cta_w0, cta_w1, packed):
    """What the boundary warp expects, from the atom range alone."""
    a0, a1 = worker_begin(natoms, nworkers, wk), worker_begin(natoms, nworkers, wk + 1)
    out = {}
    if a1 <= a0:
        return out
    back = (wk & 1) == 1
    for e in (0, 1):
        sg, eg = group_of(tasks, a0 if e == 0 else a1 - 1)
        split = sg < a0 if e == 0 else (sg >= a0 and eg > a1)
        at = ((a1 - a0) if back else min(eg, a1) - a0) if e == 0 else ((a1 - sg) if back else (a1 - a0))
        if split and at < a1 - a0:
            w1, w2 = worker_of(natoms, nworkers, sg), worker_of(natoms, nworkers, eg - 1)
            if not (packed and w1 >= cta_w0 and w2 <= cta_w1):
                out[e] = at
    return out


def test_boundary_warp_expectations_match_the_compute_warps():
    rng = random.Random(2026)
    checked = handed = 0
    for _ in range(4000):
        tasks, base = [], 0
        for _ in range(rng.randint(1, 7)):
            apr = rng.choice([1, 2, 3, 8, 28, 56])   # atoms per row group (K = 4096: 8, 14336: 28)
            tasks.append((base, apr))
            base += apr * rng.randint(1, 40)
        natoms = base
        rings, grid = rng.randint(1, 8), rng.randint(1, 24)
        nworkers = rings * grid
        packed = rng.random() < 0.5
        for cta in range(grid):
            cta_w0, cta_w1 = cta * rings, cta * rings + rings - 1
            for ring in range(rings):
                wk = cta * rings + ring if packed else ring * grid + cta
                got = compute_warp_handoffs(tasks, natoms, nworkers, wk, cta_w0, cta_w1, packed)
                want = boundary_expects(tasks, natoms, nworkers, wk, cta_w0, cta_w1, packed)
                assert got == want, (tasks, natoms, nworkers, wk, packed, got, want)
                n = worker_begin(natoms, nworkers, wk + 1) - worker_begin(natoms, nworkers, wk)
                assert all(0 < k < n for k in got.values())
                checked += 1
                handed += len(got)
    assert checked > 10000 and handed > 1000


def test_mistral_layer_hand_offs():
    """The Mistral-7B layer launch (7 matrices, 148 CTAs x 8 rings, packed):
    only groups at CTA boundaries are handed over (a few per CTA, none of
    them a warp's last flush), in the 8-atom and in the 28-atom (down)
    matrices alike."""
    rows_k = [(4096, 16), (1024, 16), (1024, 16), (4096, 16), (14336, 16), (14336, 16), (4096, 56)]
    tasks, base = [], 0
    for rows, nb in rows_k:
        apr = nb // 2                         # atoms of 2 super-blocks per 32-row group
        tasks.append((base, apr))
        base += apr * (rows // 32)
    natoms, rings, grid = base, 8, 148
    nworkers = rings * grid
    down_start = tasks[-1][0]
    early = down = 0
    for cta in range(grid):
        per_cta = 0
        for ring in range(rings):
            wk = cta * rings + ring
            got = boundary_expects(tasks, natoms, nworkers, wk, cta * rings, cta * rings + rings - 1, True)
            assert got == compute_warp_handoffs(tasks, natoms, nworkers, wk, cta * rings, cta * rings + rings - 1,
                                                True)
            n = worker_begin(natoms, nworkers, wk + 1) - worker_begin(natoms, nworkers, wk)
            assert all(k < n for k in got.values())
            per_cta += len(got)
            if worker_begin(natoms, nworkers, wk) >= down_start:
                down += len(got)
            else:
                early += len(got)
        assert per_cta <= 4
    assert early > 100 and down > 0

"""A CPU model of the dynamically scheduled GEMV's control flow (k_gemv_dyn in
gemv-q4_k-optimization_b200/csrc/q4k_kernels.cu): the per-CTA queue of row
groups (static first entries, ticket claims published two groups ahead, one
mbarrier phase per slot use), each warp's copy and sum cursors over its
share of every group, the double-buffered partial sums and their "buffer
free" barrier.  Every warp is a generator that yields a predicate where the
kernel would wait; a seeded random scheduler interleaves the warps of
several CTAs, and bulk copies land after random delays.

Checked over random geometries: no deadlock, every row group added up
exactly once, and every reduction sees the R shares of that group.  A
variant whose copy cursor reads the next queue entry eagerly (as soon as it
passes its last atom of a group) deadlocks: warp 0 then waits for an entry
that only it publishes, which is why the kernel reads entries lazily.
"""
from __future__ import annotations

import random

# kStages, kDynQ, kDynAhead of the kernel
KSTAGES, KQ, KAHEAD = 2, 16, 3


class Bar:
    """An mbarrier: arrival count and completed phases."""

    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        """try_wait.parity: has the phase of this parity completed?"""
        return (self.phase & 1) != parity


def run(G, grid, R, aprs, seed, eager=False):
    rnd = random.Random(seed)
    counter = [0]
    reduced = {}
    def apr_of(gi): return aprs[gi % len(aprs)]
    warps = []
    for cta in range(grid):
        sh = dict(q_group=[None]*KQ, q_bar=[Bar(1) for _ in range(KQ)], free_bar=[Bar(1), Bar(1)],
                  red_cnt=[0, 0], part=[[None]*R for _ in range(2)], full=[[False]*KSTAGES for _ in range(R)],
                  fullbar=[[Bar(1) for _ in range(KSTAGES)] for _ in range(R)])
        for w in range(R):
            warps.append(warp_gen(cta, w, sh, G, grid, R, apr_of, counter, reduced, rnd, eager))
    live = list(range(len(warps))); waits = {}
    steps = 0
    while live:
        steps += 1
        if steps > 10**7: return "too many steps"
        runnable = [i for i in live if waits.get(i) is None or waits[i]()]
        if not runnable: return f"DEADLOCK with {len(live)} warps waiting"
        i = rnd.choice(runnable)
        try:
            waits[i] = next(warps[i])
        except StopIteration:
            live.remove(i); waits.pop(i, None)
    for g in range(G):
        if reduced.get(g) != 1: return f"group {g} reduced {reduced.get(g)} times"
    return "ok"

def warp_gen(cta, warp, sh, G, grid, R, apr_of, counter, reduced, rnd, eager=False):
    producer = warp == 0
    def entry(k):
        if k < KAHEAD:
            gi = cta + k * grid
            return gi if gi < G else -1
            yield
        slot = k % KQ; par = (k // KQ) & 1
        yield lambda: sh['q_bar'][slot].done(par)
        return sh['q_group'][slot]
    def enter(k, gi):
        d = dict(k=k, gi=gi, need=False)
        if gi < 0: return d
        a = apr_of(gi)
        d['kp'] = warp * a // R; d['s1'] = (warp + 1) * a // R
        assert d['s1'] > d['kp']
        return d
    def step(d):
        d['kp'] += 1
        if d['kp'] == d['s1']: d['need'] = True
    def resolve(d):
        if not d['need'] or d['gi'] < 0: return d
        gi = yield from entry(d['k'] + 1)
        return enter(d['k'] + 1, gi)
    fb = sh['fullbar'][warp]
    def issue(n):  # TMA lands some time later: model as arrive after a random delay via a pending list
        s = n % KSTAGES
        pend_tma.append((s, rnd.randint(0, 20)))
    pend_tma = []
    def tick():
        for idx in range(len(pend_tma)):
            s, t = pend_tma[idx]
            pend_tma[idx] = (s, t - 1)
        for (s, t) in [x for x in pend_tma if x[1] <= 0]:
            fb[s].arrive(); pend_tma.remove((s, t))
    if producer:
        for e in range(KAHEAD):
            gi = cta + e * grid
            sh['q_group'][e] = gi if gi < G else -1; sh['q_bar'][e].arrive()
    yield None
    ic = enter(0, cta if cta < G else -1); cc = dict(ic)
    issued = 0
    while issued < KSTAGES:
        if ic['need'] and ic['k'] + 1 >= KAHEAD: break
        ic = yield from resolve(ic)
        if ic['gi'] < 0 or ic['k'] >= KAHEAD: break
        issue(issued); issued += 1; step(ic)
    yield None  # pdl_wait
    pend = 0
    filled = KAHEAD
    claiming = producer and (cta + (KAHEAD - 1) * grid) < G
    while issued < KSTAGES:
        ic = yield from resolve(ic)
        if ic['gi'] < 0: break
        issue(issued); issued += 1; step(ic)
    done = 0; group_k = -1
    while cc['gi'] >= 0:
        if producer and cc['k'] != group_k:
            group_k = cc['k']
            if claiming and cc['k'] >= 1:
                gi = grid * KAHEAD + pend; e = filled; filled += 1
                sh['q_group'][e % KQ] = gi if gi < G else -1; sh['q_bar'][e % KQ].arrive()
                claiming = gi < G
            if claiming:
                pend = counter[0]; counter[0] += 1
            yield None
        s = done % KSTAGES; par = (done // KSTAGES) & 1
        while not fb[s].done(par):
            tick(); yield None
        # compute
        ic = yield from resolve(ic)
        if ic['gi'] >= 0:
            issue(issued); issued += 1; step(ic)
            if eager:
                ic = yield from resolve(ic)
        done += 1
        tick()
        cc['kp'] += 1
        if cc['kp'] < cc['s1']:
            yield None; continue
        b = cc['k'] & 1; use = cc['k'] >> 1
        if use >= 1:
            par2 = (use - 1) & 1
            while not sh['free_bar'][b].done(par2):
                tick(); yield None
        sh['part'][b][warp] = cc['gi']
        yield None
        old = sh['red_cnt'][b]; sh['red_cnt'][b] += 1
        if old == R - 1:
            assert all(p == cc['gi'] for p in sh['part'][b]), ("partials of other groups", sh['part'][b], cc['gi'])
            reduced[cc['gi']] = reduced.get(cc['gi'], 0) + 1
            yield None
            sh['red_cnt'][b] = 0; sh['free_bar'][b].arrive()
        gi = yield from entry(cc['k'] + 1)
        cc = enter(cc['k'] + 1, gi)
        yield None
    while pend_tma:
        tick(); yield None



def _geometry(seed):
    rnd = random.Random(seed)
    R = rnd.choice([2, 3, 4, 7, 8])
    grid = rnd.choice([1, 2, 3, 5])
    G = rnd.randint(KAHEAD * grid, KAHEAD * grid + 40)
    aprs = [max(rnd.choice([R, R + 1, 2 * R, 3 * R + 1, 28]), R) for _ in range(3)]
    return G, grid, R, aprs


def test_protocol_completes_every_group_once():
    for seed in range(500):
        G, grid, R, aprs = _geometry(seed)
        assert run(G, grid, R, aprs, seed) == "ok", (seed, G, grid, R, aprs)


def test_eager_entry_reads_deadlock():
    results = [run(*_geometry(seed), seed, eager=True) for seed in range(60)]
    assert any(r.startswith("DEADLOCK") for r in results)

# SPDX-License-Identifier: Apache-2.0
"""Model checks of the device-side synchronisation protocols (CPU).

The fused kernels and the LL collectives coordinate ranks with monotonic
counters and epoch flags instead of barriers.  These tests re-state each
protocol as small cooperating processes (one per rank x CTA role) that run
under many random interleavings, with back-to-back calls and no host
synchronisation between them, and check

* liveness: every schedule completes (no wait is left unsatisfiable), and
* safety: no buffer region is overwritten for call k+1 while a reader of
  call k has not consumed it, and every read sees the data of its own call.

Modelled from the kernels (counter names as in csrc/kernels/device_common.cuh):
  all-gather + GEMM   ready / taken / localReady / staged   (csrc/fused/ag_gemm.cu)
  GEMM + RS           done / free, per-call local counters  (csrc/fused/gemm_rs.cu)
  GEMM + RS on pairs  per-half arrivals, consumed counts, free (csrc/fused/gemm_rs.cu, one kernel)
  both forms mixed    the two GEMM + RS forms alternating call by call on shared counters
  its tile walk       every pair's tile order and the accumulator-stage coupling of a CTA pair,
                      run to a fixed point for cycles of waits (csrc/kernels/gemm_sm100_pair.cuh)
  LL one-shot         per-block epochs, parity slots        (csrc/kernels/ll.cuh)
  MoE dispatch        count-matrix exchange, done counters  (csrc/fused/moe.cu)
Stream order is modelled too: a rank's kernel for call k+1 starts only after
every process of its kernel for call k has finished.
"""

import random
from collections import defaultdict

import pytest


class Deadlock(Exception):
    pass


class Sim:
    """Processes are generators yielding predicates (callables -> bool); a
    process runs until its next predicate, and the scheduler advances a
    random process whose predicate holds."""

    def __init__(self, seed):
        self.rng = random.Random(seed)
        self.procs = []  # [gen, pred]

    def spawn(self, gen):
        pred = next(gen, None)
        if pred is not None:
            self.procs.append([gen, pred])

    def run(self, max_steps=200000):
        steps = 0
        while self.procs:
            ready = [p for p in self.procs if p[1]()]
            if not ready:
                raise Deadlock(f"{len(self.procs)} processes blocked")
            p = self.rng.choice(ready)
            nxt = next(p[0], None)
            if nxt is None:
                self.procs.remove(p)
            else:
                p[1] = nxt
            steps += 1
            if steps > max_steps:
                raise Deadlock("step limit")


def kernel_chain(sim, calls, make_kernel):
    """Stream order on one rank: kernel k+1's processes start after kernel k's end."""
    def driver():
        for k in range(calls):
            live = make_kernel(k)
            for g in live["procs"]:
                sim.spawn(g)
            yield lambda: live["done"] == live["count"]
    return driver()


# ---------------------------------------------------------------------------
# all-gather + GEMM
# ---------------------------------------------------------------------------
def run_ag_gemm(n, ctas, calls, seed):
    sim = Sim(seed)
    ready = defaultdict(int)        # (at rank, of rank q)
    taken = defaultdict(int)        # (at rank, by rank p)
    local_ready = defaultdict(int)  # (at rank, shard q)
    staged = defaultdict(int)       # at rank
    # xfull[(owner, shard, slice)] = (call whose data it holds)
    xfull = {}
    errors = []

    def make_kernel(r):
        def mk(k):
            live = {"done": 0, "count": 2 * ctas}

            def copy_warps(j):
                yield lambda: all(taken[(r, p)] >= k for p in range(n) if p != r)
                # stage my slice of my shard (peers read it from my buffer)
                xfull[(r, r, j)] = k
                staged[r] += 1
                if staged[r] == (k + 1) * ctas:
                    for p in range(n):
                        ready[(p, r)] += 1
                for s in range(1, n):
                    q = (r + s) % n
                    yield lambda q=q: ready[(r, q)] >= k + 1
                    yield lambda: True  # the pull happens some time after the flag was seen
                    v = xfull.get((q, q, j))
                    if v != k:
                        errors.append(f"rank {r} call {k} pulled shard {q} slice {j} holding call {v}")
                    xfull[(r, q, j)] = k
                    local_ready[(r, q)] += 1
                    if local_ready[(r, q)] == (k + 1) * ctas:
                        taken[(q, r)] += 1
                live["done"] += 1

            def producer(j):
                # tiles of every shard, own shard first (grouped order)
                for s in range(n):
                    q = (r + s) % n
                    if q == r:
                        yield lambda: ready[(r, r)] >= k + 1
                    else:
                        yield lambda q=q: local_ready[(r, q)] >= (k + 1) * ctas
                    yield lambda: True
                    for sl in range(ctas):
                        v = xfull.get((r, q, sl))
                        if v != k:
                            errors.append(f"rank {r} call {k} GEMM read shard {q} slice {sl} holding call {v}")
                live["done"] += 1

            live["procs"] = [copy_warps(j) for j in range(ctas)] + [producer(j) for j in range(ctas)]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make_kernel(r)))
    sim.run()
    return errors


# ---------------------------------------------------------------------------
# GEMM + reduce-scatter
# ---------------------------------------------------------------------------
def run_gemm_rs(n, ctas, blocks, calls, seed):
    sim = Sim(seed)
    done = defaultdict(int)     # (at owner, from source)
    free = defaultdict(int)     # (at source, from owner)
    local_done = defaultdict(int)
    local_free = defaultdict(int)
    slot = {}                   # (owner, source) -> call of the data pushed there
    errors = []

    def make_gemm(r):
        def mk(k):
            live = {"done": 0, "count": ctas}

            def cta(j):
                # epilogue warps wait until every owner reduced the previous call
                yield lambda: all(free[(r, q)] >= k for q in range(n))
                for q in range(n):
                    slot[(q, r)] = k  # push this CTA's tiles for owner q
                local_done[r] += 1
                if local_done[r] == (k + 1) * ctas:
                    for q in range(n):
                        done[(q, r)] += 1
                live["done"] += 1

            live["procs"] = [cta(j) for j in range(ctas)]
            return live
        return mk

    def make_reduce(r):
        def mk(k):
            live = {"done": 0, "count": blocks}

            def blk(b):
                yield lambda: all(done[(r, p)] >= k + 1 for p in range(n))
                yield lambda: True
                for p in range(n):
                    if slot.get((r, p)) != k:
                        errors.append(f"owner {r} call {k} reduced source {p} holding call {slot.get((r, p))}")
                local_free[r] += 1
                if local_free[r] == (k + 1) * blocks:
                    for q in range(n):
                        free[(q, r)] += 1
                live["done"] += 1

            live["procs"] = [blk(b) for b in range(blocks)]
            return live
        return mk

    def make_call(r):
        gemm, red = make_gemm(r), make_reduce(r)

        def mk(k):
            # the GEMM and the reduction are two kernels of one call on one stream
            live = {"done": 0, "count": 1}

            def seq():
                g = gemm(k)
                for p in g["procs"]:
                    sim.spawn(p)
                yield lambda: g["done"] == g["count"]
                rd = red(k)
                for p in rd["procs"]:
                    sim.spawn(p)
                yield lambda: rd["done"] == rd["count"]
                live["done"] += 1

            live["procs"] = [seq()]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make_call(r)))
    sim.run()
    return errors


# ---------------------------------------------------------------------------
# GEMM + reduce-scatter on CTA pairs, one kernel: senders push 128-row half
# tiles and bump the owner's per-half arrival counter; the owner's epilogue
# waits for consumed + (n - 1) arrivals, reads the slots and records the new
# consumed count; the last CTA of a call frees the owner's slots on every
# rank.  Calls differ in shape (halves per owner), as in the kernel, where
# a call only touches the counters of its own tiles.
# ---------------------------------------------------------------------------
def run_gemm_rs_pair(n, ctas, calls, seed, relative=True, free_wait=True):
    sim = Sim(seed)
    rng = random.Random(seed * 7 + 1)
    halves = [rng.choice([1, 2, 3]) for _ in range(calls)]  # per call, the same on every rank
    arrive = defaultdict(int)    # (owner, half)
    consumed = defaultdict(int)  # (owner, half), local to the owner
    free = defaultdict(int)      # (at source, from owner)
    pair_free = defaultdict(int)
    slot = {}                    # (owner, source, half) -> call pushed there
    unread = set()               # pushed slots the owner has not read yet
    errors = []

    def make_kernel(r):
        def mk(k):
            live = {"done": 0, "count": ctas}
            H = halves[k]
            # rank r's order: owners r+1 .. r-1, its own rows last
            tiles = [((r + 1 + i) % n, h) for i in range(n) for h in range(H)]
            per_cta = [tiles[j::ctas] for j in range(ctas)]

            def cta(j):
                if free_wait:
                    yield lambda: all(free[(r, q)] >= k for q in range(n))
                for q, h in per_cta[j]:
                    if q != r:
                        if (q, r, h) in unread:
                            errors.append(f"rank {r} call {k} overwrote unread slot {(q, r, h)}")
                        slot[(q, r, h)] = k
                        unread.add((q, r, h))
                        yield lambda: True  # the stores and the release are separate steps
                        arrive[(q, h)] += 1
                    else:
                        target = consumed[(r, h)] + (n - 1) if relative else (k + 1) * (n - 1)
                        yield lambda t=target, hh=h: arrive[(r, hh)] >= t
                        for p in range(n):
                            if p != r:
                                if slot.get((r, p, h)) != k:
                                    errors.append(f"owner {r} call {k} half {h} read call {slot.get((r, p, h))} of {p}")
                                unread.discard((r, p, h))
                        consumed[(r, h)] = target
                pair_free[r] += 1
                if pair_free[r] == ctas:
                    pair_free[r] = 0
                    for q in range(n):
                        free[(q, r)] += 1
                live["done"] += 1

            live["procs"] = [cta(j) for j in range(ctas)]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make_kernel(r)))
    sim.run()
    return errors


# ---------------------------------------------------------------------------
# LL one-shot all-reduce (one block; the protocol is per block)
# ---------------------------------------------------------------------------
def next_ll_epoch(e, wrap_to=2):
    """csrc/kernels/ll.cuh llEpoch: 32-bit counter that skips 0 on the wrap."""
    e = (e + 1) & 0xFFFFFFFF
    return wrap_to if e == 0 else e


def run_ll(n, calls, seed, parities=2, start=0, wrap_to=2):
    sim = Sim(seed)
    epoch = defaultdict(lambda: start)  # rank -> epoch of its last LL launch
    slots = {}                 # (dst, parity, src) -> epoch written
    consumed = {}              # (dst, parity, src) -> epoch the reader has taken out
    errors = []

    def make(r):
        def mk(k):
            live = {"done": 0, "count": 1}

            def block():
                epoch[r] = next_ll_epoch(epoch[r], wrap_to)
                e = epoch[r]
                par = e % parities
                for p in range(n):
                    if p != r:
                        prev = slots.get((p, par, r))
                        if prev is not None and consumed.get((p, par, r)) != prev:
                            errors.append(f"rank {r} epoch {e} overwrote unread epoch {prev} at rank {p}")
                        slots[(p, par, r)] = e
                        yield lambda: True
                for p in range(n):
                    if p != r:
                        yield lambda p=p: slots.get((r, par, p)) == e
                        yield lambda: True
                        if slots.get((r, par, p)) != e:
                            errors.append(f"rank {r} epoch {e}: line from {p} changed before it was read")
                        consumed[(r, par, p)] = e
                live["done"] += 1

            live["procs"] = [block()]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make(r)))
    sim.run()
    return errors


# ---------------------------------------------------------------------------
# MoE dispatch (count exchange -> push -> receive) followed by combine
# ---------------------------------------------------------------------------
def run_moe(n, calls, seed):
    sim = Sim(seed)
    rows = {}                       # (at rank, parity, src) -> epoch of the count row
    disp_done = defaultdict(int)    # (at rank, from src)
    comb_done = defaultdict(int)
    rx = {}                         # (receiver, src) -> dispatch epoch of the pushed rows
    comb = {}                       # (source, expert rank) -> combine epoch of the returned rows
    errors = []

    def make(r):
        def mk(k):
            e = k + 1
            live = {"done": 0, "count": 1}

            def call():
                par = e & 1
                # 1. count rows to every rank, then wait for every row
                for p in range(n):
                    rows[(p, par, r)] = e
                yield lambda: all(rows.get((r, par, s), 0) >= e for s in range(n))
                # 2. push rows into every receiver's region
                for q in range(n):
                    prev = rx.get((q, r))
                    if prev is not None and prev != e - 1:
                        errors.append(f"rank {r} dispatch {e} overwrote rows of dispatch {prev} at {q}")
                    rx[(q, r)] = e
                    disp_done[(q, r)] += 1
                # 3. receive
                yield lambda: all(disp_done[(r, s)] >= e for s in range(n))
                yield lambda: True
                for s in range(n):
                    if rx.get((r, s)) != e:
                        errors.append(f"rank {r} dispatch {e} read rows of {rx.get((r, s))} from {s}")
                # combine: push back to every source, then wait and reduce
                for s in range(n):
                    comb[(s, r)] = e
                    comb_done[(s, r)] += 1
                yield lambda: all(comb_done[(r, q)] >= e for q in range(n))
                yield lambda: True
                for q in range(n):
                    if comb.get((r, q)) != e:
                        errors.append(f"rank {r} combine {e} read rows of {comb.get((r, q))} from {q}")
                live["done"] += 1

            live["procs"] = [call()]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make(r)))
    sim.run()
    return errors


@pytest.mark.parametrize("n,ctas", [(2, 2), (3, 2), (4, 3)])
def test_ag_gemm_protocol(n, ctas):
    for seed in range(150):
        assert run_ag_gemm(n, ctas, calls=4, seed=seed) == []


@pytest.mark.parametrize("n,ctas,blocks", [(2, 2, 2), (3, 3, 2), (4, 2, 3)])
def test_gemm_rs_protocol(n, ctas, blocks):
    for seed in range(150):
        assert run_gemm_rs(n, ctas, blocks, calls=4, seed=seed) == []


@pytest.mark.parametrize("n,ctas", [(2, 2), (3, 2), (4, 3), (8, 4)])
def test_gemm_rs_pair_protocol(n, ctas):
    for seed in range(120):
        assert run_gemm_rs_pair(n, ctas, calls=5, seed=seed) == []


# ---------------------------------------------------------------------------
# GEMM + RS with the two forms alternating on one communicator (the launcher
# picks the form per call from the shape, alike on every rank)
# ---------------------------------------------------------------------------
def run_gemm_rs_mixed(n, ctas, blocks, forms, seed, pair_counts_done=True):
    """forms[k] is "pair" (one kernel) or "two" (push kernel + sum kernel) for call k.  Shared
    counters as in csrc/fused/gemm_rs.cu: free[(source, owner)] (one bump per call, either form),
    the per-CTA GEMM call count (both forms), localDone (both forms add one per CTA, so the
    two-kernel form's "last CTA" test (k + 1) x ctas holds), done[(owner, source)] and the sum
    kernel's call count (two-kernel form only), per-half arrivals and consumed counts (one-kernel
    form only).  pair_counts_done=False drops the one-kernel form's localDone increment (negative
    control)."""
    sim = Sim(seed)
    rng = random.Random(seed * 11 + 3)
    halves = [rng.choice([1, 2, 3]) for _ in forms]
    free = defaultdict(int)
    done = defaultdict(int)
    local_done = defaultdict(int)
    local_free = defaultdict(int)
    reduce_calls = defaultdict(int)
    pair_free = defaultdict(int)
    arrive = defaultdict(int)
    consumed = defaultdict(int)
    slot = {}              # (owner, source, part) -> call
    unread = defaultdict(set)  # (owner, source) -> {(call, part)} pushed and not yet read
    errors = []

    def push(owner, src, part, k):
        stale = [c for c, _ in unread[(owner, src)] if c < k]
        if stale:
            errors.append(f"source {src} call {k} overwrote owner {owner}'s unread data of call {min(stale)}")
        slot[(owner, src, part)] = k
        unread[(owner, src)].add((k, part))

    def read(owner, src, part, k):
        if slot.get((owner, src, part)) != k:
            errors.append(f"owner {owner} call {k} read {part} of {src} holding call {slot.get((owner, src, part))}")
        unread[(owner, src)].discard((k, part))

    def make_call(r):
        def mk(k):
            live = {"done": 0, "count": 1}

            def two_kernel():
                kr = reduce_calls[r]  # the sum kernel's per-block call count
                g = {"done": 0}

                def cta(j):
                    yield lambda: all(free[(r, q)] >= k for q in range(n))
                    for q in range(n):
                        push(q, r, "all", k)
                    yield lambda: True
                    local_done[r] += 1
                    if local_done[r] == (k + 1) * ctas:
                        for q in range(n):
                            done[(q, r)] += 1
                    g["done"] += 1

                for j in range(ctas):
                    sim.spawn(cta(j))
                yield lambda: g["done"] == ctas
                b = {"done": 0}

                def blk(i):
                    yield lambda: all(done[(r, p)] >= kr + 1 for p in range(n))
                    if i == 0:
                        for p in range(n):
                            read(r, p, "all", k)
                    local_free[r] += 1
                    if local_free[r] == (kr + 1) * blocks:
                        for q in range(n):
                            free[(q, r)] += 1
                    b["done"] += 1

                for i in range(blocks):
                    sim.spawn(blk(i))
                yield lambda: b["done"] == blocks
                reduce_calls[r] += 1

            def one_kernel():
                H = halves[k]
                tiles = [((r + 1 + i) % n, h) for i in range(n) for h in range(H)]
                g = {"done": 0}

                def cta(j):
                    yield lambda: all(free[(r, q)] >= k for q in range(n))
                    for q, h in tiles[j::ctas]:
                        if q != r:
                            push(q, r, h, k)
                            yield lambda: True
                            arrive[(q, h)] += 1
                        else:
                            target = consumed[(r, h)] + (n - 1)
                            yield lambda t=target, hh=h: arrive[(r, hh)] >= t
                            for p in range(n):
                                if p != r:
                                    read(r, p, h, k)
                            consumed[(r, h)] = target
                    if pair_counts_done:
                        local_done[r] += 1
                    pair_free[r] += 1
                    if pair_free[r] == ctas:
                        pair_free[r] = 0
                        for q in range(n):
                            free[(q, r)] += 1
                    g["done"] += 1

                for j in range(ctas):
                    sim.spawn(cta(j))
                yield lambda: g["done"] == ctas

            def seq():
                yield from (one_kernel() if forms[k] == "pair" else two_kernel())
                live["done"] += 1

            live["procs"] = [seq()]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, len(forms), make_call(r)))
    sim.run()
    return errors


@pytest.mark.parametrize("n,ctas,blocks", [(2, 2, 2), (3, 2, 2), (4, 3, 2), (8, 2, 2)])
def test_gemm_rs_forms_alternate(n, ctas, blocks):
    """The one-kernel and two-kernel forms interleaved on one communicator (as shapes change from
    call to call): no deadlock, no overwritten or stale reads."""
    for seed in range(80):
        rng = random.Random(seed)
        forms = [rng.choice(["pair", "two"]) for _ in range(6)]
        assert run_gemm_rs_mixed(n, ctas, blocks, forms, seed) == [], forms


def test_model_detects_forms_without_shared_cta_count():
    """Negative control: if the one-kernel form did not add to localDone, a later two-kernel call's
    "last CTA" test would never fire and its sum kernel would wait forever."""
    failed = 0
    for seed in range(20):
        try:
            failed += bool(run_gemm_rs_mixed(3, 2, 2, ["pair", "two", "pair"], seed, pair_counts_done=False))
        except Deadlock:
            failed += 1
    assert failed > 0


# ---------------------------------------------------------------------------
# One-kernel GEMM + RS: the real tile walk, checked for cyclic waits
# ---------------------------------------------------------------------------
def pair_tile_from(tiles_m, tiles_n, t, group_rows, start_tm, cta):
    """csrc/kernels/gemm_sm100_pair.cuh pairTileFrom (no split-K): (row0, tn)."""
    t %= tiles_m * tiles_n
    group_tiles = group_rows * tiles_n
    g = t // group_tiles
    rows_here = min(group_rows, tiles_m - g * group_rows)
    local = t - g * group_tiles
    tn = local // rows_here
    tm = (g * group_rows + local % rows_here + start_tm) % tiles_m
    return tm * 256 + 128 * cta, tn


def rs_pair_walk(r, n, m, tiles_n, pairs):
    """Per pair of rank r, its pair tiles in order (pair p takes t = p, p + pairs, ...), each as the
    two CTAs' (owner, half tile) or None past M; start and groups as vcclGemmReduceScatter sets them."""
    rpr = m // n
    tiles_m = (m + 255) // 256
    start = (((r + 1) % n) * rpr // 256) % tiles_m
    shard_tiles = rpr // 256 if rpr % 256 == 0 else 0
    group = next((g for g in (16, 8, 4, 2, 1) if shard_tiles > 0 and shard_tiles % g == 0), 1)
    out = []
    for p in range(pairs):
        seq = []
        for t in range(p, tiles_m * tiles_n, pairs):
            halves = []
            for cta in (0, 1):
                row0, tn = pair_tile_from(tiles_m, tiles_n, t, group, start, cta)
                if row0 >= m:
                    halves.append(None)
                else:
                    owner = row0 // rpr
                    halves.append((owner, ((row0 - owner * rpr) // 128) * tiles_n + tn))
            seq.append(halves)
        out.append(seq)
    return out


def rs_pair_stuck(n, m, tiles_n, pairs):
    """One call of the one-kernel GEMM + RS on every rank, run to a fixed point.  A CTA's epilogue
    takes its half tiles in order; a push lands at once, an own half waits for the n - 1 arrivals;
    the pair's MMA for tile i reuses accumulator stage i % 2, so either CTA starts tile i only
    after both finished tile i - 2.  Returns the CTAs left waiting (a cycle of waits)."""
    walks = [rs_pair_walk(r, n, m, tiles_n, pairs) for r in range(n)]
    arrive = defaultdict(int)
    pos = {(r, p, c): 0 for r in range(n) for p in range(pairs) for c in (0, 1)}
    moved = True
    while moved:
        moved = False
        for (r, p, c) in pos:
            seq = walks[r][p]
            while pos[(r, p, c)] < len(seq):
                i = pos[(r, p, c)]
                if min(pos[(r, p, 0)], pos[(r, p, 1)]) < i - 1:
                    break
                h = seq[i][c]
                if h is not None:
                    owner, half = h
                    if owner != r:
                        arrive[(owner, half)] += 1
                    elif arrive[(r, half)] < n - 1:
                        break
                pos[(r, p, c)] = i + 1
                moved = True
    return [k for k, v in pos.items() if v < len(walks[k[0]][k[1]])]


@pytest.mark.parametrize("n", [2, 3, 4, 8])
def test_gemm_rs_pair_tile_walk(n):
    """Shapes the one-kernel path takes (M / n a multiple of 256): no cycle of waits for any
    column-tile count or pair-grid size (own rows end every pair's sequence)."""
    for rpr in range(256, 2049, 256):
        for tiles_n in (1, 3, 16, 29, 56):
            for pairs in (74, 37, 5, 1):
                assert rs_pair_stuck(n, rpr * n, tiles_n, pairs) == [], (rpr, tiles_n, pairs)


def test_model_detects_rs_pair_walk_with_half_pair_tiles():
    """Negative control: with 128-row shards (half pair tiles) own rows come mid-sequence, and at
    8 ranks with 56 column tiles (N = 14336) the waits close a cycle; the launcher sends those
    shapes to the two-kernel path."""
    assert rs_pair_stuck(8, 128 * 8, 56, 74)


def test_model_detects_absolute_arrival_targets():
    """Targets counted in calls instead of relative to the consumed count
    hang (or misread) as soon as consecutive calls have different shapes."""
    failed = 0
    for seed in range(60):
        try:
            failed += bool(run_gemm_rs_pair(3, 2, calls=5, seed=seed, relative=False))
        except Deadlock:
            failed += 1
    assert failed > 0


def test_model_detects_pair_rs_without_free_wait():
    """Without waiting for free[q], a fast sender overwrites a slot its owner has not read."""
    failed = 0
    for seed in range(200):
        try:
            failed += bool(run_gemm_rs_pair(3, 2, calls=4, seed=seed, free_wait=False))
        except Deadlock:
            failed += 1
    assert failed > 0


@pytest.mark.parametrize("n", [2, 3, 5, 8])
def test_ll_parity_protocol(n):
    for seed in range(200):
        assert run_ll(n, calls=6, seed=seed) == []


@pytest.mark.parametrize("n", [2, 3, 4])
def test_moe_protocol(n):
    for seed in range(200):
        assert run_moe(n, calls=4, seed=seed) == []


def test_model_detects_a_broken_protocol():
    """Sanity check of the checker: without the 'taken' wait the all-gather
    + GEMM protocol lets a rank restage its shard while a peer still pulls it."""
    def broken(n, ctas, calls, seed):
        sim = Sim(seed)
        xfull, ready, local_ready, staged = {}, defaultdict(int), defaultdict(int), defaultdict(int)
        errors = []

        def make_kernel(r):
            def mk(k):
                live = {"done": 0, "count": ctas}

                def copy_warps(j):
                    xfull[(r, r, j)] = k  # no wait for 'taken'
                    staged[r] += 1
                    if staged[r] == (k + 1) * ctas:
                        for p in range(n):
                            ready[(p, r)] += 1
                    for s in range(1, n):
                        q = (r + s) % n
                        yield lambda q=q: ready[(r, q)] >= k + 1
                        yield lambda: True
                        if xfull.get((q, q, j)) != k:
                            errors.append("stale")
                        local_ready[(r, q)] += 1
                    live["done"] += 1

                live["procs"] = [copy_warps(j) for j in range(ctas)]
                return live
            return mk

        for r in range(n):
            sim.spawn(kernel_chain(sim, calls, make_kernel(r)))
        sim.run()
        return errors

    assert any(broken(3, 2, 4, seed) for seed in range(200))


@pytest.mark.parametrize("n", [2, 3])
def test_ll_protocol_across_epoch_wrap(n):
    """Launches crossing the 32-bit epoch wrap (2^32-1 -> 2) keep the parity
    alternation and never see a line of an older launch as current."""
    for seed in range(150):
        assert run_ll(n, calls=6, seed=seed, start=0xFFFFFFFF - 3) == []


def test_model_detects_parity_break_at_wrap():
    """Wrapping to 1 instead of 2 would give two consecutive launches the same
    parity; the checker must see the overwrite."""
    def broken(seed):
        try:
            return bool(run_ll(3, calls=6, seed=seed, start=0xFFFFFFFF - 3, wrap_to=1))
        except Deadlock:
            return True

    assert any(broken(seed) for seed in range(200))


def test_model_detects_single_buffered_ll():
    """With one LL slot instead of two per source, a fast rank overwrites
    lines its peer has not read yet; the checker must see it."""
    def broken(seed):
        try:
            return bool(run_ll(3, calls=6, seed=seed, parities=1))
        except Deadlock:  # the overwritten line never shows the epoch its reader waits for
            return True

    assert any(broken(seed) for seed in range(200))


# ---------------------------------------------------------------------------
# LL broadcast: data flows only from the root, so every rank also exchanges a
# one-line token with every peer (csrc/kernels/movement.cuh, broadcastLL)
# ---------------------------------------------------------------------------
def run_ll_bcast(n, calls, seed, tokens=True):
    sim = Sim(seed)
    epoch = defaultdict(int)
    data, data_read = {}, {}   # (dst, parity) -> epoch of the root's lines / epoch the reader took
    tok = {}                   # (dst, parity, src) -> epoch
    errors = []
    root = 0

    def make(r):
        def mk(k):
            live = {"done": 0, "count": 1}

            def block():
                epoch[r] += 1
                e = epoch[r]
                par = e & 1
                if tokens:
                    for p in range(n):
                        if p != r:
                            tok[(p, par, r)] = e
                if r == root:
                    for p in range(n):
                        if p != r:
                            prev = data.get((p, par))
                            if prev is not None and data_read.get((p, par)) != prev:
                                errors.append(f"root epoch {e} overwrote unread epoch {prev} at rank {p}")
                            data[(p, par)] = e
                            yield lambda: True
                else:
                    yield lambda: data.get((r, par)) == e
                    yield lambda: True
                    if data.get((r, par)) != e:
                        errors.append(f"rank {r} epoch {e}: lines changed before they were read")
                    data_read[(r, par)] = e
                if tokens:
                    for p in range(n):
                        if p != r:
                            yield lambda p=p: tok.get((r, par, p)) == e
                live["done"] += 1

            live["procs"] = [block()]
            return live
        return mk

    for r in range(n):
        sim.spawn(kernel_chain(sim, calls, make(r)))
    sim.run()
    return errors


@pytest.mark.parametrize("n", [2, 3, 8])
def test_ll_broadcast_token_protocol(n):
    for seed in range(200):
        assert run_ll_bcast(n, calls=6, seed=seed) == []


def test_model_detects_broadcast_without_tokens():
    """Without the token exchange the root can run two calls ahead and
    overwrite lines a slow rank has not read (the bug the tokens fixed)."""
    def broken(seed):
        try:
            return bool(run_ll_bcast(3, calls=6, seed=seed, tokens=False))
        except Deadlock:
            return True

    assert any(broken(seed) for seed in range(300))


# ---------------------------------------------------------------------------
# point-to-point slot ring (csrc/kernels/movement.cuh, p2pKernel): per (peer,
# channel) a sender and a receiver walk one sequence of chunks; the sender
# waits until the receiver freed the slot it is about to reuse.
# ---------------------------------------------------------------------------
def run_p2p_ring(msgs, slots, seed):
    """msgs: chunk counts of consecutive messages on one (sender, receiver, channel)."""
    sim = Sim(seed)
    head = [0]   # written by the sender: chunks published
    tail = [0]   # written by the receiver: chunks consumed
    ring = {}    # slot -> sequence number it holds
    errors = []
    state = {"sent": 0, "recvd": 0}

    def sender():
        for m in msgs:
            base = state["sent"]
            for q in range(m):
                seq = base + q
                if seq >= slots:
                    yield lambda seq=seq: tail[0] >= seq - slots + 1
                held = ring.get(seq % slots)
                if held is not None and held >= tail[0]:
                    errors.append(f"chunk {seq} overwrote unread chunk {held}")
                ring[seq % slots] = seq
                yield lambda: True
                head[0] = seq + 1
            state["sent"] = base + m

    def receiver():
        for m in msgs:
            base = state["recvd"]
            for q in range(m):
                seq = base + q
                yield lambda seq=seq: head[0] >= seq + 1
                yield lambda: True
                if ring.get(seq % slots) != seq:
                    errors.append(f"read chunk {ring.get(seq % slots)} for {seq}")
                tail[0] = seq + 1
            state["recvd"] = base + m

    sim.spawn(sender())
    sim.spawn(receiver())
    sim.run()
    return errors


@pytest.mark.parametrize("slots", [1, 2, 4])
def test_p2p_ring_protocol(slots):
    rng = random.Random(slots)
    for seed in range(200):
        msgs = [rng.randint(1, 9) for _ in range(rng.randint(1, 5))]
        assert run_p2p_ring(msgs, slots, seed) == []


# ---------------------------------------------------------------------------
# NVLS all-reduce staging (csrc/kernels/collectives.cuh, allReduceNvls and
# allReduceNvlsPipe).  Sizes are in 16-byte units.  Each staging unit of each
# rank holds (call, piece, phase): 'in' after the copy-in, 'red' after the
# owner's multimem store, 'out' once the copy-out has read it.  Block b of
# every rank meets only block b of the others (blockBarrier).
# ---------------------------------------------------------------------------
def block_range(total, parts, idx):
    per = -(-total // parts)
    lo = min(per * idx, total)
    return lo, min(lo + per, total)


class StagingModel:
    def __init__(self, n, blocks, seed):
        self.sim = Sim(seed)
        self.n, self.blocks = n, blocks
        self.cell = {}                 # (rank, unit) -> (call, piece, phase)
        self.bar = defaultdict(int)    # (rank, block) -> barriers passed
        self.errors = []

    def barrier(self, r, b):
        self.bar[(r, b)] += 1
        t = self.bar[(r, b)]
        yield lambda: all(self.bar[(q, b)] >= t for q in range(self.n))

    def copy_in(self, r, unit, k, p):
        old = self.cell.get((r, unit))
        if old is not None and old[2] != "out":
            self.errors.append(f"rank {r} call {k} piece {p} overwrote unit {unit} holding {old}")
        self.cell[(r, unit)] = (k, p, "in")

    def reduce(self, unit, k, p):
        """multimem.ld_reduce of one unit, then (later) the multimem store."""
        for q in range(self.n):
            if self.cell.get((q, unit)) != (k, p, "in"):
                self.errors.append(f"call {k} piece {p} reduced unit {unit} of rank {q}: {self.cell.get((q, unit))}")
        yield lambda: True
        for q in range(self.n):
            self.cell[(q, unit)] = (k, p, "red")

    def copy_out(self, r, unit, k, p):
        if self.cell.get((r, unit)) != (k, p, "red"):
            self.errors.append(f"rank {r} call {k} piece {p} copied out unit {unit}: {self.cell.get((r, unit))}")
        self.cell[(r, unit)] = (k, p, "out")

    def run(self, calls, block_fn):
        def make(r):
            def mk(k):
                live = {"done": 0, "count": self.blocks}

                def blk(b):
                    yield from block_fn(r, b, k)
                    live["done"] += 1

                live["procs"] = [blk(b) for b in range(self.blocks)]
                return live
            return mk

        for r in range(self.n):
            self.sim.spawn(kernel_chain(self.sim, calls, make(r)))
        self.sim.run()
        return self.errors


def run_nvls_rounds(n, blocks, total, round_units, calls, seed, fixed_split=True):
    """allReduceNvls: copy in, barrier, reduce own chunk, barrier, copy out,
    round after round through one staging region."""
    M = StagingModel(n, blocks, seed)
    rng = M.sim.rng
    if fixed_split:
        cb = -(-total // n) if total <= round_units else round_units // n
    step = None

    def block_fn(r, b, k):
        yield from M.barrier(r, b)
        off, p = 0, 0
        while off < total:
            if fixed_split:
                cbr = cb
                m = min(total - off, cb * n)
            else:  # split every round afresh (the short last round re-splits)
                m = min(total - off, round_units)
                cbr = -(-m // n)
            s0, s1 = block_range(cbr, blocks, b)
            ins = [q * cbr + u for q in range(n) for u in range(s0, s1) if q * cbr + u < m]
            rng.shuffle(ins)
            for unit in ins:
                yield lambda: True
                M.copy_in(r, unit, k, p)
            yield from M.barrier(r, b)
            for unit in range(r * cbr + s0, min(r * cbr + s1, m)):
                yield lambda: True
                yield from M.reduce(unit, k, p)
            yield from M.barrier(r, b)
            for unit in ins:
                yield lambda: True
                M.copy_out(r, unit, k, p)
            off += m
            p += 1

    return M.run(calls, block_fn)


def run_nvls_pipe(n, blocks, total, slot_units, pieces, calls, seed):
    """allReduceNvlsPipe: three slots; step s copies piece s in, reduces piece
    s-1 and copies piece s-2 out (three warp roles, interleaved at random),
    then one barrier."""
    M = StagingModel(n, blocks, seed)
    rng = M.sim.rng
    cb = min(-(-(-(-total // pieces)) // n), slot_units // n)
    cb = max(cb, 1)
    piece = cb * n
    P = -(-total // piece)

    def m_of(p):
        return min(piece, total - p * piece)

    def block_fn(r, b, k):
        s0, s1 = block_range(cb, blocks, b)
        yield from M.barrier(r, b)
        for st in range(P + 2):
            ops = []
            if st < P:
                ops += [("in", st, (st % 3) * slot_units + q * cb + u)
                        for q in range(n) for u in range(s0, s1) if q * cb + u < m_of(st)]
            if 1 <= st <= P:
                p = st - 1
                ops += [("red", p, (p % 3) * slot_units + r * cb + u)
                        for u in range(s0, s1) if r * cb + u < m_of(p)]
            if st >= 2:
                p = st - 2
                ops += [("out", p, (p % 3) * slot_units + q * cb + u)
                        for q in range(n) for u in range(s0, s1) if q * cb + u < m_of(p)]
            rng.shuffle(ops)
            for kind, p, unit in ops:
                yield lambda: True
                if kind == "in":
                    M.copy_in(r, unit, k, p)
                elif kind == "red":
                    yield from M.reduce(unit, k, p)
                else:
                    M.copy_out(r, unit, k, p)
            if st == P + 1:
                break
            yield from M.barrier(r, b)

    return M.run(calls, block_fn)


@pytest.mark.parametrize("n,blocks,total", [(2, 2, 37), (3, 3, 50), (4, 2, 29)])
def test_nvls_round_protocol(n, blocks, total):
    for seed in range(60):
        assert run_nvls_rounds(n, blocks, total, round_units=16, calls=3, seed=seed) == []


def test_model_detects_resplit_last_round():
    """Splitting the short last round afresh hands a block units that a slower
    block still reads; the checker must see it (the kernels keep the split)."""
    assert any(run_nvls_rounds(2, 3, 37, round_units=16, calls=2, seed=s, fixed_split=False) for s in range(300))


@pytest.mark.parametrize("n,blocks,total,pieces", [(2, 2, 37, 4), (3, 2, 50, 3), (4, 3, 64, 4), (2, 3, 9, 4),
                                                   (3, 1, 200, 2)])
def test_nvls_pipe_protocol(n, blocks, total, pieces):
    for seed in range(60):
        assert run_nvls_pipe(n, blocks, total, slot_units=24, pieces=pieces, calls=3, seed=seed) == []


def test_model_detects_two_slot_pipe():
    """With two slots, copy-in of piece s lands in the slot whose piece s-2 is
    still being copied out in the same step."""
    def two_slots(seed):
        M = StagingModel(2, 1, seed)
        rng = M.sim.rng
        n, cb, P = 2, 2, 4

        def block_fn(r, b, k):
            yield from M.barrier(r, b)
            for st in range(P + 2):
                ops = []
                if st < P:
                    ops += [("in", st, (st % 2) * 8 + u) for u in range(n * cb)]
                if 1 <= st <= P:
                    ops += [("red", st - 1, ((st - 1) % 2) * 8 + r * cb + u) for u in range(cb)]
                if st >= 2:
                    ops += [("out", st - 2, ((st - 2) % 2) * 8 + u) for u in range(n * cb)]
                rng.shuffle(ops)
                for kind, p, unit in ops:
                    yield lambda: True
                    if kind == "in":
                        M.copy_in(r, unit, k, p)
                    elif kind == "red":
                        yield from M.reduce(unit, k, p)
                    else:
                        M.copy_out(r, unit, k, p)
                if st < P + 1:
                    yield from M.barrier(r, b)

        return M.run(2, block_fn)

    assert any(two_slots(s) for s in range(100))


# ---------------------------------------------------------------------------
# Window collectives (csrc/kernels/window.cuh): each block publishes its
# call's descriptor in its own ctrl slot, meets the peers (start barrier),
# reads every peer's descriptor, moves data in place on the peers' buffers,
# and meets them again (end barrier) before the kernel may end.
# ---------------------------------------------------------------------------
def run_window(n, blocks, calls, seed, end_barrier=True):
    M = StagingModel(n, blocks, seed)
    desc = {}                 # (rank, block) -> call number published
    data = {}                 # (rank, block) -> call whose data the buffer holds / "reading"
    errors = M.errors

    def block_fn(r, b, k):
        desc[(r, b)] = k
        yield from M.barrier(r, b)
        for q in range(n):
            yield lambda: True
            if desc.get((q, b)) != k:
                errors.append(f"rank {r} block {b} call {k} read rank {q}'s descriptor of call {desc.get((q, b))}")
        # write my piece of every rank's receive buffer, read every send buffer
        for q in range(n):
            yield lambda: True
            if data.get(("send", q, b), k) not in (k,):
                errors.append(f"rank {r} call {k} read rank {q}'s send buffer holding call {data.get(('send', q, b))}")
        if end_barrier:
            yield from M.barrier(r, b)
        # after the kernel the rank's next call refills its send buffer
        data[("send", r, b)] = k + 1

    for r in range(n):
        for b in range(blocks):
            data[("send", r, b)] = 0
    return M.run(calls, block_fn)


@pytest.mark.parametrize("n,blocks", [(2, 1), (3, 2), (4, 3)])
def test_window_protocol(n, blocks):
    for seed in range(100):
        assert run_window(n, blocks, calls=4, seed=seed) == []


def test_model_detects_window_without_end_barrier():
    """Without the end barrier a rank refills its send buffer for the next
    call while a peer still reads it."""
    assert any(run_window(3, 1, 4, seed=s, end_barrier=False) for s in range(200))

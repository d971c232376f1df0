"""Model check of the fused-layer kernel's synchronisation (CPU).

The per-CTA roles of fused_layer.cu - TMA producer, MMA issuer, epilogue
warps - are restated as generators that yield the condition they wait on,
in the kernel's order: the ring of `stages` slots (full / empty barriers),
the two TMEM accumulators (tfull / tempty), the stream-K split of each GEMM
phase with its split-tile counters (arrive without waiting, reduce after
all own arrivals; last arriver for whole-tile epilogues), the grid barrier
between phases, and the per-CTA-index meetings of the peer all-reduce
phase across ranks.  Random schedulers interleave every CTA of every rank;
each run must finish (no deadlock) and respect the data dependencies:

* a phase's activation tiles are loaded only after every CTA of the rank
  has finished the previous phase;
* a split tile is reduced only after all its contributors stored partials;
* a rank's peer phase reads the other ranks' partials only after all of
  their CTAs finished the GEMM phase that wrote them.
"""
import random

import pytest


def it_begin(p, P, W):
    return p * W // P


def phase_ctas(W, P):
    """fused_layer.cu phase_range(): CTAs 0..Pf-1 split a phase's W, Pf = min(W, P)."""
    return min(W, P)


def phase_range(pc, Pf, W):
    return (it_begin(pc, Pf, W), it_begin(pc + 1, Pf, W)) if pc < Pf else (0, 0)


def owner_of(x, P, W):
    q = min(x * P // W, P - 1)
    while q + 1 < P and it_begin(q + 1, P, W) <= x:
        q += 1
    while q > 0 and it_begin(q, P, W) > x:
        q -= 1
    return q


def unit_range(ph, unit, units, split):
    """(b, e), Pf of a unit in a GEMM phase ("gemm", W, KT, dist[, dp]):
    stream-K over Pf = split(W, units) units, or - data-parallel phases
    (fused_layer.cu phase_range() with ph.dp) - whole tiles over
    Pf = min(tiles, units) units."""
    W, KT = ph[1], ph[2]
    if len(ph) > 4 and ph[4]:
        tiles = W // KT
        pf = min(tiles, units)
        if unit >= pf:
            return (0, 0), pf
        return ((unit * tiles // pf) * KT, ((unit + 1) * tiles // pf) * KT), pf
    pf = split(W, units)
    return phase_range(unit, pf, W), pf


class Rank:
    def __init__(self, P):
        self.gbar = 0
        self.counters = {}           # (phase, tile) -> arrivals
        self.departed = {}
        self.phase_done = [set() for _ in range(16)]   # CTAs finished with phase f
        self.peer_ctr = [0] * P
        self.flags = {}              # (cta, from_rank) -> epoch


class CTA:
    def __init__(self, rank, pc, stages):
        self.rank, self.pc = rank, pc
        self.full = [0] * stages     # completed phases of each full barrier
        self.empty = [0] * stages
        self.tfull = [0, 0]
        self.tempty = [0, 0]         # arrivals / 4 warps -> completed phases


def run(phases, P, stages, R, seed, split=phase_ctas, CG=1):
    """phases: list of ("gemm", W, KT, dist) | ("norm",) | ("peer",);
    split(W, units): the number of units sharing a GEMM phase's iterations;
    CG = 2: CTA pairs (cta_group::2) - both CTAs' loads complete on the
    leader's full barrier, the leader alone issues MMAs and commits to both
    CTAs, both epilogues arrive on the leader's accumulator-empty barrier."""
    rnd = random.Random(seed)
    assert P % CG == 0
    units = P // CG
    per_round = 1 + 2 * CG           # leader's expect + A and B loads of every CTA of the unit
    ranks = [Rank(P) for _ in range(R)]
    ctas = [[CTA(r, pc, stages) for pc in range(P)] for r in range(R)]
    for r in range(R):
        for c in ctas[r]:
            c.full_count = [0] * stages

    def land(leader, s, rnd_):
        # a transfer of round rnd_ must not reach the barrier before round rnd_-1 completed
        assert leader.full_count[s] >= rnd_ * per_round, "a load reached the next round of a full barrier"
        leader.full_count[s] += 1

    def producer(r, pc):
        c = ctas[r][pc]
        unit, crank = pc // CG, pc % CG
        leader = ctas[r][unit * CG]
        i = 0
        for f, ph in enumerate(phases):
            if ph[0] != "gemm":
                continue
            W, KT = ph[1], ph[2]
            (b, e), _ = unit_range(ph, unit, units, split)
            if b >= e:
                continue
            npre = min(e - b, stages)
            for k in range(npre):          # weight tiles first
                s, rnd_ = (i + k) % stages, (i + k) // stages
                if rnd_ > 0:
                    yield lambda s=s, rnd_=rnd_: c.empty[s] >= rnd_
                if crank == 0:
                    land(leader, s, rnd_)  # expect
                land(leader, s, rnd_)      # A
            if f > 0:                      # activations after the grid barrier
                yield lambda f=f: ranks[r].gbar >= P * f
                assert len(ranks[r].phase_done[f - 1]) == P, "B tiles before the previous phase ended"
            for k in range(npre):
                s, rnd_ = (i + k) % stages, (i + k) // stages
                land(leader, s, rnd_)      # B
            for k in range(npre, e - b):
                s, rnd_ = (i + k) % stages, (i + k) // stages
                yield lambda s=s, rnd_=rnd_: c.empty[s] >= rnd_
                if crank == 0:
                    land(leader, s, rnd_)
                land(leader, s, rnd_)
                land(leader, s, rnd_)
            i += e - b

    def mma(r, pc):
        if pc % CG:
            return
        c = ctas[r][pc]
        pair = [ctas[r][pc + q] for q in range(CG)]
        unit = pc // CG
        i = seg = 0
        for f, ph in enumerate(phases):
            if ph[0] != "gemm":
                continue
            W, KT = ph[1], ph[2]
            (b, e), _ = unit_range(ph, unit, units, split)
            if b >= e:
                continue
            for t in range(b // KT, (e - 1) // KT + 1):
                tb = t * KT
                k0, k1 = max(b, tb) - tb, min(e, tb + KT) - tb
                buf, use = seg & 1, seg >> 1
                if use > 0:
                    yield lambda buf=buf, use=use: c.tempty[buf] >= use * CG
                for _ in range(k0, k1):
                    s, rnd_ = i % stages, i // stages
                    yield lambda s=s, rnd_=rnd_: c.full_count[s] >= (rnd_ + 1) * per_round
                    for q in pair:         # commit to every CTA of the unit
                        q.empty[s] += 1
                    i += 1
                for q in pair:
                    q.tfull[buf] += 1
                seg += 1

    def epilogue(r, pc):
        c = ctas[r][pc]
        rk = ranks[r]
        unit, crank = pc // CG, pc % CG
        leader = ctas[r][unit * CG]
        seg = 0
        for f, ph in enumerate(phases):
            if f > 0:
                yield lambda f=f: rk.gbar >= P * f
            if ph[0] in ("peer", "peer2"):    # one-shot: one meeting; two-shot: two
                for meeting in range(1 if ph[0] == "peer" else 2):
                    e = rk.peer_ctr[pc] = rk.peer_ctr[pc] + 1
                    for q in range(R):
                        ranks[q].flags[(pc, r)] = e
                    yield lambda e=e: all(rk.flags.get((pc, q), 0) >= e for q in range(R))
                    for q in range(R):   # the partials of every rank are complete
                        assert len(ranks[q].phase_done[f - 1]) == P, "peer read before a rank's partials"
            elif ph[0] == "gemm":
                W, KT, dist = ph[1], ph[2], ph[3]
                (b, e), Pf = unit_range(ph, unit, units, split)
                pend = []
                if b < e:
                    for t in range(b // KT, (e - 1) // KT + 1):
                        tb = t * KT
                        k0, k1 = max(b, tb) - tb, min(e, tb + KT) - tb
                        buf, use = seg & 1, seg >> 1
                        yield lambda buf=buf, use=use: c.tfull[buf] >= use + 1
                        leader.tempty[buf] += 1
                        seg += 1
                        if k0 == 0 and k1 == KT:
                            continue
                        key = (f, t * CG + crank)
                        q_lo, q_hi = owner_of(tb, Pf, W), owner_of(tb + KT - 1, Pf, W)
                        rk.counters[key] = rk.counters.get(key, 0) + 1
                        if dist:
                            pend.append((key, q_hi - q_lo + 1))
                        elif rk.counters[key] == q_hi - q_lo + 1:
                            rk.counters[key] = 0   # last arriver finishes the tile
                for key, nq in pend:
                    yield lambda key=key, nq=nq: rk.counters[key] >= nq
                    rk.departed[key] = rk.departed.get(key, 0) + 1
                    if rk.departed[key] == nq:
                        rk.counters[key] = rk.departed[key] = 0
            rk.phase_done[f].add(pc)
            rk.gbar += 1

    actors = []
    for r in range(R):
        for pc in range(P):
            for role in (producer, mma, epilogue):
                actors.append([role(r, pc), None, False])
    steps = 0
    while True:
        live = [a for a in actors if not a[2]]
        if not live:
            break
        ready = [a for a in live if a[1] is None or a[1]()]
        assert ready, "deadlock"
        a = rnd.choice(ready)
        try:
            a[1] = next(a[0])
        except StopIteration:
            a[2] = True
        steps += 1
        assert steps < 2_000_000
    for rk in ranks:
        assert rk.gbar == P * len(phases)
        assert all(v == 0 for v in rk.counters.values())


# a decoder layer's phases; (W, KT) chosen so tiles split across CTAs
LAYER = [("gemm", 5 * 4, 4, True), ("norm",), ("gemm", 9 * 4, 4, False), ("gemm", 5 * 6, 6, True), ("norm",),
         ("gemm", 6 * 4, 4, False)]
TP_LAYER = [("gemm", 5 * 4, 4, True), ("peer",), ("norm",), ("gemm", 9 * 4, 4, False), ("gemm", 5 * 6, 6, True),
            ("peer",), ("norm",), ("gemm", 6 * 4, 4, False)]


@pytest.mark.parametrize("P,stages", [(3, 2), (6, 3), (7, 5), (12, 2)])
@pytest.mark.parametrize("seed", range(4))
def test_single_rank_layer_never_deadlocks(P, stages, seed):
    run(LAYER, P, stages, R=1, seed=seed)


@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("seed", range(3))
def test_tensor_parallel_layer_never_deadlocks(R, seed):
    run(TP_LAYER, P=5, stages=3, R=R, seed=seed)


@pytest.mark.parametrize("R", [2, 4])
@pytest.mark.parametrize("seed", range(3))
def test_tensor_parallel_layer_two_shot_never_deadlocks(R, seed):
    layer = [("peer2",) if ph[0] == "peer" else ph for ph in TP_LAYER]
    run(layer, P=5, stages=3, R=R, seed=seed)


@pytest.mark.parametrize("P,stages", [(4, 2), (8, 3), (12, 5)])
@pytest.mark.parametrize("seed", range(4))
def test_cta_pairs_never_deadlock_or_mix_rounds(P, stages, seed):
    """CG = 2: both CTAs' loads complete on the leader's full barrier, yet a
    transfer of the next round never reaches it before the current round
    completed (each CTA waits for its own empty barrier, which the leader's
    commit releases only after consuming the round)."""
    run(LAYER, P, stages, R=1, seed=seed, CG=2)
    run(SMALL_PHASES, P, stages, R=1, seed=seed, CG=2)
    run(TP_LAYER, P, stages, R=2, seed=seed, CG=2)


@pytest.mark.parametrize("seed", range(4))
def test_fewer_iterations_than_ctas(seed):
    """Phases with fewer iterations than CTAs (the small shapes of the tests):
    the CTAs past Pf sit the phase out and every split tile's contributors
    are consecutive CTAs that each own an iteration.  (Splitting over all P
    CTAs instead counted CTAs with empty ranges as contributors, and their
    tiles were never complete.)"""
    run(SMALL_PHASES, P=8, stages=2, R=1, seed=seed)


SMALL_PHASES = [("gemm", 4, 2, True), ("norm",), ("gemm", 3, 3, False), ("gemm", 6, 2, True)]


# the layer with its GEMM phases data-parallel (whole tiles per unit; fewer
# tiles than units in some, so units sit phases out)
LAYER_DP = [("gemm", 5 * 4, 4, True, True), ("norm",), ("gemm", 9 * 4, 4, False, True),
            ("gemm", 5 * 6, 6, True, False), ("norm",), ("gemm", 6 * 4, 4, False, True)]


@pytest.mark.parametrize("P,stages", [(3, 2), (6, 3), (7, 5), (12, 2)])
@pytest.mark.parametrize("seed", range(3))
def test_data_parallel_phases_never_deadlock(P, stages, seed):
    """Data-parallel GEMM phases (no split tiles, no counters) mixed with
    stream-K ones, on single CTAs, CTA pairs and two ranks."""
    run(LAYER_DP, P, stages, R=1, seed=seed)
    if P % 2 == 0:
        run(LAYER_DP, P, stages, R=1, seed=seed, CG=2)
    tp = [ph for ph in LAYER_DP]
    tp.insert(1, ("peer",))
    run(tp, P, stages, R=2, seed=seed)


def test_splitting_over_every_cta_deadlocks_small_phases():
    """The check of the check: with all P CTAs sharing a phase of W < P
    iterations, a split tile counts CTAs that own nothing as contributors
    and its reduction waits for them forever."""
    with pytest.raises(AssertionError, match="deadlock"):
        run(SMALL_PHASES, P=8, stages=2, R=1, seed=0, split=lambda W, P: P)


def test_the_model_catches_a_missing_barrier():
    """Sanity check of the check: without the producer's barrier wait, some
    schedule loads a phase's activations too early."""
    import types
    src = run.__code__
    hit = False
    for seed in range(40):
        try:
            _run_without_barrier(LAYER, P=4, stages=2, seed=seed)
        except AssertionError as e:
            hit = hit or "before the previous phase ended" in str(e)
    assert hit and isinstance(src, types.CodeType)


def _run_without_barrier(phases, P, stages, seed):
    # the producer of run() with the grid-barrier wait removed
    rnd = random.Random(seed)
    rk = Rank(P)
    done = [set() for _ in phases]

    def producer(pc):
        for f, ph in enumerate(phases):
            if ph[0] != "gemm":
                continue
            yield lambda: True
            if f > 0:
                assert len(done[f - 1]) == P, "B tiles before the previous phase ended"

    def epilogue(pc):
        for f, ph in enumerate(phases):
            if f > 0:
                yield lambda f=f: rk.gbar >= P * f
            yield lambda: True
            done[f].add(pc)
            rk.gbar += 1

    actors = [[producer(pc), None, False] for pc in range(P)] + [[epilogue(pc), None, False] for pc in range(P)]
    while any(not a[2] for a in actors):
        ready = [a for a in actors if not a[2] and (a[1] is None or a[1]())]
        a = rnd.choice(ready)
        try:
            a[1] = next(a[0])
        except StopIteration:
            a[2] = True

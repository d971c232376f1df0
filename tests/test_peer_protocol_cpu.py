"""Model check of the peer all-reduce protocol (CPU).

tsds_peer_allreduce_residual (and the peer phase of the fused-layer kernel)
rely on two claims: every rank's partial is complete when a CTA passes its
meeting, and two alternating slots are enough - a rank writes slot s again
only two calls later, when no rank can still be reading it.  Here each rank
is a stream of kernels in order (the row-parallel GEMM writing slot i % 2 of
call i, then the all-reduce whose CTAs meet the same CTA index of every
rank through per-CTA call counters and flags, wait with `>=`, and read
every rank's slot).  Random schedulers interleave the ranks' streams and
the CTAs inside each all-reduce; every run must finish and:

* a CTA reads a rank's slot only after that rank's GEMM for the call wrote it;
* a rank's GEMM never overwrites a slot some rank is still to read.
"""
import random

import pytest


def run(R, G, calls, seed, grids=None, two_shot=False):
    """R ranks, all-reduce grids of G CTAs (grids[i] per call when given:
    every rank uses the same grid for a call), `calls` calls.  two_shot: each
    CTA reduces its share of its rank's chunk from every rank's slot,
    publishes it, meets again, then copies the other ranks' published
    chunks (the fused kernel's two-shot phase)."""
    rnd = random.Random(seed)
    written = {}                         # (rank, call) -> written
    readers_left = {}                    # (rank, slot) -> set of (reader rank, cta) still to read it
    published = {}                       # (rank, cta) -> call whose chunk share is published
    copiers_left = {}                    # (rank, cta) -> set of ranks still to copy that share
    counters = [[0] * 64 for _ in range(R)]
    flags = [[[0] * R for _ in range(64)] for _ in range(R)]   # flags[owner][cta][from]

    def stream(r):
        for i in range(calls):
            g = grids[i] if grids else G
            slot = i % 2
            # the GEMM of call i: every earlier kernel of this rank has finished
            assert not readers_left.get((r, slot)), f"rank {r} overwrites slot {slot} still being read (call {i})"
            written[(r, i)] = True
            readers_left[(r, slot)] = {(q, b) for q in range(R) for b in range(g)}
            yield None
            # the all-reduce of call i: G CTAs, concurrent
            ctas = [cta(r, b, i, slot) for b in range(g)]
            pending = [[c, None] for c in ctas]
            while pending:
                ready = [p for p in pending if p[1] is None or p[1]()]
                if not ready:
                    yield lambda pending=pending: any(p[1] is None or p[1]() for p in pending)
                    continue
                p = rnd.choice(ready)
                try:
                    p[1] = next(p[0])
                except StopIteration:
                    pending.remove(p)
                yield None

    def meet(r, b):
        e = counters[r][b] = counters[r][b] + 1
        for q in range(R):
            flags[q][b][r] = e
        yield lambda: all(flags[r][b][q] >= e for q in range(R))

    def cta(r, b, i, slot):
        yield from meet(r, b)
        for q in range(R):
            assert written.get((q, i)), f"rank {r} cta {b} read rank {q}'s slot before call {i} wrote it"
            readers_left[(q, slot)].discard((r, b))
            yield None
        if not two_shot:
            return
        # publish this CTA's share of the rank's chunk (the same share index
        # is what CTA b of every other rank copies)
        assert not copiers_left.get((r, b)), f"rank {r} cta {b} overwrites a published share still to be copied"
        published[(r, b)] = i
        copiers_left[(r, b)] = {q for q in range(R) if q != r}
        yield from meet(r, b)
        for q in range(R):
            if q == r:
                continue
            assert published.get((q, b)) == i, f"rank {r} cta {b} copied rank {q}'s share before call {i} published it"
            copiers_left[(q, b)].discard(r)
            yield None

    actors = [[stream(r), None, False] for r in range(R)]
    steps = 0
    while any(not a[2] for a in actors):
        ready = [a for a in actors if not a[2] and (a[1] is None or a[1]())]
        assert ready, "deadlock"
        a = rnd.choice(ready)
        try:
            a[1] = next(a[0])
        except StopIteration:
            a[2] = True
        steps += 1
        assert steps < 1_000_000


@pytest.mark.parametrize("R,G", [(2, 1), (2, 4), (4, 3), (8, 2)])
@pytest.mark.parametrize("seed", range(5))
def test_two_slots_and_per_cta_meetings(R, G, seed):
    run(R, G, calls=8, seed=seed)


@pytest.mark.parametrize("R,G", [(2, 2), (4, 3), (8, 2)])
@pytest.mark.parametrize("seed", range(5))
def test_two_shot_publish_and_copy(R, G, seed):
    """Two-shot: a share is copied only after this call published it, and
    published again only after every rank copied it."""
    run(R, G, calls=8, seed=seed, two_shot=True)


@pytest.mark.parametrize("seed", range(5))
def test_grids_that_change_between_calls(seed):
    """Calls of different sizes (different M) use different grids; a CTA
    index skipped by a small call keeps its counter behind on every rank
    alike, so the flags still agree."""
    run(R=3, G=None, calls=9, seed=seed, grids=[4, 1, 3, 4, 2, 4, 1, 1, 3])


def test_the_check_catches_a_single_slot():
    """The check of the check: with one slot a rank overwrites partials that
    a slower rank has not read yet."""
    hit = False
    for seed in range(30):
        try:
            _run_one_slot(R=3, G=2, calls=6, seed=seed)
        except AssertionError as e:
            hit = hit or "still being read" in str(e)
    assert hit


def _run_one_slot(R, G, calls, seed):
    rnd = random.Random(seed)
    readers_left = {}
    counters = [[0] * G for _ in range(R)]
    flags = [[[0] * R for _ in range(G)] for _ in range(R)]

    def stream(r):
        for i in range(calls):
            assert not readers_left.get(r), f"rank {r} overwrites slot 0 still being read (call {i})"
            readers_left[r] = {(q, b) for q in range(R) for b in range(G)}
            yield None
            for b in range(G):
                e = counters[r][b] = counters[r][b] + 1
                for q in range(R):
                    flags[q][b][r] = e
                yield lambda b=b, e=e: all(flags[r][b][q] >= e for q in range(R))
                for q in range(R):
                    readers_left[q].discard((r, b))
                    yield None

    actors = [[stream(r), None, False] for r in range(R)]
    while any(not a[2] for a in actors):
        ready = [a for a in actors if not a[2] and (a[1] is None or a[1]())]
        a = rnd.choice(ready)
        try:
            a[1] = next(a[0])
        except StopIteration:
            a[2] = True


def run_lm(R, G, calls, seed, exit_meeting=True):
    """tsds_peer_lm_gather: each call, a rank's LM head writes its one exchange
    region (stream order: after its previous gather kernel), then the gather
    kernel's CTAs meet, read every rank's region, and meet again."""
    rnd = random.Random(seed)
    counters = [[0] * G for _ in range(R)]
    flags = [[[0] * R for _ in range(G)] for _ in range(R)]
    readers_left = {r: set() for r in range(R)}
    version = {r: -1 for r in range(R)}

    def meet(r, b):
        e = counters[r][b] = counters[r][b] + 1
        for q in range(R):
            flags[q][b][r] = e
        yield lambda: all(flags[r][b][q] >= e for q in range(R))

    def cta(r, b, i):
        yield from meet(r, b)
        for q in range(R):
            assert version[q] == i, f"rank {r} read rank {q}'s region of another call"
            readers_left[q].discard((r, b))
            yield None
        if exit_meeting:
            yield from meet(r, b)

    def stream(r):
        for i in range(calls):
            assert not readers_left[r], f"rank {r} overwrote its exchange region still being read (call {i})"
            version[r] = i
            readers_left[r] = {(q, b) for q in range(R) for b in range(G)}
            yield None
            pending = [[cta(r, b, i), None] for b in range(G)]
            while pending:
                ready = [p for p in pending if p[1] is None or p[1]()]
                if not ready:
                    yield lambda pending=pending: any(p[1] is None or p[1]() for p in pending)
                    continue
                p = rnd.choice(ready)
                try:
                    p[1] = next(p[0])
                except StopIteration:
                    pending.remove(p)
                yield None

    actors = [[stream(r), None, False] for r in range(R)]
    while any(not a[2] for a in actors):
        ready = [a for a in actors if not a[2] and (a[1] is None or a[1]())]
        assert ready, "deadlock"
        a = rnd.choice(ready)
        try:
            a[1] = next(a[0])
        except StopIteration:
            a[2] = True


@pytest.mark.parametrize("R,G", [(2, 1), (4, 3), (8, 2)])
@pytest.mark.parametrize("seed", range(5))
def test_lm_gather_one_region_with_exit_meeting(R, G, seed):
    run_lm(R, G, calls=6, seed=seed)


def test_lm_gather_without_exit_meeting_overwrites():
    """The check of the check: without the second meeting a rank's next LM
    head can overwrite the region a slower rank is still reading."""
    hit = False
    for seed in range(40):
        try:
            run_lm(3, 2, calls=5, seed=seed, exit_meeting=False)
        except AssertionError as e:
            hit = hit or "still being read" in str(e) or "of another call" in str(e)
    assert hit

"""The default verify-attention kernel's K/V ring, modelled on the CPU.

One producer streams the tiles of a CTA's work items, in order, through a
ring of `stages` shared-memory stages (full / empty mbarriers); consumer
warp (rg, kg) takes tiles kg, kg + KG, ... of each item, waiting on the
stage's full barrier by phase parity, and releases the stage (empty barrier,
RG arrivals); all consumer warps meet at the item's merge barrier.  TMA
copies may land in any order.

A parity wait is exact only while the stage's previous use has landed; the
model checks, at every wait, that the tile `stages` before the awaited one
has landed (otherwise the wait could return on the old phase and read stale
data), and that the run finishes.  Parameters come from the library's own
launch plan (tsds_attention_plan) for the shapes the engines use, so the
model follows the kernel's choices; the last test shows the check catching a
ring depth that a key-group count does not divide.
"""
import ctypes
import random

import pytest


class _Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0   # phase = completed phases

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


def _run(items, RG, KG, stages, rnd):
    """Returns 'ok', 'stale' (a parity wait that could alias) or 'stuck'."""
    full = [_Bar(1) for _ in range(stages)]
    empty = [_Bar(RG) for _ in range(stages)]
    landed = set()
    prod = {"item": 0, "t": 0, "q": 0}
    NC = RG * KG
    cons = [{"item": 0, "tile": None, "q0": 0, "state": "start"} for _ in range(NC)]
    at_barrier = set()
    inflight = []
    for _ in range(100_000):
        acts = []
        if prod["item"] < len(items):
            nt = items[prod["item"]]
            if prod["t"] >= nt:
                acts.append("next")
            else:
                q = prod["q"]
                s = q % stages
                if q < stages or empty[s].phase > (q // stages) - 1:
                    acts.append("issue")
        if inflight:
            acts.append("land")
        for c in range(NC):
            st = cons[c]
            if st["state"] in ("done", "barrier"):
                continue
            if st["state"] == "tiles" and st["tile"] < items[st["item"]]:
                qs = st["q0"] + st["tile"]
                s = qs % stages
                # the parity wait returns once (phase & 1) != (qs // stages) & 1
                if (full[s].phase & 1) == ((qs // stages) & 1):
                    continue
                if qs >= stages and qs - stages not in landed:
                    return "stale"
            acts.append(c)
        if not acts:
            done = all(c["state"] == "done" for c in cons) and prod["item"] >= len(items) and not inflight
            return "ok" if done else "stuck"
        a = rnd.choice(acts)
        if a == "next":
            prod["item"] += 1
            prod["t"] = 0
        elif a == "issue":
            inflight.append(prod["q"])
            prod["q"] += 1
            prod["t"] += 1
        elif a == "land":
            q = inflight.pop(rnd.randrange(len(inflight)))
            landed.add(q)
            full[q % stages].arrive()
        else:
            st = cons[a]
            kg = a // RG
            if st["item"] >= len(items):
                st["state"] = "done"
                continue
            nt = items[st["item"]]
            if st["state"] == "start":
                if nt == 0:          # an empty item is skipped by every warp
                    st["item"] += 1
                    continue
                st["tile"], st["state"] = kg, "tiles"
                continue
            if st["tile"] >= nt:
                st["state"] = "barrier"
                at_barrier.add(a)
                if len(at_barrier) == NC:
                    for cc in cons:
                        cc["q0"] += nt
                        cc["item"] += 1
                        cc["state"] = "start"
                    at_barrier.clear()
                continue
            qs = st["q0"] + st["tile"]
            empty[qs % stages].arrive()
            st["tile"] += KG
    return "stuck"


def _plan(B, T, Hq, Hkv, max_kv, split, sms=148):
    from tri_sds_b200 import _lib
    out = (ctypes.c_int32 * 6)()
    assert _lib.load().tsds_attention_plan(B, T, Hq, Hkv, max_kv, split, sms, out) == 0
    return list(out)


# (B, T, Hq, Hkv, max_kv, split): tree verify B=1/8, chain verify, decode, config-2 attention, 4B draft
SHAPES = [(1, 26, 64, 8, 1024, 1024), (8, 26, 64, 8, 1024, 1024), (1, 5, 64, 8, 4096, 1024),
          (8, 5, 64, 8, 4096, 1024), (1, 1, 32, 8, 1024, 1024), (2, 26, 64, 8, 1024, 128),
          (4, 5, 32, 8, 4096, 256), (1, 26, 4, 2, 128, 64)]


@pytest.mark.parametrize("shape", SHAPES)
def test_ring_protocol_of_the_library_plan(shape):
    RG, KG, nrb, nsplit, stages, threads = _plan(*shape)
    assert stages % KG == 0 and RG * KG <= 8 and threads == 32 * (1 + RG * KG)
    split = shape[-1]
    per_split = split // 64
    rnd = random.Random(sum(shape))
    for trial in range(150):
        # a CTA's items: whole splits, partial last splits, empty splits past the sequence
        items = [rnd.choice([0, per_split, per_split, rnd.randint(1, per_split)]) for _ in range(rnd.randint(1, 4))]
        assert _run(items, RG, KG, stages, rnd) == "ok", (items, RG, KG, stages)


def test_model_flags_a_ring_the_key_groups_do_not_divide():
    rnd = random.Random(1)
    results = {_run([16, 16, 9], 1, 4, 5, rnd) for _ in range(200)}
    assert "stale" in results or "stuck" in results

"""Model check of the tcgen05 verify-attention kernel's synchronisation (CPU).

verify_attn_tc_kernel (tri_sds_b200/csrc/attention.cu) runs three roles per
CTA: the TMA producer (K and V tiles of 128 keys into a 2-deep ring), the MMA
issuer (S_i = Q K_i^T into one of two TMEM buffers, O_i = P_i V_i into one
of two) and four warps of query rows (softmax of S_i into one of two P
buffers in shared memory; O_{i-1} is folded into registers after the
softmax of tile i, so the P V product of one tile overlaps the softmax of
the next).  Every hand-off is an mbarrier waited on by phase
parity, as in the kernel: a wait for parity p returns once the barrier has
completed a phase of that parity, so a waiter two phases behind would block.
Each role is a generator yielding the condition it waits on; TMA loads
complete in any order, tensor-core operations in issue order, both at a
random later step, and their reads and writes are checked at issue and at
completion.  Every run must finish and respect:

* S_i reads Q (every warp's rows written) and K_i (loaded into its stage);
* S_i overwrites an S buffer only after every warp finished reading S_{i-2};
* the warps read S_i only after S_i completed;
* the warps write P_i only after O_{i-2} (the last reader of its buffer)
  completed;
* O_i reads P_i of all four warps and V_i, and overwrites its O buffer only
  after every warp has read O_{i-2};
* the warps read O_i only after it completed;
* the producer reloads a stage only after O_{i-2}, its last reader, completed.
"""
import random

import pytest

STAGES = 2
WARPS = 4


class Bar:
    """mbarrier: `count` arrivals (+ transaction units) complete a phase."""

    def __init__(self, count):
        self.count, self.pending, self.tx, self.completed = count, count, 0, 0

    def arrive(self, n=1, expect_tx=0):
        self.tx += expect_tx
        self.pending -= n
        assert self.pending >= 0, "more arrivals than the barrier's count in one phase"
        self._settle()

    def complete_tx(self, n=1):
        self.tx -= n
        self._settle()

    def _settle(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = self.count

    def ready(self, parity):
        return (self.completed & 1) != parity


def run(n, seed, skip=None):
    rnd = random.Random(seed)
    k_full = [Bar(1) for _ in range(STAGES)]
    v_full = [Bar(1) for _ in range(STAGES)]
    kv_empty = [Bar(1) for _ in range(STAGES)]
    s_full = [Bar(1), Bar(1)]
    s_free = [Bar(WARPS), Bar(WARPS)]
    q_full = Bar(WARPS)
    p_full, o_full, o_free = [Bar(WARPS), Bar(WARPS)], [Bar(1), Bar(1)], [Bar(WARPS), Bar(WARPS)]
    st = {"k": [None] * STAGES, "v": [None] * STAGES, "S": [None, None], "O": [None, None],
          "P": [[None] * WARPS, [None] * WARPS], "Q": [False] * WARPS}
    s_read = {}                  # tile -> warps done reading S_i
    o_read = {}                  # tile -> warps done reading O_i
    done = {"S": set(), "O": set()}
    tma = []                     # pending TMA completions (any order)
    tensor = []                  # pending tensor-core ops (issue order)

    def producer():
        for i in range(n):
            s = i % STAGES
            if i >= STAGES:
                if skip != "kv_empty":
                    yield lambda: kv_empty[s].ready(((i // STAGES) - 1) & 1)
                assert i - STAGES in done["O"] and i - STAGES in done["S"], f"stage {s} reloaded while tile {i - STAGES} in use"
            st["k"][s] = st["v"][s] = None          # being overwritten
            k_full[s].arrive(expect_tx=1)
            tma.append(("k", s, i))
            v_full[s].arrive(expect_tx=1)
            tma.append(("v", s, i))
            yield None

    def check_s(i, s, sb):
        assert all(st["Q"]), "S reads Q before every warp wrote it"
        assert st["k"][s] == i, f"S_{i} reads stage {s} holding {st['k'][s]}"

    def check_o(i, s):
        assert st["P"][i & 1] == [i] * WARPS, f"O_{i} reads P {st['P'][i & 1]}"
        assert st["v"][s] == i, f"O_{i} reads V stage {s} holding {st['v'][s]}"

    def issue_s(i):
        s, sb = i % STAGES, i & 1
        yield lambda: k_full[s].ready((i // STAGES) & 1)
        if i >= 2 and skip != "s_free":
            yield lambda: s_free[sb].ready(((i - 2) >> 1) & 1)
        if i >= 2:
            assert len(s_read.get(i - 2, ())) == WARPS, f"S_{i} overwrites S_{i - 2} still being read"
        check_s(i, s, sb)
        st["S"][sb] = None
        tensor.append(("S", i, s, sb))

    def mma():
        if skip != "q_full":
            yield lambda: q_full.ready(0)
        yield from issue_s(0)
        for i in range(n):
            if i + 1 < n:
                yield from issue_s(i + 1)
            s, pb = i % STAGES, i & 1
            if skip != "p_full":
                yield lambda: p_full[pb].ready((i >> 1) & 1)
            yield lambda: v_full[s].ready((i // STAGES) & 1)
            if i >= 2 and skip != "o_free":
                yield lambda: o_free[pb].ready(((i - 2) >> 1) & 1)
            if i >= 2:
                assert len(o_read.get(i - 2, ())) == WARPS, f"O_{i} overwrites O_{i - 2} still being read"
            check_o(i, s)
            st["O"][pb] = None
            tensor.append(("O", i, s, pb))

    def fold(w, j):
        """Warp w folds O_j (after the softmax of tile j + 1, or at the end)."""
        ob = j & 1
        if skip != "o_full":
            yield lambda: o_full[ob].ready((j >> 1) & 1)
        assert st["O"][ob] == j, f"warp {w} reads O buffer {ob} holding {st['O'][ob]} for tile {j}"
        yield None
        assert st["O"][ob] == j, f"warp {w}: O buffer {ob} overwritten while being read (tile {j})"
        o_read.setdefault(j, set()).add(w)
        o_free[ob].arrive()

    def warp(w):
        yield None
        st["Q"][w] = True
        q_full.arrive()
        yield None
        for i in range(n):
            sb, pb = i & 1, i & 1
            yield lambda: s_full[sb].ready((i >> 1) & 1)
            assert st["S"][sb] == i, f"warp {w} reads S buffer {sb} holding {st['S'][sb]} for tile {i}"
            yield None                              # pass 1 (row max) ... pass 2
            assert st["S"][sb] == i, f"warp {w}: S buffer {sb} overwritten during the softmax of tile {i}"
            if i >= 2:
                assert i - 2 in done["O"], f"warp {w} writes P_{i} while O_{i - 2} may read its buffer"
            st["P"][pb][w] = i
            s_read.setdefault(i, set()).add(w)
            s_free[sb].arrive()
            p_full[pb].arrive()
            if i >= 1:
                yield from fold(w, i - 1)
        if n:
            yield from fold(w, n - 1)

    def complete_tensor():
        kind, i, s, sb = tensor.pop(0)
        if kind == "S":
            check_s(i, s, sb)
            st["S"][sb] = i
            done["S"].add(i)
            s_full[sb].arrive()
        else:
            check_o(i, s)
            st["O"][sb] = i
            done["O"].add(i)
            kv_empty[s].arrive()        # both commits follow O_i
            o_full[sb].arrive()

    def complete_tma(j):
        kind, s, i = tma.pop(j)
        st[kind][s] = i
        (k_full if kind == "k" else v_full)[s].complete_tx()

    actors = [[producer(), None, False], [mma(), None, False]] + [[warp(w), None, False] for w in range(WARPS)]
    steps = 0
    while any(not a[2] for a in actors) or tma or tensor:
        ready = [a for a in actors if not a[2] and (a[1] is None or a[1]())]
        choices = [("actor", a) for a in ready] + [("tma", j) for j in range(len(tma))]
        if tensor:
            choices.append(("tensor", None))
        assert choices, "deadlock"
        kind, x = rnd.choice(choices)
        if kind == "actor":
            try:
                x[1] = next(x[0])
            except StopIteration:
                x[2] = True
        elif kind == "tma":
            complete_tma(x)
        else:
            complete_tensor()
        steps += 1
        assert steps < 200_000
    assert done["O"] == set(range(n))


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("seed", range(20))
def test_tc_attention_pipeline(n, seed):
    run(n, seed)


@pytest.mark.parametrize("skip", ["s_free", "o_free"])
@pytest.mark.parametrize("seed", range(20))
def test_the_buffer_free_waits_are_implied(skip, seed):
    """Every warp publishes P_i after its last read of S_{i-1} and of O_{i-2},
    and the issuer waits for P_i before O_i (and for P_{i-1} before S_{i+1}):
    the kernel's s_free and o_free waits are second guards of orders the P
    hand-off already gives, and the model finishes without either."""
    run(6, seed, skip=skip)


@pytest.mark.parametrize("skip", ["kv_empty", "q_full", "p_full", "o_full"])
def test_the_check_catches_a_missing_wait(skip):
    """The check of the check: without the stage-empty, Q, P or O hand-off
    some schedule reads or overwrites a buffer out of turn."""
    hit = False
    for seed in range(200):
        try:
            run(5, seed, skip=skip)
        except AssertionError:
            hit = True
            break
    assert hit

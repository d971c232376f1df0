"""The tcgen05 GEMM's two work schedules, restated on the CPU (nothing runs
on a GPU): how tsds_tc_gemm (tri_sds_b200/csrc/gemm_tc.cu) sizes the grid
and how each unit (a CTA, or a CTA pair) picks its (tile, k-block)
iterations.

* stream-K (default): unit u takes the contiguous iterations
  [u*W/PU, (u+1)*W/PU) of the flattened W = tiles x KT space; a tile cut by
  a range boundary is "split" and its contributors exchange fp32 partials.
  The epilogue keeps at most two pending split tiles per unit (registers
  pend0 / pend1) and finds a split tile's contributors as the consecutive
  units owner_of(first k-block) .. owner_of(last k-block).  Each split
  tile's rows are summed by its reducers (split_reducers in
  tri_sds_b200/csrc/tc_core.cuh), one slice each, and no unit reduces more
  than one tile.
* data-parallel (tsds_set_gemm_dp_rows, where its makespan of
  ceil(tiles / PU) tiles with PU = min(tiles, units) exceeds the ideal
  tiles / units by at most the slack, tsds_set_gemm_dp_slack, default 100%):
  unit u takes the whole tiles [u*tiles/PU, (u+1)*tiles/PU); nothing is
  split.

The checks pin the invariants the kernel relies on at the projection
shapes of the Qwen3-32B-shape target and the Qwen3-4B-shape draft."""
import pytest

SMS = 148
SMEM_PER_SM, SMEM_RESERVE, SMEM_BUDGET, A_STAGE, BK, MAX_STAGES = 233472, 8192, 220 * 1024, 16384, 64, 16


def it_begin(p, P, W):
    return p * W // P


def owner_of(x, P, W):
    q = min(x * P // W, P - 1)
    while q + 1 < P and it_begin(q + 1, P, W) <= x:
        q += 1
    while q > 0 and it_begin(q, P, W) > x:
        q -= 1
    return q


def two_split(q, P, W, KT):
    qb, qe = it_begin(q, P, W), it_begin(q + 1, P, W)
    if qe <= qb:
        return False
    f, l = qb // KT, (qe - 1) // KT
    return (f != l and owner_of(f * KT, P, W) != owner_of(f * KT + KT - 1, P, W)
            and owner_of(l * KT, P, W) != owner_of(l * KT + KT - 1, P, W))


def split_reducers(q_lo, q_hi, P, W, KT):
    return q_hi - q_lo + 1 - (1 if q_hi != q_lo and two_split(q_hi, P, W, KT) else 0)


def pow2_at_least(x):
    v = 32
    while v < x:
        v <<= 1
    return v


def plan(M, n_out, K, swiglu=False, ctas_setting=2, dp_rows=0, CG=1, slack=15):
    """tsds_tc_gemm's host arithmetic: (tiles, KT, PU, dp, stages)."""
    npad = (M + 15) // 16 * 16
    KT = (K + BK - 1) // BK
    tiles = (n_out + 64 * CG - 1) // (64 * CG) if swiglu else (n_out + 128 * CG - 1) // (128 * CG)
    tmem_cols = pow2_at_least(npad)
    ctas = ctas_setting
    while ctas > 1 and 2 * tmem_cols * ctas > 512:
        ctas -= 1
    budget = min(SMEM_PER_SM // ctas - SMEM_RESERVE, SMEM_BUDGET)
    stages = min((budget - 1024) // (A_STAGE + npad // CG * BK * 2), MAX_STAGES)
    W = tiles * KT
    units = SMS * ctas // CG
    PU = min(W, units)
    dp = False
    if dp_rows > 0 and M >= dp_rows:
        pu = min(tiles, units)
        if -(-tiles // pu) * units * 100 <= tiles * (100 + slack):
            dp, PU = True, pu
    assert W * PU < 2 ** 32
    return tiles, KT, PU, dp, stages


def ranges(tiles, KT, PU, dp):
    W = tiles * KT
    if dp:
        return [((u * tiles // PU) * KT, ((u + 1) * tiles // PU) * KT) for u in range(PU)]
    return [(it_begin(u, PU, W), it_begin(u + 1, PU, W)) for u in range(PU)]


# (n_out, K, swiglu) of each projection: 32B q/k/v, O, gate/up, down, LM head; 4B q/k/v, gate/up, down
PROJ = [(10240, 5120, False), (5120, 8192, False), (25600, 5120, True), (5120, 25600, False),
        (151936, 5120, False), (6144, 2560, False), (9728, 2560, True), (2560, 9728, False)]


@pytest.mark.parametrize("M", [1, 5, 26, 40, 208, 256])
@pytest.mark.parametrize("n_out,K,swiglu", PROJ)
@pytest.mark.parametrize("dp_rows,slack", [(0, 15), (1, 15), (1, 100), (1, 1000)])
def test_every_iteration_once_and_split_tiles_as_the_epilogue_expects(M, n_out, K, swiglu, dp_rows, slack):
    tiles, KT, PU, dp, stages = plan(M, n_out, K, swiglu, dp_rows=dp_rows, slack=slack)
    assert stages >= 2
    rs = ranges(tiles, KT, PU, dp)
    # the units' ranges tile the iteration space in order, none empty
    assert rs[0][0] == 0 and rs[-1][1] == tiles * KT
    assert all(rs[u][1] == rs[u + 1][0] for u in range(PU - 1))
    assert all(b < e for b, e in rs)
    for u, (b, e) in enumerate(rs):
        split = []
        for t in range(b // KT, (e - 1) // KT + 1):
            tb = t * KT
            k0, k1 = max(b, tb) - tb, min(e, tb + KT) - tb
            if (k0, k1) != (0, KT):
                split.append(t)
                if not dp:   # contributors: consecutive units whose ranges cover the tile
                    lo, hi = owner_of(tb, PU, tiles * KT), owner_of(tb + KT - 1, PU, tiles * KT)
                    assert lo <= u <= hi
                    assert rs[lo][0] <= tb < rs[lo][1] and rs[hi][0] <= tb + KT - 1 < rs[hi][1]
        assert len(split) <= 2           # pend0 / pend1
        if dp:
            assert not split             # nothing to exchange


@pytest.mark.parametrize("n_out,K,swiglu", PROJ)
@pytest.mark.parametrize("slack", [15, 100])
def test_data_parallel_only_within_the_slack(n_out, K, swiglu, slack):
    for M in (1, 26, 208):
        tiles, KT, PU, dp, _ = plan(M, n_out, K, swiglu, dp_rows=1, slack=slack)
        units = plan(M, n_out, K, swiglu)[2]   # stream-K's units (every projection has W >= units)
        if dp:   # balanced to one tile; the longest unit within the slack of the ideal
            per = [e // KT - b // KT for b, e in ranges(tiles, KT, PU, True)]
            assert PU <= tiles and min(per) >= 1 and max(per) - min(per) <= 1
            assert max(per) <= (1 + slack / 100) * tiles / units + 1e-9
        # off by default and below the row threshold
        assert not plan(M, n_out, K, swiglu)[3]
        assert not plan(M, n_out, K, swiglu, dp_rows=M + 1)[3]


def test_the_large_token_count_gate_up_is_data_parallel():
    """B=8 tree verify (M = 208): one CTA per SM (the accumulators fill TMEM),
    400 SwiGLU tiles over 148 units - 2 or 3 whole tiles each."""
    tiles, KT, PU, dp, stages = plan(208, 25600, 5120, True, dp_rows=128)
    assert (tiles, KT, PU, dp) == (400, 80, 148, True)
    per = sorted({e // KT - b // KT for b, e in ranges(tiles, KT, PU, True)})
    assert per == [2, 3]
    # at M = 26 (two CTAs per SM, 296 units) the 400 tiles would round up to
    # 2 per unit against a mean of 1.35: stream-K stays
    assert not plan(26, 25600, 5120, True, dp_rows=1)[3]
    # the LM head at M = 208: 1187 tiles, 8 or 9 per unit
    assert plan(208, 151936, 5120, dp_rows=128)[3]
    # q/k/v at M = 208: 80 tiles for 148 units - data-parallel on 80 CTAs only
    # with a slack of at least 85% (148 / 80 = 1.85)
    assert not plan(208, 10240, 5120, dp_rows=128)[3]
    assert plan(208, 10240, 5120, dp_rows=128, slack=84)[3] is False
    assert plan(208, 10240, 5120, dp_rows=128, slack=85)[2:4] == (80, True)


def _library_plan(epi, M, n_out, K):
    import ctypes

    from tri_sds_b200 import _lib
    out = (ctypes.c_int32 * 6)()
    st = _lib.load().tsds_tc_gemm_plan(epi, M, n_out, K, out)
    assert st == 0, st
    return list(out)


@pytest.fixture()
def switches():
    from tri_sds_b200 import _lib
    lib = _lib.load()
    yield lib
    lib.tsds_set_gemm_dp_rows(_lib.GEMM_DP_ROWS_DEFAULT)
    lib.tsds_set_gemm_dp_slack(_lib.GEMM_DP_SLACK_DEFAULT)
    lib.tsds_set_gemm_ctas_per_sm(2)


@pytest.mark.parametrize("dp_rows,slack,ctas", [(0, 15, 2), (1, 15, 2), (128, 100, 2), (1, 15, 1), (1, 1000, 3)])
def test_the_restatement_is_the_library_arithmetic(switches, dp_rows, slack, ctas):
    """tsds_tc_gemm_plan (the host planning tsds_tc_gemm launches with) gives
    the restatement's tiles, k-blocks, grid, schedule and stages at every
    projection shape and row count (one-CTA tiles; the library assumes 148
    SMs where no GPU answers, as here)."""
    switches.tsds_set_gemm_dp_rows(dp_rows)
    switches.tsds_set_gemm_dp_slack(slack)
    switches.tsds_set_gemm_ctas_per_sm(ctas)
    for n_out, K, swiglu in PROJ:
        for M in (1, 5, 26, 40, 129, 208, 256):
            tiles, KT, PU, dp, stages = plan(M, n_out, K, swiglu, ctas_setting=ctas, dp_rows=dp_rows, slack=slack)
            got = _library_plan(2 if swiglu else 0, M, n_out, K)
            assert got == [tiles, KT, PU, int(dp), stages, 1], (n_out, K, M, got)


@pytest.mark.parametrize("M", [1, 26, 208])
@pytest.mark.parametrize("n_out,K,swiglu", PROJ)
@pytest.mark.parametrize("CG", [1, 2])
def test_each_split_tile_row_is_reduced_once_and_no_unit_reduces_twice(M, n_out, K, swiglu, CG):
    """The DIST epilogue: a unit with two split tiles reduces a slice of its
    last one only; reducer c of a tile's nr takes rows [c*R/nr, (c+1)*R/nr).
    Every row of every split tile is summed exactly once, by one unit."""
    tiles, KT, PU, dp, _ = plan(M, n_out, K, swiglu, CG=CG)
    assert not dp
    W = tiles * KT
    rows = 64 if swiglu else 128
    covered, per_unit = {}, [0] * PU
    for u, (b, e) in enumerate(ranges(tiles, KT, PU, dp)):
        pend = [t for t in range(b // KT, (e - 1) // KT + 1)
                if (max(b, t * KT) - t * KT, min(e, t * KT + KT) - t * KT) != (0, KT)]
        assert (len(pend) == 2) == two_split(u, PU, W, KT)
        for t in (pend[1:] if len(pend) == 2 else pend):
            lo, hi = owner_of(t * KT, PU, W), owner_of(t * KT + KT - 1, PU, W)
            nr = split_reducers(lo, hi, PU, W, KT)
            c = u - lo
            assert 0 <= c < nr
            covered.setdefault(t, []).append((c * rows // nr, (c + 1) * rows // nr))
            per_unit[u] += 1
    assert max(per_unit) <= 1
    for t in range(tiles):
        lo, hi = owner_of(t * KT, PU, W), owner_of(t * KT + KT - 1, PU, W)
        if lo == hi:
            assert t not in covered
            continue
        sl = sorted(covered[t])
        assert len(sl) == split_reducers(lo, hi, PU, W, KT)
        assert sl[0][0] == 0 and sl[-1][1] == rows
        assert all(sl[i][1] == sl[i + 1][0] for i in range(len(sl) - 1))

"""Launch plans built on the CPU (nothing runs): under tensor parallelism the
calls that describe a rank's sharded buffers get the rank's sizes.

A plan records each C-ABI call with its arguments; building one needs no GPU.
The EAGLE cycle at TP=8 (one kv head per rank) once passed the model's global
kv-head count to the KV compaction, which then addressed past the rank's
cache; these checks pin every such size to the buffer it describes."""
import torch

from tri_sds_b200.shapes import QwenShape

SHAPE = QwenShape(hidden=256, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=1024, n_layers=2, vocab=1024)


class _Comm:
    """Collectives are recorded in plans, never called here."""

    def __init__(self, rank, size):
        self.rank, self.size = rank, size

    def all_reduce(self, t):
        raise AssertionError("not called while building a plan")

    def all_gather(self, out, inp):
        raise AssertionError("not called while building a plan")


def _calls(plan, name):
    return [args for n, fn, args in plan.calls if n == name]


def _eagle(tp):
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    t = QwenModel(SHAPE, 1, 64, 26, device="cpu", tp_rank=0, tp_size=tp, comm=_Comm(0, tp) if tp > 1 else None)
    return t, EagleEngine(t, EagleHead(t, 1), use_graph=False)


def test_tp8_plan_uses_the_rank_shard_sizes():
    t, eng = _eagle(8)
    hq, hkv = SHAPE.n_heads // 8, SHAPE.n_kv_heads // 8
    assert t.k_cache.shape[2] == hkv == 1
    (commit,) = _calls(eng.plan, "tsds_tree_commit")
    assert commit[4] == t.k_cache.shape[2] and commit[5] == t.k_cache.shape[3]
    # target attention / RoPE calls: the rank's heads; the replicated head's: all heads
    target_attn = [a for a in _calls(eng.plan, "tsds_verify_attention") if a[7] * a[8] == 26]
    assert target_attn and all((a[9], a[10]) == (hq, hkv) for a in target_attn)
    head_attn = [a for a in _calls(eng.plan, "tsds_verify_attention") if a[7] * a[8] != 26]
    assert head_attn and all((a[9], a[10]) == (SHAPE.n_heads, SHAPE.n_kv_heads) for a in head_attn)
    for a in _calls(eng.plan, "tsds_qk_norm_rope_kv"):
        assert (a[12], a[13]) in ((hq, hkv), (SHAPE.n_heads, SHAPE.n_kv_heads))
    # row-parallel projections of the target produce fp32 partials, all-reduced
    assert len(_calls(eng.plan, "tsds_linear_f32")) == 2 * SHAPE.n_layers
    assert sum(1 for n, fn, _ in eng.plan.calls if n == "all_reduce") == 2 * SHAPE.n_layers
    # vocab-parallel LM head: the rank's shard of the vocabulary
    for a in _calls(eng.plan, "tsds_lm_head_argmax"):
        assert a[8] == SHAPE.vocab // 8


def test_tp1_plan_has_no_collectives():
    t, eng = _eagle(1)
    assert not any(fn is None for _, fn, _ in eng.plan.calls)
    (commit,) = _calls(eng.plan, "tsds_tree_commit")
    assert commit[4] == SHAPE.n_kv_heads
    for a in _calls(eng.plan, "tsds_lm_head_argmax"):
        assert a[8] == SHAPE.vocab


def test_tp8_chain_plan_shards_the_target_only():
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    t = QwenModel(SHAPE, 1, 64, 5, device="cpu", tp_rank=0, tp_size=8, comm=_Comm(0, 8))
    d = QwenModel(SHAPE, 1, 64, 2, device="cpu", tp_size=8, tp_layers=False, tp_vocab=False)
    eng = SpecEngine(t, d, 4, use_graph=False)
    for a in _calls(eng.plan, "tsds_verify_attention"):
        if a[8] == 5:   # the target's verify over K+1 rows
            assert (a[9], a[10]) == (SHAPE.n_heads // 8, SHAPE.n_kv_heads // 8)
        else:           # the replicated draft
            assert (a[9], a[10]) == (SHAPE.n_heads, SHAPE.n_kv_heads)
    vocabs = sorted({a[8] for a in _calls(eng.plan, "tsds_lm_head_argmax")})
    assert vocabs == [SHAPE.vocab // 8, SHAPE.vocab]


def test_tp8_chain_plan_with_a_tensor_parallel_draft():
    """The draft sharded over the target's ranks: its attention, RoPE and LM
    head calls get the rank's shard sizes, and each of its K forwards adds
    two all-reduces per layer."""
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    K = 4
    comm = _Comm(0, 8)
    t = QwenModel(SHAPE, 1, 64, 5, device="cpu", tp_rank=0, tp_size=8, comm=comm)
    d = QwenModel(SHAPE, 1, 64, 2, device="cpu", tp_rank=0, tp_size=8, comm=comm)
    eng = SpecEngine(t, d, K, use_graph=False)
    attn = _calls(eng.plan, "tsds_verify_attention")
    assert len(attn) == SHAPE.n_layers * (K + 1)
    assert all((a[9], a[10]) == (SHAPE.n_heads // 8, SHAPE.n_kv_heads // 8) for a in attn)
    for a in _calls(eng.plan, "tsds_qk_norm_rope_kv"):
        assert (a[12], a[13]) == (SHAPE.n_heads // 8, SHAPE.n_kv_heads // 8)
    assert {a[8] for a in _calls(eng.plan, "tsds_lm_head_argmax")} == {SHAPE.vocab // 8}
    n_ar = sum(1 for n, fn, _ in eng.plan.calls if n == "all_reduce")
    assert n_ar == 2 * SHAPE.n_layers * (K + 1)
    # the draft's cache holds the rank's kv heads only
    assert d.k_cache.shape[2] == SHAPE.n_kv_heads // 8

"""Every buffer a launch plan hands to the C ABI is large enough for the sizes
passed with it (CPU only: plans are built, nothing runs).

The plan-building modules turn tensors into raw pointers with ``_p``; here
``_p`` is replaced by a reference to the tensor itself, so each recorded
call's pointer arguments can be checked against the bytes their tensors
hold from the pointer to the end of their storage.  The extents follow the
argument meanings in include/tsds.h.  Plans of the EAGLE and chain engines
are checked under tensor parallelism of 1, 2, 4 and 8 ranks and batch 1, 2
and 8 - the kind of check that catches a rank's buffer described with the
model's global sizes."""
import pytest
import torch

from tri_sds_b200.shapes import QwenShape

SHAPE = QwenShape(hidden=256, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=1024, n_layers=2, vocab=1024)
DRAFT = QwenShape(hidden=256, n_heads=8, n_kv_heads=8, head_dim=128, intermediate=512, n_layers=2, vocab=1024)


class TRef:
    """Stands in for a pointer: the tensor (view) it points into."""

    def __init__(self, t):
        self.t = t

    def bytes_left(self):
        st = self.t.untyped_storage()
        return st.nbytes() - (self.t.data_ptr() - st.data_ptr())


@pytest.fixture()
def tensor_refs(monkeypatch):
    import tri_sds_b200.eagle as eagle
    import tri_sds_b200.engine as engine
    import tri_sds_b200.model as model
    ref = lambda t: None if t is None else TRef(t)  # noqa: E731
    for mod in (model, eagle, engine):
        monkeypatch.setattr(mod, "_p", ref)
    yield


class _Comm:
    def __init__(self, rank, size):
        self.rank, self.size = rank, size

    def all_reduce(self, t):
        raise AssertionError("not called while building a plan")

    def all_gather(self, out, inp):
        raise AssertionError("not called while building a plan")


def _extents(name, a):
    """[(arg index, bytes needed or None if the pointer is unused)] for one call."""
    if name == "tsds_embed":
        ids, stride, table, out, M, N, vocab = a
        return [(0, ((M - 1) * stride + 1) * 8), (2, vocab * N * 2), (3, M * N * 2)]
    if name == "tsds_rms_norm":
        x, w, out, rows, n, ldx, ldo, eps = a
        return [(0, ((rows - 1) * ldx + n) * 2), (1, n * 2), (2, ((rows - 1) * ldo + n) * 2)]
    if name == "tsds_prep_chain":
        base, off, B, T, starts, pos = a
        return [(0, B * 4), (4, B * 4), (5, B * T * 4)]
    if name == "tsds_qk_norm_rope_kv":
        qkv, qn, kn, cos, sin, pos, starts, q, kc, vc, B, T, Hq, Hkv, D, S, rope_len, eps = a
        return [(0, B * T * (Hq + 2 * Hkv) * D * 2), (1, D * 2), (2, D * 2), (3, rope_len * D // 2 * 2),
                (4, rope_len * D // 2 * 2), (5, B * T * 4), (6, B * 4), (7, B * T * Hq * D * 2),
                (8, B * Hkv * S * D * 2), (9, B * Hkv * S * D * 2)]
    if name in ("tsds_linear", "tsds_linear_swiglu", "tsds_linear_f32"):
        x, ldx, W, out, ldo, M, n_out, K, ws, wsb = a
        rows_w = 2 * n_out if name == "tsds_linear_swiglu" else n_out
        eb = 4 if name == "tsds_linear_f32" else 2
        return [(0, ((M - 1) * ldx + K) * 2), (2, rows_w * K * 2), (3, ((M - 1) * ldo + n_out) * eb), (8, wsb)]
    if name in ("tsds_linear_residual", "tsds_linear_bias"):
        x, ldx, W, res, out, ldo, M, n_out, K, ws, wsb = a
        res_b = n_out * 2 if name == "tsds_linear_bias" else ((M - 1) * ldo + n_out) * 2
        return [(0, ((M - 1) * ldx + K) * 2), (2, n_out * K * 2), (3, res_b), (4, ((M - 1) * ldo + n_out) * 2),
                (9, wsb)]
    if name == "tsds_logits_topk":
        lg, ld, M, V, k, vals, idx, lse = a
        return [(0, ((M - 1) * ld + V) * 2), (5, M * k * 4), (6, M * k * 4), (7, M * 4)]
    if name == "tsds_tree_init":
        states, cur, lengths, tok, frow, pos, mask, starts, B = a
        return [(1, B * 8), (2, B * 4), (3, B * 8), (4, B * 4), (5, B * 4), (6, B * 4), (7, B * 4)]
    if name == "tsds_tree_step":
        states, vals, idx, lse, row_base, T, k, next_T, lengths, tok, frow, pos, mask, starts, B = a
        rows = row_base + B * T
        nt = max(next_T, 1)
        return [(1, rows * k * 4), (2, rows * k * 4), (3, rows * 4), (8, B * 4), (9, B * nt * 8), (10, B * nt * 4),
                (11, B * nt * 4), (12, B * nt * 4), (13, B * 4)]
    if name == "tsds_tree_finalize":
        states, n_nodes, k, lengths, ids, pos, masks, hrow, children, starts, B = a
        NN = n_nodes + 1
        return [(3, B * 4), (4, B * NN * 8), (5, B * NN * 4), (6, B * NN * 4), (7, B * NN * 4),
                (8, B * NN * k * 4), (9, B * 4)]
    if name == "tsds_accept_tree":
        tl, ta, hl, ids, hrow, ch, U, scratch, path, acc, tokens, cur, B, n_nodes, V, k, depth = a
        NN = n_nodes + 1
        return [(0, B * NN * V * 2), (1, B * NN * 8), (2, V * 2), (3, B * NN * 8), (4, B * NN * 4),
                (5, B * NN * k * 4), (6, B * (depth + 1) * (k + 1) * 4), (8, B * (depth + 1) * 4), (9, B * 4),
                (10, B * (depth + 2) * 8), (11, B * 8)]
    if name == "tsds_tree_commit":
        kc, vc, layers, B, Hkv, S, D, lengths, path, acc, depth, hidden, n_nodes, N, root = a
        return [(0, layers * B * Hkv * S * D * 2), (1, layers * B * Hkv * S * D * 2), (7, B * 4),
                (8, B * (depth + 1) * 4), (9, B * 4), (11, B * (n_nodes + 1) * N * 2), (14, B * N * 2)]
    if name == "tsds_eagle_inputs":
        root, hfeat, frow, tok, emb, out, B, T, N, vocab = a
        return [(0, B * N * 2), (2, B * T * 4), (3, B * T * 8), (4, vocab * N * 2), (5, B * T * 2 * N * 2)]
    if name == "tsds_verify_attention":
        q, k, v, out, starts, mask, origin, B, T, Hq, Hkv, D, S, max_kv, split, scale, ws, wsb, status = a
        assert max_kv <= S
        return [(0, B * T * Hq * D * 2), (1, B * Hkv * S * D * 2), (2, B * Hkv * S * D * 2), (3, B * T * Hq * D * 2),
                (4, B * 4), (5, B * T * 4), (16, wsb), (18, 4)]
    if name == "tsds_lm_head_argmax":
        x, ldx, W, logits, am, stride, av, M, V, K, ws, wsb = a
        return [(0, ((M - 1) * ldx + K) * 2), (2, V * K * 2), (3, M * V * 2), (4, ((M - 1) * stride + 1) * 8),
                (6, M * 4), (10, wsb)]
    if name == "tsds_residual_add_f32":
        x, part, M, N = a
        return [(0, M * N * 2), (1, M * N * 4)]
    if name == "tsds_argmax_merge":
        vals, idx, M, tp, shard, out, stride = a
        return [(0, tp * M * 4), (1, tp * M * 8), (5, ((M - 1) * stride + 1) * 8)]
    if name == "tsds_gather_shards":
        src, dst, tp, M, vs = a
        return [(0, tp * M * vs * 2), (1, M * tp * vs * 2)]
    if name == "tsds_accept_greedy":
        draft, target, acc, tokens, tlen, last, cur, B, K = a
        return [(0, B * K * 8), (1, B * (K + 1) * 8), (2, B * 4), (3, B * (K + 1) * 8), (4, B * 4), (5, B * 8),
                (6, B * 8)]
    if name == "tsds_gather_ids":
        cur, last, draft, vids, d2, B, K = a
        return [(0, B * 8), (1, B * 8), (2, B * K * 8), (3, B * (K + 1) * 8), (4, B * 2 * 8)]
    raise AssertionError(f"no extent rule for {name}")


def _check(plan):
    n = 0
    for name, fn, args in plan.calls:
        if fn is None:
            continue
        for i, need in _extents(name, args):
            ref = args[i]
            if ref is None:
                continue
            assert isinstance(ref, TRef), (name, i, ref)
            assert need <= ref.bytes_left(), (name, i, need, ref.bytes_left())
            n += 1
    return n


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 1), (4, 0), (8, 7)])
@pytest.mark.parametrize("B", [1, 2, 8])
def test_eagle_plans_fit_their_buffers(tensor_refs, tp, rank, B):
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    t = QwenModel(SHAPE, B, 96, B * 26, device="cpu", tp_rank=rank, tp_size=tp,
                  comm=_Comm(rank, tp) if tp > 1 else None)
    eng = EagleEngine(t, EagleHead(t, B), use_graph=False)
    assert _check(eng.plan) > 100
    _check(eng.verify_only_plan())


@pytest.mark.parametrize("tp,rank", [(1, 0), (8, 3)])
@pytest.mark.parametrize("B", [1, 8])
def test_chain_plans_fit_their_buffers(tensor_refs, tp, rank, B):
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    K = 4
    t = QwenModel(SHAPE, B, 96, B * (K + 1), device="cpu", tp_rank=rank, tp_size=tp,
                  comm=_Comm(rank, tp) if tp > 1 else None)
    d = QwenModel(DRAFT, B, 96, B * 2, device="cpu", tp_size=tp, tp_layers=False, tp_vocab=False)
    eng = SpecEngine(t, d, K, use_graph=False)
    assert _check(eng.plan) > 50
    _check(eng.verify_only_plan())


def test_the_check_catches_a_global_size_on_a_shard(tensor_refs):
    """The kv-head count of the model instead of the rank's cache overruns it."""
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    t = QwenModel(SHAPE, 1, 96, 26, device="cpu", tp_rank=0, tp_size=8, comm=_Comm(0, 8))
    eng = EagleEngine(t, EagleHead(t, 1), use_graph=False)
    for i, (name, fn, args) in enumerate(eng.plan.calls):
        if name == "tsds_tree_commit":
            args = list(args)
            args[4] = SHAPE.n_kv_heads
            eng.plan.calls[i] = (name, fn, tuple(args))
    with pytest.raises(AssertionError):
        _check(eng.plan)

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

from abi_extents import TRef, check_call
from tri_sds_b200.shapes import QwenShape

SHAPE = QwenShape(hidden=256, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=1024, n_layers=2, vocab=1024)
DRAFT = QwenShape(hidden=256, n_heads=8, n_kv_heads=8, head_dim=128, intermediate=512, n_layers=2, vocab=1024)


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


def _check(plan):
    return sum(check_call(name, args) for name, fn, args in plan.calls if fn is not None)


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


@pytest.mark.parametrize("tp,rank,draft_tp", [(1, 0, False), (8, 3, False), (2, 1, True), (8, 3, True)])
@pytest.mark.parametrize("B", [1, 8])
def test_chain_plans_fit_their_buffers(tensor_refs, tp, rank, draft_tp, B):
    """The draft replicated, or tensor-parallel over the target's ranks."""
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    K = 4
    comm = _Comm(rank, tp) if tp > 1 else None
    t = QwenModel(SHAPE, B, 96, B * (K + 1), device="cpu", tp_rank=rank, tp_size=tp, comm=comm)
    if draft_tp:
        d = QwenModel(DRAFT, B, 96, B * 2, device="cpu", tp_rank=rank, tp_size=tp, comm=comm)
    else:
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

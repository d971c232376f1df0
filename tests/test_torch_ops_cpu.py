"""``torch.ops.tsds`` on CPU (nothing runs on a device).

* every op is registered with the schema its in-place arguments need;
* host tensors are refused (there is no CPU implementation);
* with the library call replaced by a recorder and pointers by references to
  their tensors, each op hands the C ABI the entry points it stands for and
  buffers that reach the extents include/tsds.h gives for the sizes passed
  with them;
* index arguments that a kernel follows unchecked are range-checked first."""
import pytest
import torch

from abi_extents import TRef, check_call

bf16, i32, i64, f32 = torch.bfloat16, torch.int32, torch.int64, torch.float32
_STREAM = object()


def _ops():
    import tri_sds_b200.torch_ops  # noqa: F401  (registers the ops)
    return torch.ops.tsds


def test_every_op_is_registered_with_its_mutations():
    import tri_sds_b200.torch_ops as T
    tsds = _ops()
    mutated = {}
    for name in T.OPS:
        schema = getattr(tsds, name).default._schema
        mutated[name] = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
    assert mutated == {
        "qkv_rope_fused": {"k_cache", "v_cache"},
        "verify_attention": set(),
        "oproj_fused": set(),
        "mlp_fused": set(),
        "lm_head_topk": set(),
        "eagle_fc": set(),
        "accept_greedy": {"lengths", "last", "cur"},
        "accept_rejection": set(),
        "kv_compact": {"k_cache", "v_cache", "lengths", "root_feat"},
        "allreduce_oneshot": {"x"},
    }


class _Recorder:
    def __init__(self):
        self.calls = []

    def __call__(self, name, *args):
        self.calls.append(name)
        assert args[-1] is _STREAM, name   # every launch goes to the current stream
        assert check_call(name, args[:-1]) > 0, name


@pytest.fixture()
def recorded(monkeypatch):
    """Kernels replaced by a recorder that checks extents; host tensors of the
    right dtype pass the device checks."""
    from tri_sds_b200 import _lib, ops

    def dtype_only(dtype, *ts):
        for t in ts:
            if t is not None:
                ops._need(t.dtype == dtype, f"expected {dtype}")

    rec = _Recorder()
    monkeypatch.setattr(ops, "_p", lambda t: None if t is None else TRef(t))
    monkeypatch.setattr(ops, "_stream", lambda: _STREAM)
    monkeypatch.setattr(ops, "_cuda", dtype_only)
    monkeypatch.setattr(ops, "_bf16_cuda", lambda *ts: dtype_only(bf16, *ts))
    monkeypatch.setattr(_lib, "call", rec)
    yield rec


def _r(*shape, dtype=bf16):
    return torch.randn(*shape).to(dtype)


B, T, HQ, HKV, D, S, N, I, V = 2, 5, 4, 2, 128, 64, 256, 512, 1000


def _qkv_args():
    return (_r(B * T, N), _r(N), _r((HQ + 2 * HKV) * D, N), _r(D), _r(D), _r(S, D // 2), _r(S, D // 2),
            torch.arange(B * T, dtype=i32), torch.tensor([3, 7], dtype=i32), _r(B, HKV, S, D), _r(B, HKV, S, D),
            HQ, HKV)


def test_qkv_rope_fused(recorded):
    q = _ops().qkv_rope_fused(*_qkv_args())
    assert q.shape == (B * T, HQ * D)
    assert recorded.calls == ["tsds_rms_norm", "tsds_linear", "tsds_qk_norm_rope_kv"]


@pytest.mark.parametrize("tree", [False, True])
def test_verify_attention(recorded, tree):
    mask = torch.full((B, T), 1, dtype=i32) if tree else None
    o = _ops().verify_attention(_r(B, T, HQ, D), _r(B, HKV, S, D), _r(B, HKV, S, D), torch.tensor([3, 7], dtype=i32),
                                mask)
    assert o.shape == (B, T, HQ, D)
    assert recorded.calls == ["tsds_verify_attention"]


def test_oproj_and_mlp(recorded):
    x = _r(B * T, N)
    assert _ops().oproj_fused(_r(B * T, HQ * D), _r(N, HQ * D), x).shape == x.shape
    assert _ops().mlp_fused(x, _r(N), _r(2 * I, N), _r(N, I)).shape == x.shape
    assert recorded.calls == ["tsds_linear_residual", "tsds_rms_norm", "tsds_linear_swiglu", "tsds_linear_residual"]


@pytest.mark.parametrize("k", [1, 4, 8])
def test_lm_head_topk(recorded, k):
    logits, vals, idx, lse = _ops().lm_head_topk(_r(3, N), _r(N), _r(V, N), k)
    assert logits.shape == (3, V) and vals.shape == idx.shape == (3, k) and lse.shape == (3,)
    assert (vals.dtype, idx.dtype, lse.dtype) == (f32, i32, f32)
    assert recorded.calls == ["tsds_rms_norm", "tsds_lm_head_argmax", "tsds_logits_topk"]


def test_lm_head_topk_k_must_be_supported(recorded):
    with pytest.raises(ValueError):
        _ops().lm_head_topk(_r(3, N), _r(N), _r(V, N), 3)
    assert recorded.calls == []


def test_eagle_fc(recorded):
    out = _ops().eagle_fc(_r(7, N), torch.randint(0, V, (7,)), _r(V, N), _r(N, 2 * N), _r(N))
    assert out.shape == (7, N)
    assert recorded.calls == ["tsds_eagle_inputs", "tsds_linear_bias"]


def test_accept_greedy(recorded):
    K = 4
    acc, tokens = _ops().accept_greedy(torch.zeros(B, K, dtype=i64), torch.zeros(B, K + 1, dtype=i64),
                                       torch.zeros(B, dtype=i32), torch.zeros(B, dtype=i64), torch.zeros(B, dtype=i64))
    assert acc.shape == (B,) and tokens.shape == (B, K + 1)
    assert recorded.calls == ["tsds_accept_greedy"]


def _tree(k=2, depth=2):
    """A 5-node tree per sequence: 0 -> {1, 2}, 1 -> {3, 4}; head rows 0, 1."""
    NN = 5
    children = torch.full((B, NN, k), -1, dtype=i32)
    children[:, 0] = torch.tensor([1, 2], dtype=i32)
    children[:, 1] = torch.tensor([3, 4], dtype=i32)
    hrow = torch.full((B, NN), -1, dtype=i32)
    hrow[:, 0], hrow[:, 1] = 0, 1
    ids = torch.randint(0, V, (B, NN))
    return NN, k, depth, ids, hrow, children


@pytest.mark.parametrize("greedy", [False, True])
def test_accept_rejection(recorded, greedy):
    NN, k, depth, ids, hrow, children = _tree()
    U = None if greedy else torch.rand(B, depth + 1, k + 1)
    am = torch.randint(0, V, (B * NN,)) if greedy else None
    path, acc, tokens, bonus = _ops().accept_rejection(_r(B * NN, V), _r(2, V), ids, hrow, children, U, am, depth)
    assert path.shape == (B, depth + 1) and acc.shape == (B,) and tokens.shape == (B, depth + 2)
    assert bonus.shape == (B,)
    assert recorded.calls == ["tsds_accept_tree_rule"]


def test_accept_rejection_checks_its_indices(recorded):
    NN, k, depth, ids, hrow, children = _tree()
    U = torch.rand(B, depth + 1, k + 1)
    bad = children.clone()
    bad[1, 1, 0] = NN
    with pytest.raises(ValueError, match="children"):
        _ops().accept_rejection(_r(B * NN, V), _r(2, V), ids, hrow, bad, U, None, depth)
    bad = hrow.clone()
    bad[0, 1] = 2            # node 1 has children; only head rows 0, 1 exist
    with pytest.raises(ValueError, match="hrow"):
        _ops().accept_rejection(_r(B * NN, V), _r(2, V), ids, bad, children, U, None, depth)
    bad[0, 1] = 1
    bad[0, 3] = 9            # node 3 is a leaf: its head row is never read
    _ops().accept_rejection(_r(B * NN, V), _r(2, V), ids, bad, children, U, None, depth)
    assert recorded.calls == ["tsds_accept_tree_rule"]


def _commit_args(depth=2, NN=5, layers=3):
    path = torch.tensor([[1, 3, -1], [2, -1, -1]], dtype=i32)
    acc = torch.tensor([2, 1], dtype=i32)
    return (_r(layers, B, HKV, S, D), _r(layers, B, HKV, S, D), torch.tensor([10, 20], dtype=i32), path, acc,
            _r(B * NN, N), _r(B, N), depth)


def test_kv_compact(recorded):
    args = _commit_args()
    _ops().kv_compact(*args)
    assert recorded.calls == ["tsds_tree_commit"]


@pytest.mark.parametrize("field,index,value", [(3, (0, 1), 5), (3, (1, 0), -1), (4, (0,), 3), (2, (1,), S)])
def test_kv_compact_checks_its_indices(recorded, field, index, value):
    args = list(_commit_args())
    args[field] = args[field].clone()
    args[field][index] = value
    with pytest.raises(ValueError, match="out of range"):
        _ops().kv_compact(*args)
    assert recorded.calls == []


class _FakeGroup:
    """tp.PeerAllReduce's op-level interface with host tensors as slots."""

    def __init__(self, rank, size, max_elems):
        import ctypes
        import tri_sds_b200.tp as tp
        self.rank, self.size, self.max_elems = rank, size, max_elems
        self.slots = [torch.zeros(max_elems, dtype=torch.float32) for _ in range(2)]
        self.bufs = (ctypes.c_void_p * size)(*[0x1000 * (q + 1) for q in range(size)])
        self.next_slot = tp.PeerAllReduce.next_slot.__get__(self)

    def slot_tensor(self, slot, n):
        return self.slots[slot][:n]


def test_allreduce_oneshot_alternates_slots(recorded):
    import tri_sds_b200.tp as tp
    M, N = 26, 256
    grp = _FakeGroup(1, 4, M * N)
    gid = tp.register_peer_group(grp)
    x = _r(M, N)
    seen = []
    for i in range(3):
        part = torch.full((M, N), float(i + 1))
        _ops().allreduce_oneshot(x, part, gid)
        seen.append(float(grp.slots[i % 2][0]))
    # the partial of call i sits in slot i % 2 when its kernel runs
    assert seen == [1.0, 2.0, 3.0] and float(grp.slots[0][0]) == 3.0 and float(grp.slots[1][0]) == 2.0
    assert recorded.calls == ["tsds_peer_allreduce_residual"] * 3


def test_allreduce_oneshot_checks_shapes(recorded):
    import tri_sds_b200.tp as tp
    gid = tp.register_peer_group(_FakeGroup(0, 2, 64))
    with pytest.raises(ValueError):
        _ops().allreduce_oneshot(_r(4, 32), torch.zeros(4, 32), gid)     # M * N > the group's slots
    with pytest.raises(ValueError):
        _ops().allreduce_oneshot(_r(2, 8), torch.zeros(2, 4), gid)       # partial of another shape
    assert recorded.calls == []


def test_host_tensors_are_refused():
    """No CPU implementation: the device checks reject host tensors before any
    pointer reaches the library."""
    tsds = _ops()
    NN, k, depth, ids, hrow, children = _tree()
    cases = [
        lambda: tsds.qkv_rope_fused(*_qkv_args()),
        lambda: tsds.verify_attention(_r(B, T, HQ, D), _r(B, HKV, S, D), _r(B, HKV, S, D),
                                      torch.tensor([3, 7], dtype=i32)),
        lambda: tsds.oproj_fused(_r(B * T, HQ * D), _r(N, HQ * D), _r(B * T, N)),
        lambda: tsds.mlp_fused(_r(B * T, N), _r(N), _r(2 * I, N), _r(N, I)),
        lambda: tsds.lm_head_topk(_r(3, N), _r(N), _r(V, N), 4),
        lambda: tsds.eagle_fc(_r(7, N), torch.randint(0, V, (7,)), _r(V, N), _r(N, 2 * N), _r(N)),
        lambda: tsds.accept_greedy(torch.zeros(B, 4, dtype=i64), torch.zeros(B, 5, dtype=i64),
                                   torch.zeros(B, dtype=i32), torch.zeros(B, dtype=i64), torch.zeros(B, dtype=i64)),
        lambda: tsds.accept_rejection(_r(B * NN, V), _r(2, V), ids, hrow, children, torch.rand(B, depth + 1, k + 1),
                                      None, depth),
        lambda: tsds.kv_compact(*_commit_args()),
        lambda: tsds.allreduce_oneshot(_r(4, 32), torch.zeros(4, 32), 0),
    ]
    for case in cases:
        with pytest.raises(ValueError, match="CUDA"):
            case()

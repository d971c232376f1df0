"""The fused-layer kernel's host side on CPU (nothing runs on a device).

* plans: one attention launch and one fused launch per layer, with the
  phases of the per-op plan in the same order (the first is layer 0's
  norm -> q/k/v, the last ends with the down projection);
* every pointer a phase or its RoPE block hands the library reaches the
  extent its sizes imply (pointers replaced by references to their tensors);
* the ctypes structures have the C layout of include/tsds.h (compiled with
  the host compiler);
* the entry point rejects bad descriptors before any CUDA call."""
import ctypes
import os
import subprocess

import pytest
import torch

from abi_extents import TRef, check_call
from tri_sds_b200.shapes import QwenShape

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPE = QwenShape(hidden=256, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=1024, n_layers=3, vocab=1024)


@pytest.fixture()
def recorded(monkeypatch):
    import tri_sds_b200.eagle as eagle
    import tri_sds_b200.engine as engine
    import tri_sds_b200.model as model
    ref = lambda t: None if t is None else TRef(t)  # noqa: E731
    for mod in (model, eagle, engine):
        monkeypatch.setattr(mod, "_p", ref)
    monkeypatch.setattr(model, "_fused_args",
                        lambda phases, rope, peer, M, ws, wsb: (phases, len(phases), M, rope, peer, ws, wsb))
    yield


def _phase_names(phases):
    names = {0: "store", 1: "res", 2: "swiglu", 4: "f32", 5: "qkrope"}
    return [{1: "norm", 2: "peer"}.get(ph["kind"]) or names[ph["epi"]] for ph in phases]


@pytest.mark.parametrize("B,T", [(1, 26), (8, 26), (2, 5)])
def test_fused_plan_shape_and_extents(recorded, B, T):
    from tri_sds_b200.model import QwenModel
    m = QwenModel(SHAPE, B, 96, B * T, device="cpu", fused_layers=True)
    pl = m.layers_plan(B, T)
    names = [n for n, fn, a in pl.calls]
    L = SHAPE.n_layers
    assert names == ["tsds_fused_layer"] + ["tsds_verify_attention", "tsds_fused_layer"] * L
    fused = [a for n, fn, a in pl.calls if n == "tsds_fused_layer"]
    assert _phase_names(fused[0][0]) == ["norm", "qkrope"]
    for a in fused[1:-1]:
        assert _phase_names(a[0]) == ["res", "norm", "swiglu", "res", "norm", "qkrope"]
    assert _phase_names(fused[-1][0]) == ["res", "norm", "swiglu", "res"] and fused[-1][3] is None
    # each layer's rope block writes that layer's caches
    for i, a in enumerate(fused[:-1]):
        assert a[3]["k_cache"].t.data_ptr() == m.k_cache[i].data_ptr()
        assert a[3]["T"] == T and a[2] == B * T
    for n, fn, a in pl.calls:
        assert check_call(n, a) > 0
    # the per-op plan of the same model: 8 library calls per layer, or with
    # the RMSNorms applied by the residual projections (fuse_norm) 7 for
    # layer 0 and 6 for the others
    m.fused_layers = False
    assert not m.fuse_norm   # the default
    assert len(m.layers_plan(B, T).calls) == 8 * L
    m.fuse_norm = True
    pn = m.layers_plan(B, T)
    names = [n for n, _, _ in pn.calls]
    assert len(names) == 6 * L + 1 and names.count("tsds_rms_norm") == 1
    assert names.count("tsds_linear_residual_norm") == 2 * L - 1 and not pn.final_normed
    assert m.layers_plan(B, T, final_norm=True).final_normed
    for n, fn, a in pn.calls:
        assert check_call(n, a) > 0


def test_eagle_engine_plans_with_fused_layers(recorded):
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    t = QwenModel(SHAPE, 2, 96, 2 * 26, device="cpu", fused_layers=True)
    head = EagleHead(t, 2)
    eng = EagleEngine(t, head, use_graph=False)
    n_fused = sum(1 for n, fn, a in eng.plan.calls if n == "tsds_fused_layer")
    assert n_fused >= SHAPE.n_layers + 1
    for n, fn, a in eng.plan.calls:
        if fn is not None:
            check_call(n, a)


class FakePeer:
    """tp.PeerAllReduce's interface with host tensors as slots."""

    def __init__(self, rank, size, max_elems):
        self.rank, self.size, self.max_elems = rank, size, (max_elems + 63) // 64 * 64
        self.slots = [torch.zeros(self.max_elems, dtype=torch.float32) for _ in range(2)]
        self.bufs = (ctypes.c_void_p * size)(*[0x1000 * (p + 1) for p in range(size)])

    def slot_ptr(self, slot):
        return TRef(self.slots[slot])


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 1), (8, 6)])
def test_tensor_parallel_fused_plan_with_peer_phases(recorded, tp, rank):
    from tri_sds_b200.model import QwenModel

    class _Comm:
        def __init__(self):
            self.rank, self.size = rank, tp

    B, T = 2, 26
    peer = FakePeer(rank, tp, B * T * SHAPE.hidden)
    m = QwenModel(SHAPE, B, 96, B * T, device="cpu", tp_rank=rank, tp_size=tp, comm=_Comm(), peer=peer,
                  fused_layers=True)
    assert m.fused_layers
    pl = m.layers_plan(B, T)
    names = [n for n, fn, a in pl.calls]
    assert names == ["tsds_fused_layer"] + ["tsds_verify_attention", "tsds_fused_layer"] * SHAPE.n_layers
    fused = [a for n, fn, a in pl.calls if n == "tsds_fused_layer"]
    mid = ["f32", "peer", "norm", "swiglu", "f32", "peer", "norm", "qkrope"]
    for a in fused[1:-1]:
        assert _phase_names(a[0]) == mid
        o, red_o, _, _, d, red_d = a[0][:6]
        # each partial goes to the slot its all-reduce phase reads
        assert o["out"].t is peer.slots[0] and red_o["n_out"] == 0
        assert d["out"].t is peer.slots[1] and red_d["n_out"] == 1
        assert a[4] is peer
    assert _phase_names(fused[-1][0]) == mid[:6]
    # the rank's shard sizes: local heads and FFN columns
    qk = fused[0][0][1]
    assert qk["n_out"] == (SHAPE.n_heads + 2 * SHAPE.n_kv_heads) // tp * 128
    assert fused[1][0][3]["n_out"] == SHAPE.intermediate // tp
    for n, fn, a in pl.calls:
        assert check_call(n, a) > 0


@pytest.mark.parametrize("threshold,epi", [(1 << 40, 0), (0, 1)])
def test_peer_phases_pick_one_or_two_shot(recorded, monkeypatch, threshold, epi):
    """PEER phases run two-shot (epi 1) once a rank would pull more than
    TWO_SHOT_BYTES of the others' partials one-shot."""
    import tri_sds_b200.model as model
    from tri_sds_b200.model import QwenModel
    monkeypatch.setattr(model, "TWO_SHOT_BYTES", threshold)

    class _Comm:
        rank, size = 0, 4

    peer = FakePeer(0, 4, 26 * SHAPE.hidden)
    m = QwenModel(SHAPE, 1, 96, 26, device="cpu", tp_rank=0, tp_size=4, comm=_Comm(), peer=peer, fused_layers=True)
    peers = [ph for n, fn, a in m.layers_plan(1, 26).calls if n == "tsds_fused_layer" for ph in a[0]
             if ph["kind"] == 2]
    assert peers and all(ph["epi"] == epi for ph in peers)


def test_tensor_parallel_model_keeps_the_per_op_plan():
    from tri_sds_b200.model import QwenModel

    class _Comm:
        rank, size = 0, 2

    m = QwenModel(SHAPE, 1, 96, 26, device="cpu", tp_rank=0, tp_size=2, comm=_Comm(), fused_layers=True)
    assert not m.fused_layers


def test_struct_layouts_match_the_header(tmp_path):
    from tri_sds_b200 import _lib
    src = tmp_path / "layout.c"
    src.write_text(f'''#include <stddef.h>
#include <stdio.h>
#include "{ROOT}/include/tsds.h"
int main(void) {{
  printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(tsds_fused_phase), offsetof(tsds_fused_phase, w),
         offsetof(tsds_fused_phase, res), offsetof(tsds_fused_phase, eps), sizeof(tsds_qk_rope),
         offsetof(tsds_qk_rope, T), sizeof(tsds_peer_group), offsetof(tsds_peer_group, max_elems));
  return 0;
}}
''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    P, Q, G = _lib.FusedPhase, _lib.QkRope, _lib.PeerGroup
    assert got == [ctypes.sizeof(P), P.w.offset, P.res.offset, P.eps.offset, ctypes.sizeof(Q), Q.T.offset,
                   ctypes.sizeof(G), G.max_elems.offset]


def test_entry_point_rejects_bad_descriptors():
    """Every descriptor here fails a host-side check, so nothing is launched
    (the pointers are not device memory) on a machine with or without a GPU."""
    from tri_sds_b200 import _lib
    lib = _lib.load()
    M = 26
    nb = lib.tsds_fused_layer_workspace_bytes(M)
    assert nb > 0 and lib.tsds_fused_layer_workspace_bytes(0) == 0 and lib.tsds_fused_layer_workspace_bytes(257) == 0
    ws = ctypes.c_void_p(0x100000)

    def ph(**kw):
        d = dict(kind=0, epi=0, x=0x1000, ldx=256, K=256, w=0x2000, n_out=256, res_ld=0, res=None, out=0x3000,
                 ldo=256, eps=0.0)
        d.update(kw)
        return _lib.FusedPhase(**d)

    def run(phases, m=M, qr=None, wsb=nb):
        arr = (_lib.FusedPhase * max(1, len(phases)))(*phases)
        return lib.tsds_fused_layer(arr, len(phases), m, qr, None, ws, wsb, None)

    assert run([]) == 1                                   # no phase
    assert run([ph()] * 9) == 1                           # more than 8
    assert run([ph()], m=0) == 1 and run([ph()], m=257) == 1
    assert run([ph()], wsb=nb - 1) == 4                   # workspace too small
    assert run([ph(epi=3)]) == 1                          # the LM-head epilogue is not a fused phase
    assert run([ph(epi=1)]) == 1                          # residual without res
    assert run([ph(epi=5)]) == 1                          # QKROPE without its parameters
    qr = _lib.QkRope(cos=1, sin=1, positions=1, starts=1, q_out=1, k_cache=1, v_cache=1, T=26, Hq=4, Hkv=2, S=64,
                     rope_len=64)
    assert run([ph(epi=5, n_out=1152)], qr=ctypes.pointer(qr)) == 1    # n_out != (Hq + 2 Hkv) * 128
    assert run([ph(kind=1, K=250)]) == 1                  # norm row not a multiple of 8
    assert run([ph(kind=7)]) == 1
    assert run([ph(x=0x1008)]) == 2                       # x not 16-byte aligned
    assert run([ph(kind=2, K=256, n_out=0)]) == 1         # an all-reduce phase without a peer group
    bufs = (ctypes.c_void_p * 2)(0x10000, 0x20000)

    def group(**kw):
        d = dict(bufs=ctypes.cast(bufs, ctypes.c_void_p), rank=0, tp=2, max_elems=M * 256)
        d.update(kw)
        return ctypes.pointer(_lib.PeerGroup(**d))

    arr = (_lib.FusedPhase * 1)(ph(kind=2, K=256, n_out=0))
    for bad in (group(tp=9), group(rank=2), group(max_elems=M * 256 - 1)):
        assert lib.tsds_fused_layer(arr, 1, M, None, bad, ws, nb, None) == 1
    arr = (_lib.FusedPhase * 1)(ph(kind=2, K=256, n_out=2))  # slot not 0 / 1
    assert lib.tsds_fused_layer(arr, 1, M, None, group(), ws, nb, None) == 1

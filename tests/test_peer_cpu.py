"""The peer-memory all-reduce on CPU (nothing runs on a device).

* ``tp.PeerAllReduce`` exchanges the ranks' IPC handles over the process
  group and builds the pointer table the kernel takes (2 and 4 gloo ranks,
  with the library's allocation / IPC entry points replaced by stand-ins);
* a TP plan with peer all-reduces writes each row-parallel partial into the
  rank's peer slot, alternates slots 0 / 1, calls no NCCL all-reduce, and
  hands the library buffers that reach their extents;
* the entry points' host-side argument checks and buffer layout."""
import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from abi_extents import TRef, check_call
from tri_sds_b200.shapes import QwenShape

SHAPE = QwenShape(hidden=256, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=1024, n_layers=3, vocab=1024)
MAPPED = 0x7000_0000   # where a stand-in import "maps" a peer's buffer


def _fake_lib(rank, log):
    """Stand-ins for the allocation / IPC entry points (host-only)."""
    def call(name, *args):
        log.append(name)
        if name == "tsds_peer_alloc":
            args[1]._obj.value = 0x1000_0000 * (rank + 1)
        elif name == "tsds_peer_export":
            ctypes.memmove(args[1], (ctypes.c_uint64 * 1)(args[0].value), 8)
        elif name == "tsds_peer_import":
            own = ctypes.c_uint64.from_buffer_copy(bytes(args[0])[:8]).value
            args[1]._obj.value = own + MAPPED
        elif name not in ("tsds_peer_close", "tsds_peer_free"):
            raise AssertionError(name)
    return call


def _exchange_worker(rank, tp, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=tp)
    try:
        from tri_sds_b200 import _lib, tp as tpm
        log = []
        _lib.call = _fake_lib(rank, log)
        peer = tpm.PeerAllReduce(rank, tp, 1000)
        table = [peer.bufs[p] for p in range(tp)]
        slot1 = peer.slot_ptr(1).value - peer._own.value
        peer.close()
        q.put((rank, table, slot1, peer.max_elems, log))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None, None, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tp", [2, 4])
def test_handles_exchanged_and_pointer_table_built(tp):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(daemon=True, target=_exchange_worker, args=(r, tp, port, q)) for r in range(tp)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=120) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    from tri_sds_b200 import _lib
    for rank, table, slot1, max_elems, log in res:
        assert isinstance(table, list), table
        own = 0x1000_0000 * (rank + 1)
        assert table == [own if p == rank else 0x1000_0000 * (p + 1) + MAPPED for p in range(tp)]
        assert max_elems == 1024 and slot1 == _lib.query("tsds_peer_slot_offset", max_elems, 1)
        # one allocation, one export, tp-1 imports, and on close tp-1 unmaps and one free
        assert log == (["tsds_peer_alloc", "tsds_peer_export"] + ["tsds_peer_import"] * (tp - 1)
                       + ["tsds_peer_close"] * (tp - 1) + ["tsds_peer_free"])


class _Comm:
    def __init__(self, rank, size):
        self.rank, self.size = rank, size

    def all_reduce(self, t):
        raise AssertionError("not called while building a plan")

    def all_gather(self, out, inp):
        raise AssertionError("not called while building a plan")


class FakePeer:
    """The interface QwenModel uses: rank, size, max_elems, bufs, slot_ptr;
    the slots are host tensors so the plan's pointers can be checked."""

    def __init__(self, rank, size, max_elems):
        self.rank, self.size, self.max_elems = rank, size, (max_elems + 63) // 64 * 64
        self.slots = [torch.zeros(self.max_elems, dtype=torch.float32) for _ in range(2)]
        self.bufs = (ctypes.c_void_p * size)(*[0x1000 * (p + 1) for p in range(size)])

    def slot_ptr(self, slot):
        return TRef(self.slots[slot])


@pytest.fixture()
def tensor_refs(monkeypatch):
    import tri_sds_b200.eagle as eagle
    import tri_sds_b200.engine as engine
    import tri_sds_b200.model as model
    ref = lambda t: None if t is None else TRef(t)  # noqa: E731
    for mod in (model, eagle, engine):
        monkeypatch.setattr(mod, "_p", ref)
    yield


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 1), (8, 5)])
def test_plan_uses_the_peer_slots(tensor_refs, tp, rank):
    """(tp = 1: a one-rank group, the peer paths on one GPU.)"""
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    B = 2
    peer = FakePeer(rank, tp, B * 26 * SHAPE.hidden)
    t = QwenModel(SHAPE, B, 96, B * 26, device="cpu", tp_rank=rank, tp_size=tp, comm=_Comm(rank, tp), peer=peer)
    eng = EagleEngine(t, EagleHead(t, B), use_graph=False)
    for plan in (eng.plan, eng.verify_only_plan()):
        names = [n for n, fn, _ in plan.calls]
        assert "all_reduce" not in names and "tsds_residual_add_f32" not in names
        ars = [(i, a) for i, (n, fn, a) in enumerate(plan.calls) if n == "tsds_peer_allreduce_residual"]
        assert len(ars) == 2 * SHAPE.n_layers
        for j, (i, a) in enumerate(ars):
            slot = a[4]
            assert slot == j % 2 and (a[2], a[3]) == (rank, tp) and a[1] is peer.bufs
            assert a[7] == peer.max_elems
            # the projection right before writes its fp32 partial into this slot
            n, fn, g = plan.calls[i - 1]
            assert n == "tsds_linear_f32" and g[3].t is peer.slots[slot]
            assert g[5] == a[5] and g[6] == a[6] == SHAPE.hidden
        for n, fn, a in plan.calls:
            if fn is not None:
                check_call(n, a)


class FakeExchangePeer(FakePeer):
    """FakePeer with an exchange region for the vocab-parallel LM head."""

    def __init__(self, rank, size, max_elems, exchange_bytes):
        super().__init__(rank, size, max_elems)
        self.exchange_bytes = exchange_bytes
        self.exchange = torch.zeros(exchange_bytes, dtype=torch.uint8)

    def exchange_at(self, offset):
        return TRef(self.exchange[offset:])


@pytest.mark.parametrize("tp,rank", [(1, 0), (2, 0), (8, 7)])
def test_lm_head_gathers_over_peer_memory(tensor_refs, tp, rank):
    """With an exchange region, a tensor-parallel EAGLE cycle has no NCCL
    step at all: the row-parallel all-reduces run on peer memory and every
    vocab-parallel LM head (the target's and the head passes') writes its
    candidates / logits into the exchange region that tsds_peer_lm_gather
    reads."""
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.tp import lm_exchange_layout
    B = 2
    rows = B * 26
    xb = lm_exchange_layout(rows, SHAPE.vocab // tp)[2]
    peer = FakeExchangePeer(rank, tp, rows * SHAPE.hidden, xb)
    t = QwenModel(SHAPE, B, 96, rows, device="cpu", tp_rank=rank, tp_size=tp, comm=_Comm(rank, tp), peer=peer)
    eng = EagleEngine(t, EagleHead(t, B), use_graph=False)
    assert eng.head.model.lm_peer is peer
    calls = eng.plan.calls
    assert not any(fn is None for _, fn, _ in calls)          # no NCCL (Python collective) steps
    names = [n for n, _, _ in calls]
    assert "tsds_argmax_merge" not in names and "tsds_gather_shards" not in names
    gathers = [i for i, n in enumerate(names) if n == "tsds_peer_lm_gather"]
    assert len(gathers) == 6                                   # the target's verify + five head passes
    for i in gathers:
        n, fn, lm = calls[i - 1]
        assert n == "tsds_lm_head_argmax" and lm[4].t.data_ptr() == peer.exchange.data_ptr()
    for n, fn, a in calls:
        check_call(n, a)


def test_lm_gather_host_checks():
    from tri_sds_b200 import _lib
    lib = _lib.load()
    bufs = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    out, st = ctypes.c_void_p(0x30000), ctypes.c_void_p(0x40000)

    def run(tp=2, rank=0, xb=4096, rows=4, vl=64, val_off=256, log_off=512, logits=None):
        return lib.tsds_peer_lm_gather(bufs, rank, tp, 1024, xb, rows, vl, val_off, log_off, out, 1, logits, st, None)

    assert run(tp=9) == 1 and run(rank=2) == 1 and run(rows=0) == 1
    assert run(val_off=16) == 2                               # candidates overlap the values
    assert run(xb=16) == 1                                    # the values do not fit the region
    assert run(logits=ctypes.c_void_p(0x50000), log_off=256) == 1          # logits overlap the values
    assert run(logits=ctypes.c_void_p(0x50000), xb=600) == 1               # logits do not fit


def test_peer_needs_matching_rank_and_room():
    from tri_sds_b200.model import QwenModel
    with pytest.raises(AssertionError):
        QwenModel(SHAPE, 1, 96, 26, device="cpu", tp_rank=0, tp_size=2, comm=_Comm(0, 2),
                  peer=FakePeer(1, 2, 26 * SHAPE.hidden))
    with pytest.raises(AssertionError):
        QwenModel(SHAPE, 1, 96, 26, device="cpu", tp_rank=0, tp_size=2, comm=_Comm(0, 2),
                  peer=FakePeer(0, 2, 5 * SHAPE.hidden))


def test_entry_point_checks_and_layout():
    """Argument checks return before any CUDA call; the layout is the
    documented one (32 KB header, two 256-byte-rounded fp32 slots, then a
    256-byte-rounded bf16 region published by the two-shot all-reduce, then
    the LM head's exchange region)."""
    from tri_sds_b200 import _lib
    lib = _lib.load()
    assert lib.tsds_peer_handle_bytes() == 64
    assert lib.tsds_peer_buffer_bytes(0, 0) == 0
    assert lib.tsds_peer_buffer_bytes(1000, 0) == 32768 + 2 * 4096 + 2048
    assert lib.tsds_peer_buffer_bytes(1000, 1000) == 32768 + 2 * 4096 + 2048 + 1024   # exchange, 256-aligned
    assert lib.tsds_peer_exchange_offset(1000) == 32768 + 2 * 4096 + 2048
    assert lib.tsds_peer_slot_offset(1000, 0) == 32768 and lib.tsds_peer_slot_offset(1000, 1) == 32768 + 4096
    bufs = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    x = ctypes.c_void_p(0x30000)
    st = ctypes.c_void_p(0x40000)
    bad = [
        (x, bufs, 0, 9, 0, 1, 8, 64),    # tp > 8
        (x, bufs, 2, 2, 0, 1, 8, 64),    # rank >= tp
        (x, bufs, 0, 2, 2, 1, 8, 64),    # slot not 0 / 1
        (x, bufs, 0, 2, 0, 1, 6, 64),    # N % 4
        (x, bufs, 0, 2, 0, 9, 8, 64),    # M * N > max_elems
        (None, bufs, 0, 2, 0, 1, 8, 64),
    ]
    for args in bad:
        assert lib.tsds_peer_allreduce_residual(*args, st, None) == 1, args
    assert lib.tsds_peer_allreduce_residual(ctypes.c_void_p(0x30002), bufs, 0, 2, 0, 1, 8, 64, st, None) == 2
    unaligned = (ctypes.c_void_p * 2)(0x10000, 0x20008)
    assert lib.tsds_peer_allreduce_residual(x, unaligned, 0, 2, 0, 1, 8, 64, st, None) == 2
    assert lib.tsds_peer_alloc(16, ctypes.byref(ctypes.c_void_p())) == 1     # smaller than the header
    assert lib.tsds_status_string(9) == b"CUDA runtime call (allocation / IPC) failed"


@pytest.mark.parametrize("tp,rank", [(2, 1), (8, 3)])
def test_sharded_chain_draft_shares_the_slot_alternation(tensor_refs, tp, rank):
    """A chain draft sharded over the target's ranks with the target's peer
    group: every peer all-reduce of the cycle - the draft's K forwards, then
    the target's verify - takes slot 0, 1, 0, 1, ... in order, so no rank
    writes a slot another rank may still read; no NCCL step remains, and
    every call fits its buffers."""
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.tp import lm_exchange_layout
    B, K = 2, 4
    rows = B * (K + 1)
    xb = lm_exchange_layout(rows, SHAPE.vocab // tp)[2]
    peer = FakeExchangePeer(rank, tp, rows * SHAPE.hidden, xb)
    comm = _Comm(rank, tp)
    t = QwenModel(SHAPE, B, 96, rows, device="cpu", tp_rank=rank, tp_size=tp, comm=comm, peer=peer)
    d = QwenModel(SHAPE, B, 96, B * 2, device="cpu", tp_rank=rank, tp_size=tp, comm=comm, peer=peer)
    eng = SpecEngine(t, d, K, use_graph=False)
    calls = eng.plan.calls
    assert not any(fn is None for _, fn, _ in calls)
    slots = [a[4] for n, _, a in calls if n == "tsds_peer_allreduce_residual"]
    assert len(slots) == 2 * SHAPE.n_layers * (K + 1)
    assert slots == [j % 2 for j in range(len(slots))]
    assert sum(1 for n, _, _ in calls if n == "tsds_peer_lm_gather") == K + 1
    for n, fn, a in calls:
        check_call(n, a)

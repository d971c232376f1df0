"""Tensor parallelism over the GPUs of one node (one process per GPU).

Megatron-style split of a Qwen3 decoder layer across ``tp`` ranks:

* q/k/v projection: column-parallel by heads - rank r holds q heads
  ``[r*Hq/tp, (r+1)*Hq/tp)`` and kv heads ``[r*Hkv/tp, ...)`` (at tp = 8 one
  kv head per rank), so attention runs on local heads with no exchange;
* O projection: row-parallel - rank r holds the input columns of its q
  heads and produces an fp32 partial of the full output;
* gate/up: column-parallel (rows ``[r*I/tp, (r+1)*I/tp)`` of each);
* down: row-parallel (the matching input columns), fp32 partial;
* LM head: vocab-parallel (rows ``[r*V/tp, (r+1)*V/tp)``);
* embedding and norm gains: replicated.

Exchange per layer: two all-reduces (sum) of the fp32 partials of O and
down, followed by the residual add with the reference's rounding; at the
LM head, an all-gather of each row's (value, index) argmax candidate (and,
when full logits are needed, of the logits shards).  The all-gathers are
NCCL's through ``torch.distributed``; the all-reduces are NCCL's too, or
(``PeerAllReduce``) this library's one-shot kernel over NVLink peer memory,
fused with the residual add.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def local_dims(shape, tp: int) -> dict:
    assert shape.n_heads % tp == 0 and shape.n_kv_heads % tp == 0 and shape.intermediate % tp == 0
    return {"n_heads": shape.n_heads // tp, "n_kv_heads": shape.n_kv_heads // tp,
            "intermediate": shape.intermediate // tp}


def shard_layer(L: dict, shape, rank: int, tp: int) -> dict:
    """HF-layout layer weights -> rank r's shard (same keys)."""
    if tp == 1:
        return L
    D, I = shape.head_dim, shape.intermediate
    qh, kh, il = shape.n_heads // tp, shape.n_kv_heads // tp, I // tp
    q = slice(rank * qh * D, (rank + 1) * qh * D)
    kv = slice(rank * kh * D, (rank + 1) * kh * D)
    ff = slice(rank * il, (rank + 1) * il)
    return {
        "q": L["q"][q], "k": L["k"][kv], "v": L["v"][kv],
        "o": L["o"][:, q].contiguous(),
        "gate": L["gate"][ff], "up": L["up"][ff],
        "down": L["down"][:, ff].contiguous(),
        "ln1": L["ln1"], "ln2": L["ln2"], "q_norm": L["q_norm"], "k_norm": L["k_norm"],
    }


def vocab_shard(t: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    v = t.shape[0] // tp
    return t[rank * v:(rank + 1) * v].contiguous()


class Comm:
    """The process group's collectives, on the current stream."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    def all_reduce(self, t: torch.Tensor):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor):
        dist.all_gather_into_tensor(out, inp, group=self.group)


class LocalComm:
    """Single-rank stand-in (tp = 1): collectives are no-ops."""
    rank, size = 0, 1

    def all_reduce(self, t):
        return None

    def all_gather(self, out, inp):
        out.copy_(inp)


def lm_exchange_layout(rows: int, vocab_shard: int) -> tuple[int, int, int]:
    """(values offset, logits offset, bytes) of a vocab-parallel LM head's
    exchange region for up to `rows` rows (tsds_peer_lm_gather): local
    indices int64 at 0, values fp32, then the logits shard [rows][vocab_shard]
    bf16, each 256-byte aligned."""
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    val_off = up(8 * rows)
    log_off = val_off + up(4 * rows)
    return val_off, log_off, log_off + up(2 * rows * vocab_shard)


class _CudaView:
    """__cuda_array_interface__ of n fp32 at a device address (torch.as_tensor
    wraps it without a copy or ownership)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


_GROUPS: dict = {}


def register_peer_group(peer: "PeerAllReduce") -> int:
    """Id under which torch.ops.tsds.allreduce_oneshot finds `peer`.  A group
    used by the op should not also serve a model's launch plans (the slot
    alternation is per user)."""
    gid = len(_GROUPS)
    _GROUPS[gid] = peer
    return gid


def peer_group(gid: int) -> "PeerAllReduce":
    return _GROUPS[gid]


class PeerAllReduce:
    """Peer buffers of the ranks of one node, for tsds_peer_allreduce_residual.

    Allocates this rank's buffer (``max_elems`` fp32 per slot), exchanges
    CUDA IPC handles over ``group`` (any backend: the handles are bytes) and
    maps every other rank's buffer.  ``bufs`` is the host pointer table the
    kernel takes; ``slot_ptr(s)`` is where this rank's row-parallel GEMM
    writes its partial for a call on slot s.  Every rank must construct it at
    the same point (the exchange is a collective)."""

    def __init__(self, rank: int, size: int, max_elems: int, group=None, exchange_bytes: int = 0):
        assert 1 <= size <= 8 and 0 <= rank < size
        self.rank, self.size = rank, size
        self.broken = False   # set when a device wait on the group gave up: the group is then unusable
        self.max_elems = (max_elems + 63) // 64 * 64
        self.exchange_bytes = exchange_bytes
        self._own = ctypes.c_void_p()
        self._imported: list[ctypes.c_void_p] = []
        _lib.call("tsds_peer_alloc", _lib.query("tsds_peer_buffer_bytes", self.max_elems, exchange_bytes),
                  ctypes.byref(self._own))
        try:
            hb = _lib.query("tsds_peer_handle_bytes")
            mine = (ctypes.c_uint8 * hb)()
            _lib.call("tsds_peer_export", self._own, mine)
            handles = [None] * size
            if size == 1:   # one rank: nothing to exchange (no process group needed)
                handles[0] = bytes(mine)
            else:
                dist.all_gather_object(handles, bytes(mine), group=group)
            ptrs = []
            for p, h in enumerate(handles):
                if p == rank:
                    ptrs.append(self._own.value)
                    continue
                mapped = ctypes.c_void_p()
                _lib.call("tsds_peer_import", (ctypes.c_uint8 * hb).from_buffer_copy(h), ctypes.byref(mapped))
                self._imported.append(mapped)
                ptrs.append(mapped.value)
            self.bufs = (ctypes.c_void_p * size)(*ptrs)
        except BaseException:
            self.close()
            raise

    def slot_ptr(self, slot: int) -> ctypes.c_void_p:
        return ctypes.c_void_p(self._own.value + _lib.query("tsds_peer_slot_offset", self.max_elems, slot))

    def exchange_at(self, offset: int) -> ctypes.c_void_p:
        """Address `offset` bytes into this rank's exchange region."""
        assert 0 <= offset < max(self.exchange_bytes, 1)
        return ctypes.c_void_p(self._own.value + _lib.query("tsds_peer_exchange_offset", self.max_elems) + offset)

    def slot_tensor(self, slot: int, n: int) -> torch.Tensor:
        """fp32 tensor view of the first n elements of this rank's slot (no copy)."""
        assert 0 < n <= self.max_elems
        return torch.as_tensor(_CudaView(self.slot_ptr(slot).value, n), device=torch.device("cuda"))

    def next_slot(self) -> int:
        """Slot for the next op-level all-reduce on this group (alternates;
        every rank makes the same sequence of calls)."""
        self._op_calls = getattr(self, "_op_calls", 0) + 1
        return (self._op_calls - 1) % 2

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every kernel
        that uses them has finished on every rank)."""
        for m in self._imported:
            _lib.call("tsds_peer_close", m)
        self._imported = []
        if self._own.value:
            _lib.call("tsds_peer_free", self._own)
            self._own = ctypes.c_void_p()

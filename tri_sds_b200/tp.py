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
when full logits are needed, of the logits shards).  Collectives are NCCL's
through ``torch.distributed``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


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

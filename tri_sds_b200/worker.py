"""TriSDSWorker: the spec worker the plugin installs (tri_sds/worker.py:9-68).

Same class name, base class, methods and ``SDS_ENABLED`` gate as the
reference (worker.py:19-21, 32-45).  With ``SDS_ENABLED=1`` the three
methods run this package's device path instead of SGLang's:

* ``forward_batch_generation(batch)``: one full speculative cycle (draft ->
  verify -> accept -> commit) for the batch's sequences; returns the
  emitted tokens ``[B, K+1]`` (-1 padded) and accept lengths ``[B]``.
  (The reference raises NotImplementedError here, worker.py:49-51.)
* ``draft(batch)``: the K draft tokens ``[B, K]`` of the next cycle
  (the reference returns the GPT-2 draft's logits, worker.py:53-64).
* ``verify(batch)``: the target's verify pass + acceptance over the drafts
  of the last ``draft`` call (the reference raises, worker.py:66-68).

The engine is attached with ``attach_engine`` (or built lazily by the
subclass hook ``_init_engine``); it owns the weights and KV caches.

The worker follows the batch it is given.  It remembers the request ids
(``batch.reqs[i].rid`` when the batch carries SGLang requests), else the
prompt it prepared the engine from.  A batch with other requests, or without
requests a prompt other than the prepared one, prefills the engine again
from that batch; one token per sequence (``input_ids`` [B, 1]) continues the
prepared batch.  A batch whose size differs from the engine's raises
``ValueError`` before anything runs.
"""
from __future__ import annotations

import os

import torch

from .sglang_compat import ScheduleBatch, StandaloneWorker


def prompt_tensor(batch: ScheduleBatch):
    """The batch's prompts as a [B, P] id tensor and their lengths: a [B, P]
    tensor (with ``seq_lens`` when its rows are padded) or one [P] prompt as
    they are; a list of per-sequence prompts of different lengths is padded
    with zeros behind each prompt (lengths then give the real tokens, None
    when every row is full)."""
    ids = batch.input_ids
    lengths = getattr(batch, "seq_lens", None)
    if isinstance(ids, (list, tuple)) and ids and not isinstance(ids[0], int):
        seqs = [torch.as_tensor(x, dtype=torch.int64).reshape(-1) for x in ids]
        n = [int(x.numel()) for x in seqs]
        if min(n) < 1:
            raise ValueError("every prompt needs at least one token")
        P = max(n)
        out = torch.zeros(len(seqs), P, dtype=torch.int64)
        for b, x in enumerate(seqs):
            out[b, :n[b]] = x
        if lengths is None and min(n) < P:
            lengths = torch.tensor(n, dtype=torch.int32)
        return out, lengths
    ids = torch.as_tensor(ids)
    if ids.dim() == 1:
        ids = ids.unsqueeze(0)
    if lengths is not None:
        lengths = torch.as_tensor(lengths).to(torch.int32).reshape(-1)
    return ids, lengths


def request_ids(batch: ScheduleBatch):
    """The batch's request identities (SGLang's ``batch.reqs[i].rid``) as a
    tuple, or None when the batch carries no requests."""
    reqs = getattr(batch, "reqs", None)
    if not reqs:
        return None
    return tuple(getattr(r, "rid", id(r)) for r in reqs)


class TriSDSWorker(StandaloneWorker):
    sds_enabled: bool = False
    engine = None

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.sds_enabled = os.environ.get("SDS_ENABLED", "0") == "1"
        self._prefilled = False
        self._rids = None
        self._prompt = None

    # -- engine ----------------------------------------------------------------
    def attach_engine(self, engine):
        self.engine = engine
        self._prefilled = False
        self._rids = None
        self._prompt = None

    def _init_engine(self):
        raise RuntimeError("TriSDSWorker needs an engine: call attach_engine(SpecEngine(...))")

    def _engine_batch(self) -> int:
        return int(self.engine.tokens.shape[0])

    def _is_new_batch(self, batch: ScheduleBatch, ids: torch.Tensor, lengths) -> bool:
        """True when ``batch`` is not the continuation of the prepared one:
        other request ids, or (without ids) a prompt other than the prepared
        prompt.  One token per sequence ([B, 1]) is the current token of a
        continuing batch."""
        rids = request_ids(batch)
        if rids is not None or self._rids is not None:
            return rids != self._rids
        if ids.shape[1] == 1 and not isinstance(batch.input_ids, (list, tuple)):
            return False
        key = (ids.detach().cpu(), None if lengths is None else lengths.detach().cpu())
        old = self._prompt
        return not (old is not None and old[0].shape == key[0].shape and torch.equal(old[0], key[0])
                    and (old[1] is None) == (key[1] is None) and (old[1] is None or torch.equal(old[1], key[1])))

    def _ensure(self, batch: ScheduleBatch):
        """Prefill the engine from ``batch`` on the first call and whenever
        the batch is a new one; returns True when it did."""
        if self.engine is None:
            self._init_engine()
        ids, lengths = prompt_tensor(batch)
        if ids.shape[0] != self._engine_batch():
            raise ValueError(f"batch of {ids.shape[0]} sequences, but the engine serves "
                             f"{self._engine_batch()}: attach an engine built for this batch size")
        if self._prefilled and not self._is_new_batch(batch, ids, lengths):
            return False
        self.engine.prepare(ids, lengths)
        self._prefilled = True
        self._rids = request_ids(batch)
        self._prompt = (ids.detach().cpu(), None if lengths is None else lengths.detach().cpu())
        return True

    # -- dispatch (worker.py:32-45) -------------------------------------------
    def forward_batch_generation(self, batch: ScheduleBatch):
        if not self.sds_enabled:
            return super().forward_batch_generation(batch)
        return self._forward_batch_generation_sds(batch)

    def draft(self, batch: ScheduleBatch):
        if not self.sds_enabled:
            return super().draft(batch)
        return self._draft_sds(batch)

    def verify(self, batch: ScheduleBatch):
        if not self.sds_enabled:
            return super().verify(batch)
        return self._verify_sds(batch)

    # -- SDS implementations ---------------------------------------------------
    def _forward_batch_generation_sds(self, batch: ScheduleBatch):
        """One speculative cycle: (tokens [B, K+1] padded -1, accept_len [B]).

        The first call prefills from ``batch.input_ids`` ([B, P] prompt).
        Later calls may carry the current token of each sequence
        (``input_ids`` of shape [B, 1], e.g. the previous cycle's bonus
        token, on the host); the results come back on the host then."""
        first = self._ensure(batch)
        ids = batch.input_ids
        if not first and isinstance(ids, torch.Tensor) and not ids.is_cuda and ids.dim() == 2 and ids.shape[1] == 1:
            B, W = self.engine.tokens.shape
            if getattr(self, "_host_bufs", None) is None or self._host_bufs[1].shape != (B, W):
                pin = torch.cuda.is_available()
                self._host_bufs = (torch.empty(B, dtype=torch.int64, pin_memory=pin),
                                   torch.empty(B, W, dtype=torch.int64, pin_memory=pin),
                                   torch.empty(B, dtype=torch.int32, pin_memory=pin))
            cur_h, tok_h, acc_h = self._host_bufs
            cur_h.copy_(ids[:, 0])
            return self.engine.step_host(cur_h, tok_h, acc_h)
        tokens, n = self.engine.step()
        return tokens.clone(), n.clone()

    def _draft_sds(self, batch: ScheduleBatch):
        self._ensure(batch)
        return self.engine.run_draft().clone()

    def _verify_sds(self, batch: ScheduleBatch):
        self._ensure(batch)
        tokens, n = self.engine.run_verify()
        return tokens.clone(), n.clone()

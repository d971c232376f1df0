"""TriSDSWorker: the spec worker the plugin installs (tri_sds/worker.py:19-78).

Same class name, base class, methods and ``SDS_ENABLED`` gate as the
reference.  With ``SDS_ENABLED=1`` the three methods run this package's
device path instead of SGLang's:

* ``forward_batch_generation(batch)``: one full speculative cycle (draft ->
  verify -> accept -> commit) for the batch's sequences; returns the
  emitted tokens ``[B, K+1]`` (-1 padded) and accept lengths ``[B]``.
  (The reference raises NotImplementedError here, worker.py:59-61.)
* ``draft(batch)``: the K draft tokens ``[B, K]`` of the next cycle
  (the reference returns the GPT-2 draft's logits, worker.py:63-74).
* ``verify(batch)``: the target's verify pass + acceptance over the drafts
  of the last ``draft`` call (the reference raises, worker.py:76-78).

The engine is attached with ``attach_engine`` (or built lazily by the
subclass hook ``_init_engine``); it owns the weights and KV caches.
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


class TriSDSWorker(StandaloneWorker):
    sds_enabled: bool = False
    engine = None

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.sds_enabled = os.environ.get("SDS_ENABLED", "0") == "1"
        self._prefilled = False

    # -- engine ----------------------------------------------------------------
    def attach_engine(self, engine):
        self.engine = engine
        self._prefilled = False

    def _init_engine(self):
        raise RuntimeError("TriSDSWorker needs an engine: call attach_engine(SpecEngine(...))")

    def _ensure(self, batch: ScheduleBatch):
        if self.engine is None:
            self._init_engine()
        if not self._prefilled:
            ids, lengths = prompt_tensor(batch)
            self.engine.prepare(ids, lengths)
            self._prefilled = True

    # -- dispatch (worker.py:42-55) -------------------------------------------
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
        first = not self._prefilled
        self._ensure(batch)
        ids = batch.input_ids
        if not first and isinstance(ids, torch.Tensor) and not ids.is_cuda and ids.dim() == 2 and ids.shape[1] == 1:
            B, W = self.engine.tokens.shape
            if getattr(self, "_host_bufs", None) is None:
                self._host_bufs = (torch.empty(B, dtype=torch.int64).pin_memory(),
                                   torch.empty(B, W, dtype=torch.int64).pin_memory(),
                                   torch.empty(B, dtype=torch.int32).pin_memory())
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

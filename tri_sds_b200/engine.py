"""Chain speculative decoding on the device: draft -> verify -> accept -> commit.

One cycle (for B sequences, K draft tokens) is a single launch plan with
no host synchronisation, captured once in a CUDA graph and replayed:

1. ``tsds_gather_ids``: draft input ``[last, cur]``;
2. draft step 1 (T=2 at rows L-1, L) and steps 2..K (T=1 at L+i-1), each a
   full draft forward whose LM-head argmax writes ``draft_tok[:, i-1]``;
3. ``tsds_gather_ids``: verify input ``[cur, d_1..d_K]``;
4. target verify forward (T=K+1 at rows L..L+K), argmax of every row;
5. ``tsds_accept_greedy``: accept lengths, emitted tokens, and the commit
   ``target.lengths += n+1``, ``last``/``cur`` for the next cycle.

``L`` is the target's committed length; the draft's cache is addressed
relative to it (its valid prefix is always L-1 rows), so the draft needs
no length bookkeeping of its own.  Semantics are those of the oracle's
chain cycle: greedy output equals greedy autoregressive output.
"""
from __future__ import annotations

import torch

from .model import Plan, QwenModel, StatusWatch, _p


class SpecEngine:
    def __init__(self, target: QwenModel, draft: QwenModel, k: int, use_graph: bool = True):
        assert target.batch == draft.batch
        assert target.max_rows >= target.batch * (k + 1) and draft.max_rows >= draft.batch * 2
        self.target, self.draft, self.k = target, draft, k
        B = target.batch
        dev = target.device
        i64 = dict(dtype=torch.int64, device=dev)
        self.draft_tok = torch.zeros(B, max(k, 1), **i64)
        self.verify_ids = torch.zeros(B, k + 1, **i64)
        self.draft_ids2 = torch.zeros(B, 2, **i64)
        self.target_argmax = torch.zeros(B, k + 1, **i64)
        self.accept_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(B, k + 1, **i64)
        self.last = torch.zeros(B, **i64)
        self.cur = torch.zeros(B, **i64)
        self.use_graph = use_graph
        self.graph = None
        self.plan_launches = None
        self.draft_plan = self._draft_plan()
        self.verify_plan = self._verify_plan()
        self.plan = Plan()
        self.plan.extend(self.draft_plan)
        self.plan.extend(self.verify_plan)

    def _draft_plan(self) -> Plan:
        t, d, K = self.target, self.draft, self.k
        B = t.batch
        pl = Plan()
        pl.add("tsds_gather_ids", _p(self.cur), _p(self.last), _p(self.draft_tok), None, _p(self.draft_ids2), B, K)
        tok = self.draft_tok
        pl.extend(d.forward_plan(self.draft_ids2, 1, B, 2, t.lengths, -1, tok, K, last_only=True))
        for i in range(2, K + 1):
            pl.extend(d.forward_plan(tok[:, i - 2:], K, B, 1, t.lengths, i - 1, tok[:, i - 1:], K, last_only=True))
        return pl

    def _verify_plan(self) -> Plan:
        t, K = self.target, self.k
        B = t.batch
        pl = Plan()
        pl.add("tsds_gather_ids", _p(self.cur), _p(self.last), _p(self.draft_tok), _p(self.verify_ids), None, B, K)
        pl.extend(t.forward_plan(self.verify_ids, 1, B, K + 1, t.lengths, 0, self.target_argmax, 1))
        pl.add("tsds_accept_greedy", _p(self.draft_tok), _p(self.target_argmax), _p(self.accept_len),
               _p(self.tokens), _p(t.lengths), _p(self.last), _p(self.cur), B, K)
        return pl

    def verify_only_plan(self) -> Plan:
        """The target's verify forward alone (for timing the verify step)."""
        t = self.target
        return t.forward_plan(self.verify_ids, 1, t.batch, self.k + 1, t.lengths, 0, self.target_argmax, 1)

    def kernel_launches_per_cycle(self) -> int:
        return self.plan.kernel_count()

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        """Fill both caches from a [B, P] prompt (ragged: ``lengths[b]`` real
        tokens per row); returns the first token [B].  The draft caches every
        prompt token but the last, which its first step consumes."""
        B, P = prompt.shape
        dev = self.target.device
        prompt = prompt.to(dev)
        hidden = self.target.prefill(prompt, lengths)
        first = self.target.logits_of(self.target.last_rows(hidden, lengths)).argmax(-1)
        if lengths is None:
            if P > 1:
                self.draft.prefill(prompt[:, :P - 1])
            self.last.copy_(prompt[:, -1])
        else:
            n = torch.as_tensor(lengths).to(device=dev, dtype=torch.int64)
            if P > 1:
                self.draft.prefill(prompt[:, :P - 1], torch.clamp(n - 1, min=1))
                self.draft.lengths.copy_((n - 1).to(torch.int32))   # 0 for a one-token prompt
            self.last.copy_(prompt[torch.arange(B, device=dev), n - 1])
        self.cur.copy_(first)
        return first

    def _capture(self):
        from . import _lib
        c0 = _lib.query("tsds_launch_count")
        self.plan.run()  # eager warm-up (module loading, attributes) before capture
        self.plan_launches = _lib.query("tsds_launch_count") - c0
        torch.cuda.synchronize()
        # restore nothing: capture only records; callers re-prefill after
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.plan.run()
        self.graph = g

    def run_draft(self) -> torch.Tensor:
        """Draft half of a cycle (eager): the K draft tokens [B, K]."""
        self.draft_plan.run()
        return self.draft_tok

    def run_verify(self):
        """Verify + accept + commit over the current drafts (eager)."""
        self.verify_plan.run()
        return self.tokens, self.accept_len

    def step(self):
        """One cycle; returns device tensors (tokens [B,K+1] padded -1, accept_len [B])."""
        self.target.ensure_usable()
        if self.use_graph:
            self.graph.replay()
        else:
            self.plan.run()
        return self.tokens, self.accept_len

    def step_host(self, cur_host: torch.Tensor, tokens_host: torch.Tensor, accept_host: torch.Tensor):
        """One cycle driven from the host: copy the current tokens [B] in
        (pinned -> device), run the cycle, copy tokens / accept lengths out
        (device -> pinned) and wait for them."""
        self.cur.copy_(cur_host, non_blocking=True)
        self.step()
        tokens_host.copy_(self.tokens, non_blocking=True)
        accept_host.copy_(self.accept_len, non_blocking=True)
        if getattr(self, "_watch", None) is None:
            self._watch = StatusWatch(self.target.status_regions() + self.draft.status_regions())
        self._watch.copy()   # the kernels' status words, read with the results
        torch.cuda.current_stream().synchronize()
        self._watch.check()
        return tokens_host, accept_host

    def prepare(self, prompt: torch.Tensor, lengths: torch.Tensor | None = None):
        """Prefill, capture the cycle graph (its warm-up run disturbs the
        caches, so the prefill is redone after capture), return first tokens."""
        if self.use_graph and self.graph is None:
            self.prefill(prompt, lengths)
            self._capture()
        return self.prefill(prompt, lengths)

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n_new: int, lengths: torch.Tensor | None = None):
        """Greedy speculative generation; returns ([B, n_new] tokens, accept lens per cycle)."""
        B = prompt.shape[0]
        first = self.prepare(prompt, lengths).cpu()
        out = [[int(first[b])] for b in range(B)]
        accepts = []
        while min(len(o) for o in out) < n_new:
            tokens, n = self.step()
            tokens, n = tokens.cpu(), n.cpu()
            accepts.append(n.clone())
            for b in range(B):
                out[b].extend(int(x) for x in tokens[b, :int(n[b]) + 1])
        return torch.tensor([o[:n_new] for o in out]), torch.stack(accepts)


class AutoregressiveEngine:
    """Greedy decoding with the target alone (one T=1 forward per token)."""

    def __init__(self, target: QwenModel, use_graph: bool = True):
        self.target = target
        B = target.batch
        dev = target.device
        self.cur = torch.zeros(B, dtype=torch.int64, device=dev)
        self.last = torch.zeros(B, dtype=torch.int64, device=dev)
        self.next = torch.zeros(B, dtype=torch.int64, device=dev)
        self.acc = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(B, 1, dtype=torch.int64, device=dev)
        pl = target.forward_plan(self.cur, 1, B, 1, target.lengths, 0, self.next, 1, last_only=True)
        pl.add("tsds_accept_greedy", _p(self.next), _p(self.next), _p(self.acc), _p(self.tokens), _p(target.lengths),
               _p(self.last), _p(self.cur), B, 0)
        self.plan = pl
        self.use_graph = use_graph
        self.graph = None

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n_new: int, lengths: torch.Tensor | None = None) -> torch.Tensor:
        prompt = prompt.to(self.target.device)

        def prefill():
            hidden = self.target.prefill(prompt, lengths)
            self.cur.copy_(self.target.logits_of(self.target.last_rows(hidden, lengths)).argmax(-1))
            return self.cur.clone()

        if self.use_graph and self.graph is None:
            prefill()
            self.plan.run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.plan.run()
            self.graph = g
        out = [prefill()]
        for _ in range(n_new - 1):
            if self.use_graph:
                self.graph.replay()
            else:
                self.plan.run()
            out.append(self.cur.clone())
        return torch.stack(out, dim=1).cpu()

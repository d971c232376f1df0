"""CPU oracle of the chain speculative-decoding cycle (test infrastructure).

The reference wires only ``draft`` (tri_sds/worker.py:53-64); ``verify``,
acceptance and KV rollback raise or live in SGLang (worker.py:49-51,66-68),
which is not part of the reference tree.  The semantics are therefore
written down here and pinned by properties (greedy spec output equals
greedy autoregressive output), not by reference golden vectors.

Cycle, per sequence b with ``L = target.lengths[b]`` committed target rows
and ``cur`` the newest token (not yet in any cache), ``last`` the token
before it:

1. draft step 1 runs ``[last, cur]`` at positions ``L-1, L`` (rewriting the
   draft's row L-1 with identical values when it already holds it), then
   steps 2..K run ``d_{i-1}`` at position ``L+i-1``; ``d_i`` = argmax.
2. the target verifies ``[cur, d_1..d_K]`` at positions ``L..L+K``.
3. greedy acceptance: ``n`` = length of the longest prefix with
   ``d_{i+1} == y_i`` (y = target argmax); the cycle emits
   ``d_1..d_n, y_n`` (n+1 tokens).
4. commit: ``target.lengths = L+n+1``; ``draft.lengths = L+n``; the rows
   written past those lengths are stale and overwritten by later steps.
"""
from __future__ import annotations

import torch

from .qwen import QwenOracle


def greedy_accept(draft_tokens: torch.Tensor, target_argmax: torch.Tensor):
    """draft_tokens [B,K], target_argmax [B,K+1] ->
    (accept_len [B] int32, tokens [B,K+1] int64 padded with -1).

    ``tokens[b, :n+1] = target_argmax[b, :n+1]`` (the accepted drafts equal
    the target's argmax there, and position n is the bonus token)."""
    B, K = draft_tokens.shape
    match = (draft_tokens == target_argmax[:, :K]).to(torch.int64)
    n = torch.cumprod(match, dim=1).sum(dim=1)
    idx = torch.arange(K + 1).unsqueeze(0)
    tokens = torch.where(idx <= n.unsqueeze(1), target_argmax, torch.full_like(target_argmax, -1))
    return n.to(torch.int32), tokens


class ChainSpecOracle:
    """Greedy chain speculative decoding with a separate draft model."""

    def __init__(self, target: QwenOracle, draft: QwenOracle, k: int):
        assert target.batch == draft.batch
        self.target, self.draft, self.k = target, draft, k

    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        B, P = prompt.shape
        self.target.reset_cache()
        self.draft.reset_cache()
        logits, _ = self.target.forward(prompt)
        self.target.lengths[:] = P
        if P > 1:
            self.draft.forward(prompt[:, :P - 1])
        self.draft.lengths[:] = P - 1
        self.last = prompt[:, -1].clone()
        self.cur = logits[:, -1].argmax(-1)
        return self.cur.clone()

    def draft_chain(self):
        """K greedy draft steps; returns d [B,K]."""
        L = self.target.lengths.clone()
        k = self.k
        ids = torch.stack([self.last, self.cur], dim=1)
        logits, _ = self.draft.forward(ids, starts=L - 1)
        d = [logits[:, -1].argmax(-1)]
        for i in range(2, k + 1):
            logits, _ = self.draft.forward(d[-1].unsqueeze(1), starts=L + i - 1)
            d.append(logits[:, -1].argmax(-1))
        return torch.stack(d, dim=1)

    def step(self):
        """One cycle -> (tokens [B,K+1] padded -1, accept_len [B])."""
        d = self.draft_chain()
        L = self.target.lengths.clone()
        ids = torch.cat([self.cur.unsqueeze(1), d], dim=1)
        logits, _ = self.target.forward(ids, starts=L)
        y = logits.argmax(-1)
        n, tokens = greedy_accept(d, y)
        n64 = n.to(torch.int64)
        self.target.lengths = L + n64 + 1
        self.draft.lengths = L + n64
        bidx = torch.arange(d.shape[0])
        self.last = torch.where(n64 == 0, self.cur, d[bidx, (n64 - 1).clamp(min=0)])
        self.cur = y[bidx, n64]
        return tokens, n

    def generate(self, prompt: torch.Tensor, n_new: int):
        B = prompt.shape[0]
        first = self.prefill(prompt)
        out = [[int(first[b])] for b in range(B)]
        accepts = []
        while min(len(o) for o in out) < n_new:
            tokens, n = self.step()
            accepts.append(n.clone())
            for b in range(B):
                out[b].extend(int(t) for t in tokens[b, :int(n[b]) + 1])
        return torch.tensor([o[:n_new] for o in out]), torch.stack(accepts)


def autoregressive(target: QwenOracle, prompt: torch.Tensor, n_new: int) -> torch.Tensor:
    """Plain greedy decoding with the target alone (one token per forward)."""
    B, P = prompt.shape
    target.reset_cache()
    logits, _ = target.forward(prompt)
    target.lengths[:] = P
    tok = logits[:, -1].argmax(-1)
    out = [tok]
    for _ in range(n_new - 1):
        logits, _ = target.forward(tok.unsqueeze(1))
        target.lengths += 1
        tok = logits[:, -1].argmax(-1)
        out.append(tok)
    return torch.stack(out, dim=1)

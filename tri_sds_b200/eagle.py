"""EAGLE tree speculative decoding on the device.

The draft head (the workload's form of ``tri_sds/triton_kernels/eagle_head.py``):
fc [N, 2N] + bias over [feature | token embedding], then one decoder layer
of the target's shape whose attention covers the current draft tree only,
then the target's final norm and LM head.  One cycle, for B sequences:

1. ``tsds_tree_init``: root = (feature of the last committed row, current token);
2. ``depth`` head passes: pass 0 over the root, passes 1.. over the frontier
   (<= topk nodes per sequence); each pass = input gather, fc + bias, the
   decoder layer (tree mask over the head's small cache, positions L + depth),
   final norm + LM head (logits kept for the acceptance), top-k +
   log-sum-exp, ``tsds_tree_step`` (children, next frontier);
3. ``tsds_tree_finalize``: the ``n_nodes`` best nodes + root, ancestor masks;
4. one target pass over the tree (attention with the ancestor mask);
5. ``tsds_accept_tree_rule``: rejection sampling at temperature 1 with
   supplied uniforms (or greedy), emitted tokens, ``cur`` <- bonus.  The
   tree's children are its top-k (chosen without the uniforms), so the
   default rule is the target-only one (``ACCEPT_TARGET``: accept child x if
   u < p(x), else drop x from p), under which the emitted tokens follow the
   target's distribution; ``ACCEPT_DRAFT`` (u q(x) < p(x), residual
   max(p - q, 0)) is lossless only for children drawn from q;
6. ``tsds_tree_commit``: KV compaction, next root feature, lengths += a + 1
   (with a target on paged KV, ``tsds_tree_commit_paged``: the accepted
   nodes' pool rows take the next positions in the table, no K/V moves).

Semantics are the oracle's (oracle/eagle.py).
"""
from __future__ import annotations

from dataclasses import replace

import torch

from .model import Plan, QwenModel, StatusWatch, _p
from .shapes import QwenShape


class EagleHead:
    """fc + bias and one target-shape decoder layer, sharing the target's
    embedding, final norm and LM head."""

    def __init__(self, target: QwenModel, batch: int, topk: int = 4, depth: int = 5, weights: dict | None = None,
                 seed: int = 0, share: "EagleHead | None" = None):
        """``share``: another head (same shape) whose fc and layer weights
        this one uses, for a target over the same weights at another batch
        size."""
        s = target.shape
        self.shape = replace(s, n_layers=1)
        self.rows_per_seq = 1 + topk * (depth - 1)
        dev = target.device
        lw = None
        if weights is not None:
            lw = {"layers": [weights["layer"]], "embed": None, "lm_head": None, "norm": None}
        self.model = QwenModel(self.shape, batch=batch, max_seq=32, max_rows=batch * topk, device=dev, weights=lw,
                               seed=seed, share_embeddings=target, rope_len=target.rope_len, fused_layers=target.fused_layers,
                               share_weights=None if share is None else share.model)
        if share is not None:
            self.fc_w, self.fc_b = share.fc_w, share.fc_b
        elif weights is not None:
            self.fc_w = weights["fc"].to(dev, torch.bfloat16).contiguous()
            self.fc_b = weights["fc_bias"].to(dev, torch.bfloat16).contiguous()
        else:
            g = torch.Generator(device=dev)
            g.manual_seed(seed + 1)
            self.fc_w = (torch.randn(s.hidden, 2 * s.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            self.fc_b = (torch.randn(s.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)


ACCEPT_DRAFT, ACCEPT_TARGET = 0, 1


class EagleEngine:
    def __init__(self, target: QwenModel, head: EagleHead, topk: int = 4, depth: int = 5, n_nodes: int = 25,
                 greedy: bool = False, use_graph: bool = True, seed: int = 0, rule: int = ACCEPT_TARGET):
        B = target.batch
        s = target.shape
        NN = n_nodes + 1
        assert target.max_rows >= B * NN and NN <= 32
        self.target, self.head = target, head
        self.topk, self.depth, self.n_nodes, self.greedy = topk, depth, n_nodes, greedy
        assert rule in (ACCEPT_DRAFT, ACCEPT_TARGET)
        self.rule = rule
        dev = target.device
        R = B * head.rows_per_seq
        i64, i32, f32, bf = (dict(dtype=t, device=dev) for t in (torch.int64, torch.int32, torch.float32,
                                                                   torch.bfloat16))
        from . import _lib
        self.states = torch.zeros(_lib.query("tsds_tree_state_bytes", B), dtype=torch.uint8, device=dev)
        self.x2 = torch.zeros(B * topk, 2 * s.hidden, **bf)
        self.head_feat = torch.zeros(R, s.hidden, **bf)
        self.head_logits = torch.zeros(R, s.vocab, **bf)
        self.head_argmax = torch.zeros(R, **i64)
        self.vals = torch.zeros(R, topk, **f32)
        self.idx = torch.zeros(R, topk, **i32)
        self.lse = torch.zeros(R, **f32)
        self.pass_tok = torch.zeros(B * topk, **i64)
        self.pass_featrow = torch.zeros(B * topk, **i32)
        self.pass_pos = torch.zeros(B * topk, **i32)
        self.pass_mask = torch.zeros(B * topk, **i32)
        self.pass_starts = torch.zeros(B, **i32)
        self.ids = torch.zeros(B * NN, **i64)
        self.vmask = torch.zeros(B * NN, **i32)
        self.hrow = torch.zeros(B * NN, **i32)
        self.children = torch.zeros(B * NN * topk, **i32)
        self.target_logits = torch.zeros(B * NN, s.vocab, **bf)
        self.target_argmax = torch.zeros(B * NN, **i64)
        self.U = torch.zeros(B, depth + 1, topk + 1, **f32)
        self.path = torch.zeros(B * (depth + 1), **i32)
        self.accept_len = torch.zeros(B, **i32)
        self.tokens = torch.zeros(B, depth + 2, **i64)
        self.cur = torch.zeros(B, **i64)
        self.root_feat = torch.zeros(B, s.hidden, **bf)
        # pooled KV: the pool rows each commit keeps (root + accepted nodes, -1 padded)
        self.kept_rows = torch.full((B, depth + 2), -1, **i64)
        self.gen = torch.Generator(device=dev)
        self.gen.manual_seed(seed)
        self.use_graph = use_graph
        self.graph = None
        self.plan = self._cycle_plan()
        self.plan_launches = None

    # -- one cycle ---------------------------------------------------------------
    def _head_pass(self, pl: Plan, d: int):
        t, h, hm = self.target, self.head, self.head.model
        s = t.shape
        B, k = t.batch, self.topk
        T = 1 if d == 0 else k
        base = 0 if d == 0 else B * (1 + k * (d - 1))
        M = B * T
        feat = self.head_feat[base:base + M]
        pl.add("tsds_eagle_inputs", _p(self.root_feat), _p(self.head_feat), _p(self.pass_featrow),
               _p(self.pass_tok), _p(t.embed_w), _p(self.x2), B, T, s.hidden, s.vocab)
        pl.add("tsds_linear_bias", _p(self.x2), 2 * s.hidden, _p(h.fc_w), _p(h.fc_b), _p(feat), s.hidden, M,
               s.hidden, 2 * s.hidden, _p(hm.lin_ws), hm.lin_ws_bytes)
        lp = hm.layers_plan(B, T, tree_mask=self.pass_mask, mask_origin=0, x=feat, starts=self.pass_starts,
                            positions=self.pass_pos, final_norm=True)
        pl.extend(lp)
        pl.extend(hm.head_plan(B, T, self.head_argmax[base:], 1, last_only=False,
                               logits_out=self.head_logits[base:], x=feat, normed=lp.final_normed))
        pl.add("tsds_logits_topk", _p(self.head_logits[base:]), s.vocab, M, s.vocab, k, _p(self.vals[base:]),
               _p(self.idx[base:]), _p(self.lse[base:]))
        next_T = k if d + 1 < self.depth else 0
        pl.add("tsds_tree_step", _p(self.states), _p(self.vals), _p(self.idx), _p(self.lse), base, T, k, next_T,
               _p(t.lengths), _p(self.pass_tok), _p(self.pass_featrow), _p(self.pass_pos), _p(self.pass_mask),
               _p(self.pass_starts), B)

    def _cycle_plan(self) -> Plan:
        t = self.target
        s = t.shape
        B, k, NN = t.batch, self.topk, self.n_nodes + 1
        pl = Plan()
        pl.add("tsds_tree_init", _p(self.states), _p(self.cur), _p(t.lengths), _p(self.pass_tok),
               _p(self.pass_featrow), _p(self.pass_pos), _p(self.pass_mask), _p(self.pass_starts), B)
        for d in range(self.depth):
            self._head_pass(pl, d)
        pl.add("tsds_tree_finalize", _p(self.states), self.n_nodes, k, _p(t.lengths), _p(self.ids),
               _p(t.positions), _p(self.vmask), _p(self.hrow), _p(self.children), _p(t.starts), B)
        pl.add("tsds_embed", _p(self.ids), 1, _p(t.embed_w), _p(t.x), B * NN, s.hidden, s.vocab)
        lp = t.layers_plan(B, NN, tree_mask=self.vmask, mask_origin=-1, final_norm=True)
        pl.extend(lp)
        pl.extend(t.head_plan(B, NN, self.target_argmax, 1, last_only=False, logits_out=self.target_logits,
                              normed=lp.final_normed))
        pl.add("tsds_accept_tree_rule", _p(self.target_logits), _p(self.target_argmax), _p(self.head_logits),
               _p(self.ids), _p(self.hrow), _p(self.children), None if self.greedy else _p(self.U),
               self.rule, _p(self.path), _p(self.accept_len), _p(self.tokens), _p(self.cur), B,
               self.n_nodes, s.vocab, k, self.depth)
        if t.kv is not None:
            # pooled KV: the accepted nodes' pool rows become the next
            # positions (table entries move, K/V stay); kept_rows lists them
            kv = t.kv
            pl.add("tsds_tree_commit_paged", _p(kv.table), kv.table_ld, _p(kv.req_rows), _p(t.lengths),
                   _p(self.path), _p(self.accept_len), self.depth, _p(self.kept_rows), _p(t.x), self.n_nodes,
                   s.hidden, _p(self.root_feat), B)
            return pl
        # the cache's own kv-head count: under tensor parallelism a rank holds
        # only its shard of the kv heads
        pl.add("tsds_tree_commit", _p(t.k_cache), _p(t.v_cache), s.n_layers, B, t.k_cache.shape[2], t.max_seq,
               s.head_dim, _p(t.lengths), _p(self.path), _p(self.accept_len), self.depth, _p(t.x), self.n_nodes,
               s.hidden, _p(self.root_feat))
        return pl

    def verify_only_plan(self) -> Plan:
        """The target's tree verify forward alone (for timing the verify step)."""
        t = self.target
        s = t.shape
        B, NN = t.batch, self.n_nodes + 1
        pl = Plan()
        pl.add("tsds_embed", _p(self.ids), 1, _p(t.embed_w), _p(t.x), B * NN, s.hidden, s.vocab)
        lp = t.layers_plan(B, NN, tree_mask=self.vmask, mask_origin=-1, final_norm=True)
        pl.extend(lp)
        pl.extend(t.head_plan(B, NN, self.target_argmax, 1, last_only=False, logits_out=self.target_logits,
                              normed=lp.final_normed))
        return pl

    @property
    def k(self):
        return self.topk

    def step_host(self, cur_host: torch.Tensor, tokens_host: torch.Tensor, accept_host: torch.Tensor):
        """One cycle driven from the host (pinned buffers), as SpecEngine.step_host."""
        self.cur.copy_(cur_host, non_blocking=True)
        self.step()
        tokens_host.copy_(self.tokens, non_blocking=True)
        accept_host.copy_(self.accept_len, non_blocking=True)
        if getattr(self, "_watch", None) is None:
            self._watch = StatusWatch(self.target.status_regions() + self.head.model.status_regions())
        self._watch.copy()   # the kernels' status words, read with the results
        torch.cuda.current_stream().synchronize()
        self._watch.check()
        return tokens_host, accept_host

    # -- driving -----------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        """Prefill the target from a [B, P] prompt (ragged: ``lengths[b]``
        real tokens per row); the root of the first tree is each sequence's
        last prompt token's feature and argmax."""
        t = self.target
        prompt = prompt.to(t.device)
        hidden = t.prefill(prompt, lengths)
        last = t.last_rows(hidden, lengths)
        first = t.logits_of(last).argmax(-1)
        self.cur.copy_(first)
        self.root_feat.copy_(last)
        return first

    def draw_uniforms(self, U: torch.Tensor | None = None):
        if U is None:
            torch.rand(self.U.shape, generator=self.gen, device=self.U.device, out=self.U)
        else:
            self.U.copy_(U)

    def _capture(self):
        from . import _lib
        c0 = _lib.query("tsds_launch_count")
        self.plan.run()
        self.plan_launches = _lib.query("tsds_launch_count") - c0
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.plan.run()
        self.graph = g

    def prepare(self, prompt: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        if self.use_graph and self.graph is None:
            self.prefill(prompt, lengths)
            self._capture()
        return self.prefill(prompt, lengths)

    def step(self, U: torch.Tensor | None = None):
        """One cycle -> (tokens [B, depth+2] padded -1, accept_len [B])."""
        self.target.ensure_usable()
        if not self.greedy:
            self.draw_uniforms(U)
        if self.use_graph:
            self.graph.replay()
        else:
            self.plan.run()
        return self.tokens, self.accept_len

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, n_new: int, lengths: torch.Tensor | None = None):
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

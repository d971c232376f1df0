"""CPU oracle of the EAGLE draft head, tree drafting and rejection sampling
(test infrastructure).

Reference form (pinned by golden vectors): ``EagleHeadRef`` restates
``tri_sds/triton_kernels/eagle_head.py:16-97`` (fc over [features | token
embeddings] with bias, RMSNorm, single-head causal attention with head dim =
hidden and no RoPE, o-proj + residual, RMSNorm, SwiGLU + residual) and
``eagle_draft_decode_ref`` the chain draft of ``eagle_head.py:100-129``
(argmax over the target's final norm + LM head of each predicted feature).
The state-dict layout quirks of ``load_state_dict`` (eagle_head.py:52-74)
are kept: fc and q/k/v weights are stored [in, out], o/gate/up/down [out, in].

Workload form (what the device runs): the head is fc [N, 2N] (+ bias) over
[feature | embedding] followed by one Qwen3 decoder layer of the target's
shape (GQA, QK-norm, RoPE) whose attention covers the current draft tree
only - as in the reference, where the head attends over the draft chain
that starts at the last verified feature and not over the prompt.

Tree drafting, rejection sampling and KV compaction are absent from the
reference (SGLang owns them); their semantics are defined here:

* node n's head input is (feature predicted for its parent, token of n); the
  root's is (target hidden state of the last committed row, current token).
  Its output feature f_n gives q_n = softmax(lm_head(norm(f_n))), the
  distribution of n's children.
* depth 1: the root's top-4 tokens (value desc, index asc).  Each later
  depth expands the frontier (<= 4 nodes): every frontier node's top-4
  children become candidates with cumulative score = parent score +
  log q(child); the 4 best candidates (score desc, creation order asc) form
  the next frontier.  After ``depth`` head passes, all candidates are ranked
  (score desc, depth asc, creation order asc) and the best ``n_nodes`` kept;
  scores never increase along a path, so kept nodes form a tree.
* verify: the target runs [root, kept nodes] (creation order, parents first)
  at positions L + depth with the ancestor mask.
* rejection sampling at temperature 1: at node n with target distribution
  p and draft distribution q, children are tried in draft-rank order; child
  x is accepted when ``u * q(x) < p(x)``; on rejection p <- norm(max(p - q,
  0)) and q <- q with q(x) = 0, renormalised; when no child is accepted (or
  n has none) the bonus token is drawn from p by inverse CDF with one more
  uniform.  Uniforms come in ``[B, depth + 1, topk + 1]``: u[b, d, i] for the
  i-th child tried at depth d, u[b, d, topk] for the bonus draw.
* greedy (temperature 0): accept the child equal to the target's argmax.
* KV compaction: the accepted path's nodes move from rows L + node_index to
  rows L + 1 .. L + a of every layer; lengths += a + 1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .qwen import QwenShape, apply_rope, precompute_rope, rms_norm


# ---------------------------------------------------------------------------
# reference form (eagle_head.py)
# ---------------------------------------------------------------------------

class EagleHeadRef:
    """eagle_head.py:16-97 restated; weights from the reference's state dict."""

    def __init__(self, sd: dict, dtype=torch.float32):
        t = lambda k: sd[k].to(dtype) if k in sd else None  # noqa: E731
        self.fc_w = t("fc.weight")                      # [2N, N]
        self.N = self.fc_w.shape[1]
        self.fc_b = t("fc.bias") if "fc.bias" in sd else torch.zeros(self.N, dtype=dtype)
        self.attn_norm = t("attn.norm.weight")
        self.q_w, self.k_w, self.v_w = t("attn.q_proj.weight"), t("attn.k_proj.weight"), t("attn.v_proj.weight")
        self.o_w = t("attn.o_proj.weight").T.contiguous()
        self.ffn_norm = t("ffn.norm.weight")
        self.g_w = t("ffn.gate_proj.weight").T.contiguous()
        self.u_w = t("ffn.up_proj.weight").T.contiguous()
        self.d_w = t("ffn.down_proj.weight").T.contiguous()

    def forward(self, features: torch.Tensor, token_embeds: torch.Tensor) -> torch.Tensor:
        B, T = features.shape[:2]
        h = torch.cat([features, token_embeds], dim=-1) @ self.fc_w + self.fc_b
        a_in = rms_norm(h.reshape(B * T, self.N), self.attn_norm).reshape(B, T, self.N)
        q = (a_in @ self.q_w).unsqueeze(1)
        k = (a_in @ self.k_w).unsqueeze(1)
        v = (a_in @ self.v_w).unsqueeze(1)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        h = h + a.squeeze(1) @ self.o_w
        f_in = rms_norm(h.reshape(B * T, self.N), self.ffn_norm).reshape(B, T, self.N)
        return h + (F.silu(f_in @ self.g_w) * (f_in @ self.u_w)) @ self.d_w


def eagle_draft_decode_ref(last_hidden, last_token, head: EagleHeadRef, embed_w, norm_w, lm_head_w, n_draft=4):
    """eagle_head.py:100-129: chain draft by argmax."""
    B = last_hidden.shape[0]
    feats, toks = [last_hidden], [last_token]
    out_tok, out_logits = [], []
    for _ in range(n_draft):
        pred = head.forward(torch.cat(feats, 1), embed_w[torch.cat(toks, 1)])
        nxt = pred[:, -1:, :]
        logits = rms_norm(nxt.reshape(B, -1), norm_w) @ lm_head_w.T
        tok = logits.argmax(-1, keepdim=True)
        out_tok.append(tok)
        out_logits.append(logits)
        feats.append(nxt)
        toks.append(tok)
    return out_tok, out_logits


# ---------------------------------------------------------------------------
# workload form: fc + one target-shape Qwen3 decoder layer over the tree
# ---------------------------------------------------------------------------

def random_eagle_weights(shape: QwenShape, seed: int, dtype=torch.bfloat16, std: float = 0.02) -> dict:
    g = torch.Generator().manual_seed(seed)
    N, D, I = shape.hidden, shape.head_dim, shape.intermediate

    def mat(o, i):
        return (torch.randn(o, i, generator=g) * std).to(dtype)

    def gain(n):
        return (1.0 + 0.02 * torch.randn(n, generator=g)).to(dtype)

    layer = {"q": mat(shape.q_dim, N), "k": mat(shape.kv_dim, N), "v": mat(shape.kv_dim, N),
             "o": mat(N, shape.q_dim), "gate": mat(I, N), "up": mat(I, N), "down": mat(N, I),
             "ln1": gain(N), "ln2": gain(N), "q_norm": gain(D), "k_norm": gain(D)}
    return {"fc": mat(N, 2 * N), "fc_bias": (torch.randn(N, generator=g) * std).to(dtype), "layer": layer}


class EagleHeadQwen:
    """fc [N, 2N] + bias, then one Qwen3 layer with a per-cycle tree cache."""

    def __init__(self, shape: QwenShape, w: dict, batch: int, max_rows: int = 32, max_pos: int = 4096,
                 dtype=torch.bfloat16):
        self.shape, self.dtype, self.batch, self.max_rows = shape, dtype, batch, max_rows
        cv = lambda t: t.to(dtype)  # noqa: E731
        self.fc_w_t = cv(w["fc"]).T.contiguous()
        self.fc_b = cv(w["fc_bias"])
        L = w["layer"]
        self.qkv_w_t = torch.cat([cv(L["q"]), cv(L["k"]), cv(L["v"])], 0).T.contiguous()
        self.o_w_t = cv(L["o"]).T.contiguous()
        self.gu_w_t = torch.cat([cv(L["gate"]), cv(L["up"])], 0).T.contiguous()
        self.d_w_t = cv(L["down"]).T.contiguous()
        self.ln1, self.ln2 = cv(L["ln1"]), cv(L["ln2"])
        self.qn, self.kn = cv(L["q_norm"]), cv(L["k_norm"])
        self.cos, self.sin = precompute_rope(shape.head_dim, max_pos, shape.rope_theta, dtype)
        self.reset()

    def reset(self):
        s = self.shape
        self.k = torch.zeros(self.batch, s.n_kv_heads, self.max_rows, s.head_dim, dtype=self.dtype)
        self.v = torch.zeros_like(self.k)

    def forward(self, feats, embeds, rows: torch.Tensor, positions: torch.Tensor, masks: torch.Tensor):
        """T nodes per sequence.  rows[b, t]: cache row of the node; positions
        [b, t]: RoPE position; masks[b, t]: bitmask over cache rows 0..31 that
        the node attends to (its ancestors and itself).  Returns features [B, T, N]."""
        s = self.shape
        B, T, N = feats.shape
        h = torch.cat([feats, embeds], -1) @ self.fc_w_t + self.fc_b
        xn = rms_norm(h, self.ln1, s.eps)
        qkv = xn @ self.qkv_w_t
        q = rms_norm(qkv[..., :s.q_dim].reshape(B, T, s.n_heads, s.head_dim), self.qn, s.eps).transpose(1, 2)
        k = rms_norm(qkv[..., s.q_dim:s.q_dim + s.kv_dim].reshape(B, T, s.n_kv_heads, s.head_dim), self.kn,
                     s.eps).transpose(1, 2)
        v = qkv[..., s.q_dim + s.kv_dim:].reshape(B, T, s.n_kv_heads, s.head_dim).transpose(1, 2)
        q = apply_rope(q, self.cos, self.sin, positions)
        k = apply_rope(k, self.cos, self.sin, positions)
        outs = []
        for b in range(B):
            for t in range(T):
                self.k[b, :, int(rows[b, t])] = k[b, :, t]
                self.v[b, :, int(rows[b, t])] = v[b, :, t]
            kk = self.k[b].repeat_interleave(s.q_per_kv, 0)
            vv = self.v[b].repeat_interleave(s.q_per_kv, 0)
            key = torch.arange(self.max_rows)
            vis = ((masks[b].to(torch.int64).unsqueeze(1) >> key) & 1) == 1       # [T, R]
            m = torch.zeros(T, self.max_rows, dtype=q.dtype).masked_fill(~vis, float("-inf"))
            outs.append(F.scaled_dot_product_attention(q[b:b + 1], kk.unsqueeze(0), vv.unsqueeze(0), attn_mask=m))
        a = torch.cat(outs).transpose(1, 2).reshape(B, T, s.q_dim)
        h = h + a @ self.o_w_t
        xn2 = rms_norm(h, self.ln2, s.eps)
        gu = xn2 @ self.gu_w_t
        return h + (F.silu(gu[..., :s.intermediate]) * gu[..., s.intermediate:]) @ self.d_w_t


# ---------------------------------------------------------------------------
# tree drafting
# ---------------------------------------------------------------------------

def topk_desc(x: torch.Tensor, k: int):
    """Top-k of a 1-D tensor: value desc, index asc on ties."""
    idx = torch.arange(x.numel())
    order = sorted(range(x.numel()), key=lambda i: (-float(x[i]), i))[:k] if x.numel() <= 64 else None
    if order is None:
        vals, cand = torch.topk(x.float(), min(k + 16, x.numel()))
        thr = float(vals[-1])
        sel = idx[x.float() >= thr]
        order = sorted(sel.tolist(), key=lambda i: (-float(x[i]), i))[:k]
    return torch.tensor(order, dtype=torch.int64)


@dataclass
class Tree:
    tokens: list        # [n] token ids; index 0 = root (the current token)
    parent: list        # [n] parent index (-1 for the root)
    depth: list         # [n]
    mask: list          # [n] ancestor-or-self bitmask over tree indices
    head_row: list      # [n] head row whose q gives this node's children (-1: not expanded)
    children: list      # [n] list of child indices in draft-rank order
    candidates: dict | None = None   # token path from the root -> cumulative score, every candidate
    cutoff: float | None = None      # score of the last kept candidate


class TreeBuilder:
    """The tree-selection rules, fed one head pass at a time.

    ``frontier()`` lists the candidates the next pass must run (creation
    order); ``add_pass(logits)`` takes that pass's logits rows [T, V] in the
    same order; ``finish()`` keeps the ``n_nodes`` best and returns the Tree.
    Driving it with the device's own head logits checks the device's
    selection logic exactly, independent of the head's numerics."""

    def __init__(self, root_tok: int, depth: int = 5, topk: int = 4, n_nodes: int = 25):
        self.depth, self.topk, self.n_nodes = depth, topk, n_nodes
        self.cand = [dict(tok=int(root_tok), parent=-1, depth=0, score=0.0, rank=0, row=-1)]
        self._frontier = [0]
        self.passes = 0
        self.rows = 0

    def frontier(self) -> list:
        return list(self._frontier)

    def add_pass(self, logits: torch.Tensor):
        logits = logits.float()
        new = []
        for t, ci in enumerate(self._frontier):
            self.cand[ci]["row"] = self.rows + t
            lse = torch.logsumexp(logits[t], 0)
            for r, tok in enumerate(topk_desc(logits[t], self.topk).tolist()):
                new.append(dict(tok=tok, parent=ci, depth=self.cand[ci]["depth"] + 1,
                                score=self.cand[ci]["score"] + float(logits[t][tok] - lse), rank=r, row=-1))
        self.rows += len(self._frontier)
        base = len(self.cand)
        self.cand.extend(new)
        self.passes += 1
        if self.passes < self.depth:
            order = sorted(range(len(new)), key=lambda i: (-new[i]["score"], i))[:self.topk]
            self._frontier = [base + i for i in sorted(order)]
        else:
            self._frontier = []

    def finish(self) -> "Tree":
        cand = self.cand
        ids = sorted(range(1, len(cand)), key=lambda i: (-cand[i]["score"], cand[i]["depth"], i))[:self.n_nodes]
        keep = [0] + sorted(ids)
        pos_of = {ci: j for j, ci in enumerate(keep)}
        tokens = [cand[ci]["tok"] for ci in keep]
        parent = [-1 if cand[ci]["parent"] < 0 else pos_of[cand[ci]["parent"]] for ci in keep]
        dep = [cand[ci]["depth"] for ci in keep]
        mask = []
        for j in range(len(keep)):
            m, q = 0, j
            while q >= 0:
                m |= 1 << q
                q = parent[q]
            mask.append(m)
        head_row = [cand[ci]["row"] for ci in keep]
        children = [[] for _ in keep]
        for j in range(1, len(keep)):
            children[parent[j]].append(j)
        for j in range(len(keep)):
            children[j].sort(key=lambda c: cand[keep[c]]["rank"])

        def path_of(ci):
            p = []
            while ci > 0:
                p.append(cand[ci]["tok"])
                ci = cand[ci]["parent"]
            return tuple(reversed(p))
        cands = {path_of(ci): cand[ci]["score"] for ci in range(1, len(cand))}
        cutoff = cand[ids[-1]]["score"] if ids else 0.0
        return Tree(tokens, parent, dep, mask, head_row, children, cands, cutoff)


def build_tree(head: EagleHeadQwen, embed_w, norm_w, lm_head_w, root_feat, root_tok, L, depth=5, topk=4,
               n_nodes=25):
    """Tree drafting for B sequences -> (list of Tree, list of head logits [rows, V] fp32)."""
    B = root_feat.shape[0]
    head.reset()
    trees, all_logits = [], []
    for b in range(B):
        tb = TreeBuilder(int(root_tok[b]), depth, topk, n_nodes)
        feat = {0: root_feat[b]}     # input feature of each candidate
        row_of, row_mask, logits_rows = {}, [], []
        while tb.frontier():
            fr = tb.frontier()
            rows, masks = [], []
            for ci in fr:
                r = len(row_mask) + len(rows)
                m = 1 << r
                par = tb.cand[ci]["parent"]
                if par >= 0:
                    m |= row_mask[row_of[par]]
                rows.append(r)
                masks.append(m)
            feats = torch.stack([feat[ci] for ci in fr]).unsqueeze(0)
            toks = torch.tensor([tb.cand[ci]["tok"] for ci in fr])
            pos = torch.tensor([[int(L[b]) + tb.cand[ci]["depth"] for ci in fr]])
            f = _HeadView(head, b).forward(feats, embed_w[toks].unsqueeze(0), torch.tensor([rows]), pos,
                                           torch.tensor([masks]))[0]
            logits = (rms_norm(f, norm_w) @ lm_head_w.T).float()
            for t, ci in enumerate(fr):
                row_of[ci] = rows[t]
                row_mask.append(masks[t])
                logits_rows.append(logits[t])
            base = len(tb.cand)
            tb.add_pass(logits)
            for ci in range(base, len(tb.cand)):
                feat[ci] = f[fr.index(tb.cand[ci]["parent"])]
        trees.append(tb.finish())
        all_logits.append(torch.stack(logits_rows))
    return trees, all_logits


class _HeadView:
    """Run the head for one sequence b of its batch."""

    def __init__(self, head: EagleHeadQwen, b: int):
        self.head, self.b = head, b

    def forward(self, feats, embeds, rows, pos, masks):
        h = self.head
        k, v = h.k, h.v
        h.k, h.v = k[self.b:self.b + 1], v[self.b:self.b + 1]
        try:
            return h.forward(feats, embeds, rows, pos, masks)
        finally:
            k[self.b:self.b + 1] = h.k
            v[self.b:self.b + 1] = h.v
            h.k, h.v = k, v


# ---------------------------------------------------------------------------
# acceptance on a tree
# ---------------------------------------------------------------------------

def inverse_cdf(p: torch.Tensor, u: float) -> int:
    """First index whose cumulative mass exceeds u * total (fp32 cumsum)."""
    c = torch.cumsum(p.float(), 0)
    i = int(torch.searchsorted(c, torch.tensor([u * float(c[-1])], dtype=torch.float32), right=True)[0])
    i = min(i, p.numel() - 1)
    while i > 0 and float(p[i]) == 0.0:
        i -= 1
    return i


RULE_DRAFT, RULE_TARGET = 0, 1


def accept_tree_rejection(tree: Tree, target_logits: torch.Tensor, head_logits: torch.Tensor, U: torch.Tensor,
                          topk: int = 4, rule: int = RULE_DRAFT):
    """Rejection sampling at temperature 1 -> (accepted node indices, bonus token).

    target_logits [n, V] at the tree nodes; head_logits [rows, V] of the head
    passes (row tree.head_row[n] is q of node n's children); U [depth+1, topk+1].

    rule RULE_DRAFT (recursive rejection sampling against the draft's q):
    accept child x when u * q(x) < p(x); on rejection p <- norm(max(p - q, 0))
    and q <- q without x, renormalised.  The emitted token is distributed as
    p when the children are drawn from q without replacement.

    rule RULE_TARGET (the draft taken as deterministic, q one-hot on each
    child in turn): accept child x when u < p(x); on rejection p <- p without
    x, renormalised.  The emitted token is distributed as p for children
    chosen by any rule that does not look at the uniforms - the tree's top-k
    expansion included.  head_logits are not read.

    Either way the bonus is the inverse-CDF draw of the final p with
    U[depth, topk]."""
    node, path, d = 0, [], 0
    while True:
        p = torch.softmax(target_logits[node].float(), 0)
        kids = tree.children[node]
        if kids and rule == RULE_DRAFT:
            q = torch.softmax(head_logits[tree.head_row[node]].float(), 0)
        nxt = None
        for i, c in enumerate(kids):
            x = tree.tokens[c]
            u = float(U[d, i])
            if rule == RULE_TARGET:
                if u < float(p[x]):
                    nxt = c
                    break
                p = p.clone()
                p[x] = 0
                p = p / p.sum()
                continue
            if u * float(q[x]) < float(p[x]):
                nxt = c
                break
            p = torch.clamp(p - q, min=0)
            p = p / p.sum()
            q = q.clone()
            q[x] = 0
            q = q / q.sum()
        if nxt is None:
            return path, inverse_cdf(p, float(U[d, topk]))
        path.append(nxt)
        node = nxt
        d += 1


def accept_tree_greedy(tree: Tree, target_logits: torch.Tensor):
    """Greedy acceptance on a tree -> (accepted node indices, bonus token)."""
    node, path = 0, []
    while True:
        y = int(target_logits[node].argmax())
        nxt = next((c for c in tree.children[node] if tree.tokens[c] == y), None)
        if nxt is None:
            return path, y
        path.append(nxt)
        node = nxt


def compact_kv(k_caches, v_caches, b: int, L: int, path: list):
    """Move the accepted nodes' rows L + node_index to L + 1 .. L + a (every layer)."""
    for kc, vc in zip(k_caches, v_caches):
        for j, n in enumerate(path, start=1):
            kc[b, :, L + j] = kc[b, :, L + n]
            vc[b, :, L + j] = vc[b, :, L + n]

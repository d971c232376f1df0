"""EAGLE oracle: the reference head (golden vectors), tree drafting invariants,
tree verify == chain verify, rejection-sampling properties, KV compaction."""
import math

import pytest
import torch

from conftest import load_golden
from oracle import eagle as oe
from oracle.qwen import QwenOracle, QwenShape, random_qwen_weights, rms_norm

TINY = QwenShape(hidden=64, n_heads=4, n_kv_heads=2, head_dim=16, intermediate=128, n_layers=2, vocab=97)


def test_eagle_head_reference_form_matches_golden():
    fx = load_golden("eagle_ref_f32.pt")
    head = oe.EagleHeadRef(fx["state_dict"])
    tw = fx["target_weights"]
    fwd = head.forward(fx["feats"], tw["embed"][fx["toks"]])
    assert (fwd - fx["forward"]).abs().max().item() <= 1e-5
    toks, logits = oe.eagle_draft_decode_ref(fx["last_hidden"], fx["last_token"], head, tw["embed"], tw["norm"],
                                             tw["lm_head"], n_draft=4)
    assert torch.equal(torch.cat(toks, 1), fx["draft_tokens"])
    assert (torch.stack(logits, 1) - fx["draft_logits"]).abs().max().item() <= 1e-4


def _setup(B=2, dtype=torch.float32, seed=0):
    wt = random_qwen_weights(TINY, seed=seed, dtype=dtype, std=0.2)
    we = oe.random_eagle_weights(TINY, seed=seed + 1, dtype=dtype, std=0.2)
    tgt = QwenOracle(TINY, wt, batch=B, max_seq=128, dtype=dtype)
    head = oe.EagleHeadQwen(TINY, we, batch=B, max_pos=128, dtype=dtype)
    g = torch.Generator().manual_seed(seed + 2)
    prompt = torch.randint(0, TINY.vocab, (B, 12), generator=g)
    _, hidden = tgt.forward(prompt)
    tgt.lengths[:] = 12
    root_feat = hidden[:, -2]        # feature of the row before the current token
    root_tok = prompt[:, -1]
    return tgt, head, wt, root_feat, root_tok, prompt


def test_tree_structure_invariants():
    tgt, head, wt, rf, rt, _ = _setup()
    trees, hl = oe.build_tree(head, tgt.embed_w, tgt.norm_w, tgt.lm_head_w, rf, rt, tgt.lengths, depth=5, topk=4,
                              n_nodes=25)
    for tr, lg in zip(trees, hl):
        n = len(tr.tokens)
        assert n == 26 and lg.shape[0] == 17
        assert tr.parent[0] == -1 and all(0 <= tr.parent[j] < j for j in range(1, n))
        assert max(tr.depth) <= 5 and all(tr.depth[j] == tr.depth[tr.parent[j]] + 1 for j in range(1, n))
        for j in range(1, n):
            assert tr.mask[j] == tr.mask[tr.parent[j]] | (1 << j)
        for j in range(n):
            if tr.children[j]:
                assert tr.head_row[j] >= 0
                kids = oe.topk_desc(lg[tr.head_row[j]], 4).tolist()
                assert [tr.tokens[c] for c in tr.children[j]] == [k for k in kids if k in
                                                                  [tr.tokens[c] for c in tr.children[j]]]


def test_tree_verify_equals_chain_verify():
    """Every node's logits under the tree mask equal a chain forward of its root path."""
    tgt, head, wt, rf, rt, prompt = _setup(B=2)
    trees, _ = oe.build_tree(head, tgt.embed_w, tgt.norm_w, tgt.lm_head_w, rf, rt, tgt.lengths)
    B, L = 2, 12
    ids = torch.tensor([tr.tokens for tr in trees])
    masks = torch.tensor([tr.mask for tr in trees], dtype=torch.int64)
    pos = L + torch.tensor([tr.depth for tr in trees])
    logits, _ = tgt.forward(ids, starts=torch.full((B,), L), positions=pos, tree_mask=masks)
    for b, tr in enumerate(trees):
        for leaf in range(len(tr.tokens)):
            if tr.children[leaf]:
                continue
            path, j = [], leaf
            while j >= 0:
                path.append(j)
                j = tr.parent[j]
            path.reverse()
            chain = QwenOracle(TINY, wt, batch=1, max_seq=128, dtype=torch.float32)
            chain.forward(prompt[b:b + 1])
            chain.lengths[:] = L
            lc, _ = chain.forward(torch.tensor([[tr.tokens[j] for j in path]]))
            assert (lc[0] - logits[b, path]).abs().max().item() <= 1e-4


def test_rejection_accepts_a_full_path_when_draft_equals_target():
    tgt, head, wt, rf, rt, prompt = _setup(B=1)
    trees, hl = oe.build_tree(head, tgt.embed_w, tgt.norm_w, tgt.lm_head_w, rf, rt, tgt.lengths)
    tr = trees[0]
    # target logits at every node := the head's own logits (q == p wherever q exists)
    V = TINY.vocab
    tl = torch.randn(len(tr.tokens), V)
    for j in range(len(tr.tokens)):
        if tr.head_row[j] >= 0:
            tl[j] = hl[0][tr.head_row[j]]
    U = torch.rand(6, 5, generator=torch.Generator().manual_seed(3))
    path, bonus = oe.accept_tree_rejection(tr, tl, hl[0], U)
    assert len(path) >= 1 and tr.children[path[-1]] == []          # accepted down to a leaf
    assert path[0] == tr.children[0][0]                              # u*q < p always holds for the first child


def test_rejection_bonus_distribution_matches_target_without_children():
    """With nothing to accept, the bonus is an inverse-CDF sample of p (chi-square)."""
    V = 6
    p_logits = torch.tensor([0.3, -1.0, 1.2, 0.0, 2.0, -0.5])
    p = torch.softmax(p_logits, 0)
    tr = oe.Tree([0], [-1], [0], [1], [-1], [[]])
    g = torch.Generator().manual_seed(5)
    n = 20000
    counts = torch.zeros(V)
    U = torch.rand(n, 6, 5, generator=g)
    for i in range(n):
        _, tok = oe.accept_tree_rejection(tr, p_logits.unsqueeze(0), torch.zeros(1, V), U[i])
        counts[tok] += 1
    chi2 = (((counts - n * p) ** 2) / (n * p)).sum().item()
    assert chi2 < 20.5  # 5 dof, p ~ 0.001


def test_greedy_tree_acceptance_follows_target_argmax():
    tgt, head, wt, rf, rt, prompt = _setup(B=1)
    trees, _ = oe.build_tree(head, tgt.embed_w, tgt.norm_w, tgt.lm_head_w, rf, rt, tgt.lengths)
    tr = trees[0]
    V = TINY.vocab
    tl = torch.full((len(tr.tokens), V), -5.0)
    # make the target's argmax follow root -> first child -> its first child, then stop
    c1 = tr.children[0][0]
    tl[0, tr.tokens[c1]] = 5.0
    stop_tok = (max(tr.tokens) + 1) % V
    if tr.children[c1]:
        c2 = tr.children[c1][0]
        tl[c1, tr.tokens[c2]] = 5.0
        tl[c2, stop_tok] = 5.0
        expect = [c1, c2]
    else:
        tl[c1, stop_tok] = 5.0
        expect = [c1]
    path, bonus = oe.accept_tree_greedy(tr, tl)
    if not any(tr.tokens[c] == stop_tok for c in tr.children[expect[-1]]):
        assert path == expect and bonus == stop_tok


def test_kv_compaction_equals_sequential_decode():
    tgt, head, wt, rf, rt, prompt = _setup(B=1)
    trees, _ = oe.build_tree(head, tgt.embed_w, tgt.norm_w, tgt.lm_head_w, rf, rt, tgt.lengths)
    tr = trees[0]
    L = 12
    ids = torch.tensor([tr.tokens])
    tgt.forward(ids, starts=torch.tensor([L]), positions=L + torch.tensor([tr.depth]),
                tree_mask=torch.tensor([tr.mask], dtype=torch.int64))
    # a deepest path
    leaf = max(range(len(tr.tokens)), key=lambda j: tr.depth[j])
    path, j = [], leaf
    while j > 0:
        path.append(j)
        j = tr.parent[j]
    path.reverse()
    oe.compact_kv(tgt.k_caches, tgt.v_caches, 0, L, path)
    seq = QwenOracle(TINY, wt, batch=1, max_seq=128, dtype=torch.float32)
    seq.forward(prompt)
    seq.lengths[:] = L
    seq.forward(torch.tensor([[tr.tokens[0]] + [tr.tokens[j] for j in path]]))
    a = len(path)
    for kc, sc in zip(tgt.k_caches, seq.k_caches):
        assert (kc[0, :, :L + a + 1] - sc[0, :, :L + a + 1]).abs().max().item() <= 1e-5


def _one_level_tree(children_tokens):
    """Root 0 with the given child tokens (draft-rank order), no deeper nodes."""
    n = len(children_tokens)
    return oe.Tree([0] + list(children_tokens), [-1] + [0] * n, [0] + [1] * n,
                   [1] + [1 | (1 << (i + 1)) for i in range(n)], [0] + [-1] * n,
                   [list(range(1, n + 1))] + [[] for _ in range(n)])


def _first_token(path, bonus, tree):
    return tree.tokens[path[0]] if path else bonus


def _chi2(counts, p):
    n = counts.sum()
    return (((counts - n * p) ** 2) / (n * p)).sum().item()


# chi-square thresholds at ~0.001 for V-1 degrees of freedom
CHI2_999 = {5: 20.5, 7: 24.3}


def _dists(V, seed):
    g = torch.Generator().manual_seed(seed)
    # skewed, unequal target and draft distributions over a tiny vocabulary
    pl = torch.randn(V, generator=g) * 1.5
    ql = torch.randn(V, generator=g) * 1.5
    return pl, ql, torch.softmax(pl, 0), torch.softmax(ql, 0), g


@pytest.mark.parametrize("k,seed", [(1, 1), (3, 2), (4, 3)])
def test_draft_rule_is_lossless_for_children_drawn_from_q(k, seed):
    """Recursive rejection sampling with k children drawn from q without
    replacement: the first emitted token (the accepted child, or the bonus
    from the residual p) is distributed as p (chi-square over 30000 trials)."""
    V = 6
    pl, ql, p, q, g = _dists(V, seed)
    n = 30000
    counts = torch.zeros(V)
    U = torch.rand(n, 2, k + 1, generator=g)
    for i in range(n):
        kids = torch.multinomial(q, k, replacement=False, generator=g).tolist()
        tr = _one_level_tree(kids)
        tl = pl.expand(k + 1, V)
        path, bonus = oe.accept_tree_rejection(tr, tl, ql.unsqueeze(0), U[i], topk=k, rule=oe.RULE_DRAFT)
        counts[_first_token(path, bonus, tr)] += 1
    assert _chi2(counts, p) < CHI2_999[V - 1]


@pytest.mark.parametrize("k,seed", [(1, 4), (3, 5), (4, 6)])
def test_target_rule_is_lossless_for_top_k_children(k, seed):
    """The target-only rule with the tree's deterministic top-k children of
    q: the first emitted token is distributed as p."""
    V = 8
    pl, ql, p, q, g = _dists(V, seed)
    kids = oe.topk_desc(ql, k).tolist()
    tr = _one_level_tree(kids)
    tl = pl.expand(k + 1, V)
    n = 30000
    counts = torch.zeros(V)
    U = torch.rand(n, 2, k + 1, generator=g)
    for i in range(n):
        path, bonus = oe.accept_tree_rejection(tr, tl, ql.unsqueeze(0), U[i], topk=k, rule=oe.RULE_TARGET)
        counts[_first_token(path, bonus, tr)] += 1
    assert _chi2(counts, p) < CHI2_999[V - 1]


def test_draft_rule_with_top_k_children_is_not_lossless():
    """Why the target-only rule exists: the draft rule assumes its children
    were drawn from q; with the tree's top-k children its output is biased
    away from p (here measurably, far beyond the chi-square bound)."""
    V, k = 6, 2
    pl, ql, p, q, g = _dists(V, 7)
    kids = oe.topk_desc(ql, k).tolist()
    tr = _one_level_tree(kids)
    n = 30000
    counts = torch.zeros(V)
    U = torch.rand(n, 2, k + 1, generator=g)
    for i in range(n):
        path, bonus = oe.accept_tree_rejection(tr, pl.expand(k + 1, V), ql.unsqueeze(0), U[i], topk=k)
        counts[_first_token(path, bonus, tr)] += 1
    assert _chi2(counts, p) > 10 * CHI2_999[V - 1]

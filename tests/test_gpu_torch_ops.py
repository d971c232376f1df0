"""``torch.ops.tsds`` on the GPU: each registered op against the oracle or a
torch reference of the same computation, called through the op layer (not
the engines).  The kernels behind the ops are the engines' kernels, covered
by the other GPU tests; these checks cover the op layer's argument plumbing
(shapes, strides, layouts, in-place arguments)."""
import os

import pytest
import torch

from oracle import eagle as oe
from oracle import qwen as oq
from oracle import spec as osp

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=1, vocab=1000)


@pytest.fixture(scope="module")
def tsds():
    import tri_sds_b200.torch_ops  # noqa: F401  (registers torch.ops.tsds)
    return torch.ops.tsds


def _bf(*shape, seed, std=1.0):
    return (torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16)


def test_qkv_rope_fused_matches_oracle_layer(tsds):
    s = oq.QwenShape(**SMALL)
    w = oq.random_qwen_weights(s, seed=0, std=0.05)
    B, T, S = 2, 5, 64
    ora = oq.QwenOracle(s, w, batch=B, max_seq=S)
    x = _bf(B, T, s.hidden, seed=1)
    starts = torch.tensor([3, 17])
    pos = starts[:, None] + torch.arange(T)[None]
    # oracle: the first half of QwenOracle.layer (norm, qkv, QK-norm, RoPE, cache write)
    L0 = w["layers"][0]
    xn = oq.rms_norm(x.reshape(B * T, -1), ora.norm1_w[0], s.eps).reshape(B, T, -1)
    qkv = xn @ ora.qkv_w_t[0]
    q = oq.rms_norm(qkv[..., :s.q_dim].reshape(B, T, s.n_heads, 128), ora.q_norm_w[0], s.eps).transpose(1, 2)
    k = oq.rms_norm(qkv[..., s.q_dim:s.q_dim + s.kv_dim].reshape(B, T, s.n_kv_heads, 128), ora.k_norm_w[0],
                    s.eps).transpose(1, 2)
    v = qkv[..., s.q_dim + s.kv_dim:].reshape(B, T, s.n_kv_heads, 128).transpose(1, 2)
    q_ref = oq.apply_rope(q, ora.cos, ora.sin, pos).transpose(1, 2).reshape(B * T, -1)
    k_ref = oq.apply_rope(k, ora.cos, ora.sin, pos)
    qkv_w = torch.cat([L0["q"], L0["k"], L0["v"]], 0).to(torch.bfloat16)
    kc = torch.zeros(B, s.n_kv_heads, S, 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    got = tsds.qkv_rope_fused(x.reshape(B * T, -1).to(DEV), L0["ln1"].to(DEV, torch.bfloat16), qkv_w.to(DEV),
                              L0["q_norm"].to(DEV, torch.bfloat16), L0["k_norm"].to(DEV, torch.bfloat16),
                              ora.cos.to(DEV), ora.sin.to(DEV), pos.reshape(-1).to(DEV, torch.int32),
                              starts.to(DEV, torch.int32), kc, vc, s.n_heads, s.n_kv_heads, s.eps)
    assert (got.cpu().float() - q_ref.float()).abs().max().item() <= 2e-2
    for b in range(B):
        st = int(starts[b])
        assert (kc[b, :, st:st + T].cpu().float() - k_ref[b].float()).abs().max().item() <= 2e-2
        assert (vc[b, :, st:st + T].cpu().float() - v[b].float()).abs().max().item() <= 2e-2


def test_verify_attention_op_matches_oracle(tsds):
    B, T, S, Hq, Hkv = 2, 5, 128, 16, 4
    q, kc, vc = _bf(B, T, Hq, 128, seed=2), _bf(B, Hkv, S, 128, seed=3), _bf(B, Hkv, S, 128, seed=4)
    st = torch.tensor([60, 71], dtype=torch.int32)
    got = tsds.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), None, 128).cpu()
    ref = oq.verify_attention(q.transpose(1, 2), kc, vc, st).transpose(1, 2)
    assert (got.float() - ref.float()).abs().max().item() <= 2e-2


def test_oproj_and_mlp_fused_match_torch(tsds):
    s = oq.QwenShape(**SMALL)
    w = oq.random_qwen_weights(s, seed=5, std=0.05)["layers"][0]
    M = 7
    x, attn = _bf(M, s.hidden, seed=6), _bf(M, s.q_dim, seed=7)
    o_w = w["o"].to(torch.bfloat16)
    got = tsds.oproj_fused(attn.to(DEV), o_w.to(DEV), x.to(DEV)).cpu().float()
    ref = (x.float() + (attn.float() @ o_w.float().T).to(torch.bfloat16).float()).to(torch.bfloat16).float()
    assert (got - ref).abs().max().item() <= 3e-2
    gu = torch.cat([w["gate"], w["up"]], 0).to(torch.bfloat16)
    dn = w["down"].to(torch.bfloat16)
    got = tsds.mlp_fused(x.to(DEV), w["ln2"].to(DEV, torch.bfloat16), gu.to(DEV), dn.to(DEV), s.eps).cpu().float()
    xn = oq.rms_norm(x, w["ln2"].to(torch.bfloat16), s.eps)
    g = xn @ gu.T
    h = torch.nn.functional.silu(g[:, :s.intermediate]) * g[:, s.intermediate:]
    ref = (x + h @ dn.T).float()
    assert (got - ref).abs().max().item() <= 3e-2


def test_lm_head_topk_op(tsds):
    N, V, M, k = 256, 1000, 6, 4
    x, norm_w, lm_w = _bf(M, N, seed=8), _bf(N, seed=9, std=0.1) + 1, _bf(V, N, seed=10, std=0.05)
    logits, vals, idx, lse = tsds.lm_head_topk(x.to(DEV), norm_w.to(DEV), lm_w.to(DEV), k, 1e-6)
    ref = (oq.rms_norm(x, norm_w) @ lm_w.T).float()
    lg = logits.cpu().float()
    assert (lg - ref).abs().max().item() <= 2e-2
    for m in range(M):
        assert idx[m].cpu().tolist() == oe.topk_desc(lg[m], k).tolist()
    assert torch.allclose(vals.cpu(), lg.gather(1, idx.cpu().long()))
    assert torch.allclose(lse.cpu(), torch.logsumexp(lg, 1), rtol=1e-5, atol=1e-5)


def test_eagle_fc_op(tsds):
    N, V, M = 256, 1000, 5
    feats, emb = _bf(M, N, seed=11), _bf(V, N, seed=12)
    fc_w, fc_b = _bf(N, 2 * N, seed=13, std=0.05), _bf(N, seed=14, std=0.1)
    ids = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(15))
    got = tsds.eagle_fc(feats.to(DEV), ids.to(DEV), emb.to(DEV), fc_w.to(DEV), fc_b.to(DEV)).cpu().float()
    x2 = torch.cat([feats, emb[ids]], -1)
    ref = ((x2 @ fc_w.T).float() + fc_b.float()).to(torch.bfloat16).float()
    assert (got - ref).abs().max().item() <= 3e-2


def test_accept_greedy_op(tsds):
    B, K = 4, 4
    g = torch.Generator().manual_seed(16)
    tgt = torch.randint(0, 50, (B, K + 1), generator=g)
    draft = tgt[:, :K].clone()
    draft[0, 0] += 1
    draft[1, 2] += 1
    draft[3, 3] += 1
    start = [10, 20, 30, 40]
    lengths = torch.tensor(start, dtype=torch.int32, device=DEV)
    last = torch.zeros(B, dtype=torch.int64, device=DEV)
    cur = torch.zeros(B, dtype=torch.int64, device=DEV)
    n, tokens = tsds.accept_greedy(draft.to(DEV), tgt.to(DEV), lengths, last, cur)
    n_ref, tok_ref = osp.greedy_accept(draft, tgt)
    assert n.cpu().tolist() == n_ref.tolist()
    assert torch.equal(tokens.cpu(), tok_ref)
    # each sequence commits its accepted drafts plus the bonus token
    assert lengths.cpu().tolist() == [L0 + int(a) + 1 for L0, a in zip(start, n_ref)]


def _random_trees(B, V, seed):
    """B trees built by the oracle's selection rules from random head logits;
    -> (trees, head logits [B*17, V] bf16, hrow [B, 26], children [B, 26, 4], ids [B, 26])."""
    g = torch.Generator().manual_seed(seed)
    trees, rows = [], []
    for b in range(B):
        tb = oe.TreeBuilder(int(torch.randint(0, V, (1,), generator=g)))
        hl = []
        while tb.frontier():
            lg = (torch.randn(len(tb.frontier()), V, generator=g) * 3).to(torch.bfloat16)
            hl.append(lg)
            tb.add_pass(lg)
        trees.append(tb.finish())
        rows.append(torch.cat(hl))
    R = rows[0].shape[0]
    head = torch.cat(rows)
    hrow = torch.tensor([[b * R + max(r, 0) for r in t.head_row] for b, t in enumerate(trees)], dtype=torch.int32)
    children = torch.full((B, 26, 4), -1, dtype=torch.int32)
    for b, t in enumerate(trees):
        for j, ch in enumerate(t.children):
            children[b, j, :len(ch)] = torch.tensor(ch, dtype=torch.int32)
    ids = torch.tensor([t.tokens for t in trees], dtype=torch.int64)
    return trees, head, hrow, children, ids, R


def test_accept_rejection_op_matches_oracle(tsds):
    B, V = 3, 1000
    trees, head, hrow, children, ids, R = _random_trees(B, V, seed=17)
    tl = (torch.randn(B * 26, V, generator=torch.Generator().manual_seed(18)) * 3).to(torch.bfloat16)
    U = torch.rand(B, 6, 5, generator=torch.Generator().manual_seed(19))
    path, acc, tokens, bonus = tsds.accept_rejection(tl.to(DEV), head.to(DEV), ids.to(DEV), hrow.to(DEV),
                                                     children.to(DEV), U.to(DEV), None, 5)
    for b in range(B):
        p_ref, bonus_ref = oe.accept_tree_rejection(trees[b], tl[b * 26:(b + 1) * 26].float(),
                                                    head[b * R:(b + 1) * R].float(), U[b])
        n = int(acc[b])
        assert n == len(p_ref) and path[b, :n].cpu().tolist() == p_ref
        assert int(bonus[b]) == bonus_ref and int(tokens[b, n]) == bonus_ref
        assert tokens[b, :n].cpu().tolist() == [trees[b].tokens[j] for j in p_ref]
    # greedy: uniforms None, the target's argmax per node
    am = tl.float().argmax(-1)
    path, acc, tokens, bonus = tsds.accept_rejection(tl.to(DEV), head.to(DEV), ids.to(DEV), hrow.to(DEV),
                                                     children.to(DEV), None, am.to(DEV), 5)
    for b in range(B):
        p_ref, bonus_ref = oe.accept_tree_greedy(trees[b], tl[b * 26:(b + 1) * 26].float())
        n = int(acc[b])
        assert n == len(p_ref) and path[b, :n].cpu().tolist() == p_ref and int(bonus[b]) == bonus_ref


def test_kv_compact_op_matches_oracle(tsds):
    layers, B, Hkv, S, N, NN, depth = 2, 2, 2, 64, 256, 26, 5
    kc, vc = _bf(layers, B, Hkv, S, 128, seed=20), _bf(layers, B, Hkv, S, 128, seed=21)
    hidden = _bf(B * NN, N, seed=22)
    lengths = torch.tensor([5, 30], dtype=torch.int32)
    path = torch.tensor([[2, 7, 11, -1, -1, -1], [-1] * 6], dtype=torch.int32)
    acc = torch.tensor([3, 0], dtype=torch.int32)
    kd, vd = kc.to(DEV), vc.to(DEV)
    ld = lengths.to(DEV)
    root = torch.zeros(B, N, dtype=torch.bfloat16, device=DEV)
    tsds.kv_compact(kd, vd, ld, path.to(DEV), acc.to(DEV), hidden.to(DEV), root, depth)
    kr, vr = [kc[i].clone() for i in range(layers)], [vc[i].clone() for i in range(layers)]
    for b in range(B):
        oe.compact_kv(kr, vr, b, int(lengths[b]), path[b, :int(acc[b])].tolist())
    assert torch.equal(kd.cpu(), torch.stack(kr)) and torch.equal(vd.cpu(), torch.stack(vr))
    assert ld.cpu().tolist() == [5 + 3 + 1, 30 + 0 + 1]
    assert torch.equal(root[0].cpu(), hidden[0 * NN + 11]) and torch.equal(root[1].cpu(), hidden[1 * NN + 0])

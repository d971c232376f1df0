"""EAGLE tree speculative decoding on the device vs the oracle (oracle/eagle.py):
tree selection, head logits, both acceptance rules over many uniform sets,
forced acceptance with the KV compaction checked row for row, and greedy
speculative decoding equal to autoregressive decoding."""
from dataclasses import replace

import pytest
import torch

from oracle import eagle as oe
from oracle import qwen as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)
NN, K, DEPTH = 26, 4, 5


def _setup(B=2, P=10, std=0.08, greedy=False, seed=0, rule=None, weights=None):
    from tri_sds_b200 import ops
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    oshape, dshape = oq.QwenShape(**SMALL), QwenShape(**SMALL)
    if weights is None:
        wt = oq.random_qwen_weights(oshape, seed=seed, std=std)
        we = oe.random_eagle_weights(oshape, seed=seed + 1, std=std)
    else:
        wt, we = weights
        oshape = replace(oshape, n_layers=len(wt["layers"]))
        dshape = replace(dshape, n_layers=len(wt["layers"]))
    tgt = QwenModel(dshape, batch=B, max_seq=128, max_rows=B * NN, device=DEV, weights=wt)
    head = EagleHead(tgt, B, weights=we)
    kw = {} if rule is None else {"rule": rule}
    eng = EagleEngine(tgt, head, greedy=greedy, use_graph=False, **kw)
    prompt = torch.randint(0, oshape.vocab, (B, P), generator=torch.Generator().manual_seed(seed + 2))
    return oshape, wt, we, tgt, head, eng, prompt


def _device_trees(eng, B, k=K):
    ids = eng.ids.view(B, NN).cpu()
    children = eng.children.view(B, NN, k).cpu()
    hrow = eng.hrow.view(B, NN).cpu()
    mask = eng.vmask.view(B, NN).cpu()
    return ids, children, hrow, mask


def _oracle_tree(ids, children, hrow, b):
    return oe.Tree(ids[b].tolist(), None, None, None, hrow[b].tolist(),
                   [[c for c in children[b, j].tolist() if c >= 0] for j in range(NN)])


def _mirror_weights(std=0.3, seed=40):
    """A one-layer target whose attention output is zeroed (O = 0), so a
    token's hidden state depends on the token alone, and a head that
    reproduces it: fc = [0 | I] passes the token embedding through, the
    head's layer is the target's.  The head's logits for a node's children
    are then the target's logits at that node, bit for bit (every GEMM's
    row result is independent of the row count), i.e. q = p."""
    shape = replace(oq.QwenShape(**SMALL), n_layers=1)
    wt = oq.random_qwen_weights(shape, seed=seed, std=std)
    L = wt["layers"][0]
    L["o"] = torch.zeros_like(L["o"])
    N = shape.hidden
    fc = torch.zeros(N, 2 * N, dtype=torch.bfloat16)
    fc[:, N:] = torch.eye(N, dtype=torch.bfloat16)
    we = {"fc": fc, "fc_bias": torch.zeros(N, dtype=torch.bfloat16), "layer": {k: v.clone() for k, v in L.items()}}
    return wt, we


def test_eagle_tree_selection_matches_oracle():
    """The device's tree equals the oracle's selection rules driven by the
    device's own head logits (pass by pass), exactly."""
    B, k = 2, K
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B)
    eng.prefill(prompt)
    eng.draw_uniforms()
    eng.plan.run()
    torch.cuda.synchronize()
    ids, children, hrow, mask = _device_trees(eng, B)
    hl = eng.head_logits.float().cpu()
    cur = eng.ids.view(B, NN)[:, 0].cpu()
    for b in range(B):
        tb = oe.TreeBuilder(int(cur[b]))
        d = 0
        while tb.frontier():
            T = len(tb.frontier())
            base = 0 if d == 0 else B * (1 + k * (d - 1))
            tb.add_pass(hl[base + b * T: base + (b + 1) * T])
            d += 1
        tr = tb.finish()
        assert ids[b].tolist() == tr.tokens
        assert mask[b].tolist() == tr.mask
        assert [[c for c in children[b, j].tolist() if c >= 0] for j in range(NN)] == tr.children


def test_eagle_head_logits_match_oracle():
    """The root pass of the head on the device vs the oracle head on the
    device's own inputs (root feature, current token): logits within 2e-2."""
    B = 2
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B)
    eng.prefill(prompt)
    eng.draw_uniforms()
    eng.plan.run()
    torch.cuda.synchronize()
    P = prompt.shape[1]
    ohead = oe.EagleHeadQwen(oshape, we, batch=B, max_pos=128)
    ora = oq.QwenOracle(oshape, wt, batch=B, max_seq=128)
    # the root feature the device used was its prefill's last hidden state
    hidden = tgt.prefill(prompt.to(DEV))[:, -1].cpu()
    cur = eng.ids.view(B, NN)[:, 0].cpu()
    f = ohead.forward(hidden.unsqueeze(1), ora.embed_w[cur].unsqueeze(1), torch.zeros(B, 1, dtype=torch.int64),
                      torch.full((B, 1), P), torch.ones(B, 1, dtype=torch.int64))
    ref = (oq.rms_norm(f[:, 0], ora.norm_w) @ ora.lm_head_w.T).float()
    got = eng.head_logits[:B].float().cpu()
    assert (got - ref).abs().max().item() <= 2e-2


@pytest.mark.parametrize("rule", [oe.RULE_DRAFT, oe.RULE_TARGET])
def test_accept_tree_kernel_matches_oracle_on_device_logits(rule):
    """The acceptance kernel as a function: the oracle, fed the device's tree,
    logits and uniforms, makes the same decisions - for both rules, over 128
    seeded uniform sets (two sequences x 64 sets) on one verified tree, and
    over three engine cycles."""
    from tri_sds_b200 import _lib, ops
    B = 2
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B, std=0.05, rule=rule)
    eng.prefill(prompt)
    for cycle in range(3):
        L = tgt.lengths.cpu().clone()
        U = torch.rand(B, DEPTH + 1, K + 1, generator=torch.Generator().manual_seed(10 + cycle))
        eng.step(U.to(DEV))
        torch.cuda.synchronize()
        ids, children, hrow, _ = _device_trees(eng, B)
        tl = eng.target_logits.view(B, NN, -1).float().cpu()
        hl = eng.head_logits.float().cpu()
        for b in range(B):
            path, bonus = oe.accept_tree_rejection(_oracle_tree(ids, children, hrow, b), tl[b], hl, U[b], rule=rule)
            n = int(eng.accept_len[b])
            assert n == len(path), (cycle, b, n, path)
            assert eng.path.view(B, DEPTH + 1)[b, :n].cpu().tolist() == path
            assert int(eng.tokens[b, n]) == bonus
            assert int(tgt.lengths[b]) == int(L[b]) + n + 1
    # many uniform sets on the last cycle's tree and logits (the kernel alone)
    ids, children, hrow, _ = _device_trees(eng, B)
    tl = eng.target_logits.view(B, NN, -1).float().cpu()
    hl = eng.head_logits.float().cpu()
    path = torch.empty(B, DEPTH + 1, dtype=torch.int32, device=DEV)
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    tokens = torch.empty(B, DEPTH + 2, dtype=torch.int64, device=DEV)
    cur = torch.empty(B, dtype=torch.int64, device=DEV)
    g = torch.Generator().manual_seed(99)
    for trial in range(64):
        U = torch.rand(B, DEPTH + 1, K + 1, generator=g)
        # sets of small uniforms make acceptance (and deep paths) likely
        if trial % 2:
            U = U * 1e-3
        Ud = U.to(DEV)
        _lib.call("tsds_accept_tree_rule", ops._p(eng.target_logits), None, ops._p(eng.head_logits),
                  ops._p(eng.ids), ops._p(eng.hrow), ops._p(eng.children), ops._p(Ud), rule, ops._p(path),
                  ops._p(acc), ops._p(tokens), ops._p(cur), B, NN - 1, oshape.vocab, K, DEPTH, ops._stream())
        torch.cuda.synchronize()
        for b in range(B):
            p_ref, bonus = oe.accept_tree_rejection(_oracle_tree(ids, children, hrow, b), tl[b], hl, U[b], rule=rule)
            n = int(acc[b])
            assert n == len(p_ref) and path[b, :n].cpu().tolist() == p_ref, (trial, b)
            assert int(tokens[b, n]) == bonus and int(cur[b]) == bonus, (trial, b)


@pytest.mark.parametrize("mode", ["greedy", "draft", "target"])
def test_forced_acceptance_compacts_the_kv_cache(mode):
    """q = p (a head mirroring a one-layer target): greedy and the draft rule
    accept at least the root's first child every cycle (the best-scored
    node of the tree, whose token is the target's argmax, and u q(x) < p(x)
    holds for any u < 1), the target rule accepts whenever u < p(x).  After
    each cycle the committed K/V rows equal the oracle's compaction
    (oracle.compact_kv) of the pre-commit cache, in every layer, row for
    row, and the committed length grew by accept_len + 1."""
    from tri_sds_b200.model import Plan
    B = 2
    rule = oe.RULE_TARGET if mode == "target" else oe.RULE_DRAFT
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B, greedy=mode == "greedy", rule=rule,
                                                    weights=_mirror_weights())
    eng.prefill(prompt)
    g = torch.Generator().manual_seed(5)
    total = 0
    for cycle in range(4):
        L = tgt.lengths.cpu().clone()
        U = torch.rand(B, DEPTH + 1, K + 1, generator=g) * (0.05 if mode == "target" else 1.0)
        if mode != "greedy":
            eng.draw_uniforms(U.to(DEV))
        calls = eng.plan.calls
        assert calls[-1][0] == "tsds_tree_commit"
        head_calls, tail = Plan(calls=calls[:-1]), Plan(calls=calls[-1:])
        head_calls.run()
        torch.cuda.synchronize()
        kc = [tgt.k_cache[i].cpu().clone() for i in range(tgt.k_cache.shape[0])]
        vc = [tgt.v_cache[i].cpu().clone() for i in range(tgt.v_cache.shape[0])]
        tail.run()
        torch.cuda.synchronize()
        tgt.check_status()
        acc = eng.accept_len.cpu()
        if mode != "target":
            assert (acc >= 1).all(), (cycle, acc)
        total += int(acc.sum())
        pth = eng.path.view(B, DEPTH + 1).cpu()
        for b in range(B):
            a = int(acc[b])
            oe.compact_kv(kc, vc, b, int(L[b]), pth[b, :a].tolist())
            assert int(tgt.lengths[b]) == int(L[b]) + a + 1
            for i in range(len(kc)):
                rows = slice(0, int(L[b]) + a + 1)
                assert torch.equal(tgt.k_cache[i, b, :, rows].cpu(), kc[i][b, :, rows]), (cycle, b, i)
                assert torch.equal(tgt.v_cache[i, b, :, rows].cpu(), vc[i][b, :, rows]), (cycle, b, i)
    assert total > 0


def test_eagle_greedy_equals_autoregressive():
    from tri_sds_b200.engine import AutoregressiveEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    B, n_new = 2, 20
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B, std=0.08, greedy=True)
    spec, acc = eng.generate(prompt, n_new)
    ar_model = QwenModel(QwenShape(**SMALL), batch=B, max_seq=128, max_rows=B, device=DEV, weights=wt)
    ar = AutoregressiveEngine(ar_model, use_graph=False).generate(prompt, n_new)
    # equal up to the first bf16 near-tie of the target's own logits
    for b in range(B):
        diff = (spec[b] != ar[b]).nonzero()
        if diff.numel() == 0:
            continue
        i = int(diff[0])
        ora = oq.QwenOracle(oshape, wt, batch=1, max_seq=128)
        lg, _ = ora.forward(torch.cat([prompt[b], ar[b, :i]]).unsqueeze(0))
        last = lg[0, -1].float()
        margin = abs((last[int(ar[b, i])] - last[int(spec[b, i])]).item())
        assert margin <= 2e-2, (b, i, margin)


def test_mirrored_head_greedy_spec_equals_autoregressive():
    """With q = p every greedy cycle accepts at least one draft token; the
    emitted tokens still equal greedy autoregressive decoding exactly."""
    from tri_sds_b200.engine import AutoregressiveEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    B, n_new = 2, 24
    wt, we = _mirror_weights()
    oshape, _, _, tgt, head, eng, prompt = _setup(B=B, greedy=True, weights=(wt, we))
    spec, acc = eng.generate(prompt, n_new)
    assert (acc >= 1).all(), acc
    ar_model = QwenModel(replace(QwenShape(**SMALL), n_layers=1), batch=B, max_seq=128, max_rows=B, device=DEV,
                         weights=wt)
    ar = AutoregressiveEngine(ar_model, use_graph=False).generate(prompt, n_new)
    assert torch.equal(spec, ar)

"""EAGLE tree speculative decoding on the device vs the oracle (oracle/eagle.py)."""
import pytest
import torch

from oracle import eagle as oe
from oracle import qwen as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)


def _setup(B=2, P=10, std=0.08, greedy=False, seed=0):
    from tri_sds_b200 import ops
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    oshape, dshape = oq.QwenShape(**SMALL), QwenShape(**SMALL)
    wt = oq.random_qwen_weights(oshape, seed=seed, std=std)
    we = oe.random_eagle_weights(oshape, seed=seed + 1, std=std)
    tgt = QwenModel(dshape, batch=B, max_seq=128, max_rows=B * 26, device=DEV, weights=wt)
    head = EagleHead(tgt, B, weights=we)
    eng = EagleEngine(tgt, head, greedy=greedy, use_graph=False)
    prompt = torch.randint(0, oshape.vocab, (B, P), generator=torch.Generator().manual_seed(seed + 2))
    return oshape, wt, we, tgt, head, eng, prompt


def _device_trees(eng, B, NN=26, k=4):
    ids = eng.ids.view(B, NN).cpu()
    children = eng.children.view(B, NN, k).cpu()
    hrow = eng.hrow.view(B, NN).cpu()
    mask = eng.vmask.view(B, NN).cpu()
    return ids, children, hrow, mask


def test_eagle_tree_selection_matches_oracle():
    """The device's tree equals the oracle's selection rules driven by the
    device's own head logits (pass by pass), exactly."""
    B, k = 2, 4
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B)
    eng.prefill(prompt)
    eng.draw_uniforms()
    eng.plan.run()
    torch.cuda.synchronize()
    ids, children, hrow, mask = _device_trees(eng, B)
    hl = eng.head_logits.float().cpu()
    cur = eng.ids.view(B, 26)[:, 0].cpu()
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
        assert [[c for c in children[b, j].tolist() if c >= 0] for j in range(26)] == tr.children


def test_eagle_head_logits_match_oracle():
    """The root pass of the head on the device vs the oracle head on the
    device's own inputs (root feature, current token): logits within 5e-2."""
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
    cur = eng.ids.view(B, 26)[:, 0].cpu()
    f = ohead.forward(hidden.unsqueeze(1), ora.embed_w[cur].unsqueeze(1), torch.zeros(B, 1, dtype=torch.int64),
                      torch.full((B, 1), P), torch.ones(B, 1, dtype=torch.int64))
    ref = (oq.rms_norm(f[:, 0], ora.norm_w) @ ora.lm_head_w.T).float()
    got = eng.head_logits[:B].float().cpu()
    assert (got - ref).abs().max().item() <= 5e-2


def test_accept_tree_kernel_matches_oracle_on_device_logits():
    """The acceptance kernel as a function: the oracle, fed the device's tree,
    logits and uniforms, makes the same decisions."""
    B = 2
    oshape, wt, we, tgt, head, eng, prompt = _setup(B=B, std=0.05)
    eng.prefill(prompt)
    for cycle in range(3):
        L = tgt.lengths.cpu().clone()
        U = torch.rand(B, 6, 5, generator=torch.Generator().manual_seed(10 + cycle))
        eng.step(U.to(DEV))
        torch.cuda.synchronize()
        ids, children, hrow, _ = _device_trees(eng, B)
        tl = eng.target_logits.view(B, 26, -1).float().cpu()
        hl = eng.head_logits.float().cpu()
        for b in range(B):
            tr = oe.Tree(ids[b].tolist(), None, None, None, hrow[b].tolist(),
                         [[c for c in children[b, j].tolist() if c >= 0] for j in range(26)])
            path, bonus = oe.accept_tree_rejection(tr, tl[b], hl, U[b])
            n = int(eng.accept_len[b])
            assert n == len(path), (cycle, b, n, path)
            assert eng.path.view(B, 6)[b, :n].cpu().tolist() == path
            assert int(eng.tokens[b, n]) == bonus
            assert int(tgt.lengths[b]) == int(L[b]) + n + 1


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

"""Paged KV (SGLang's token pool layout) on the GPU: the pooled entry points
against the contiguous ones on the same keys.

* tsds_verify_attention_paged: K/V scattered over [pool_rows, Hkv, D] pools
  through a request-to-token table (rows of the table in a shuffled request
  order, as SGLang's req_pool_indices give them) - one row per token (page 1,
  gathered rows) and 64-token pages (TMA tiles) - equals
  tsds_verify_attention over the contiguous caches bit for bit: causal and
  tree masks, one split and several (combine pass).
* tsds_qk_norm_rope_kv_paged writes q and the K/V rows exactly where the
  contiguous kernel writes them, only at the out_cache_loc pool rows.
* tsds_tree_commit_paged swaps table entries (no K/V moves) so the accepted
  nodes take the positions tsds_tree_commit moves their rows to, lists the
  kept pool rows and advances the lengths.
* A table entry outside the pool is never dereferenced: the call reports
  TSDS_E_INDEX through the status word.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
Hq, Hkv, D = 64, 8, 128


def _pool_from_cache(kc, vc, starts_hi, page, seed):
    """Scatter contiguous caches [B, Hkv, S, D] into pools with a random
    table: one random pool row per (sequence, position) for page 1, one
    random 64-row page per (sequence, 64 positions) otherwise."""
    B, _, S, _ = kc.shape
    g = torch.Generator().manual_seed(seed)
    if page == 1:
        rows = torch.randperm(B * S + 17, generator=g)[:B * S].reshape(B, S)
        pool_rows = B * S + 17
    else:
        npg = S // page
        pages = torch.randperm(B * npg + 3, generator=g)[:B * npg].reshape(B, npg)
        rows = (pages.unsqueeze(-1) * page + torch.arange(page)).reshape(B, S)
        pool_rows = (B * npg + 3) * page
    kp = torch.zeros(pool_rows, Hkv, D, dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    r = rows.to(DEV).reshape(-1)
    kp[r] = kc.permute(0, 2, 1, 3).reshape(B * S, Hkv, D)
    vp[r] = vc.permute(0, 2, 1, 3).reshape(B * S, Hkv, D)
    # the table's rows in a shuffled request order, with spare columns
    req = torch.randperm(B + 2, generator=g)[:B]
    table = torch.full((B + 2, S + 8), -7, dtype=torch.int32)
    table[req] = torch.cat([rows.to(torch.int32), torch.zeros(B, 8, dtype=torch.int32)], 1)
    return kp, vp, table.to(DEV), req.to(DEV)


@pytest.mark.parametrize("page", [1, 64])
@pytest.mark.parametrize("B,T,split,tree", [(1, 26, 1024, True), (4, 5, 1024, False), (2, 26, 128, True),
                                            (8, 5, 256, False)])
def test_paged_attention_equals_contiguous(page, B, T, split, tree):
    from tri_sds_b200 import ops
    S = 1024
    g = torch.Generator(device=DEV).manual_seed(B * 100 + T + page)
    kc = torch.randn(B, Hkv, S, D, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, D, device=DEV, generator=g).to(torch.bfloat16)
    q = torch.randn(B, T, Hq, D, device=DEV, generator=g).to(torch.bfloat16)
    starts = torch.randint(0, S - T, (B,), device=DEV, generator=g).to(torch.int32)
    mask = None
    if tree:
        # random ancestor masks: node t sees itself and a random subset of the earlier nodes
        bits = torch.randint(0, 2 ** 31, (B, T), device=DEV, generator=g).to(torch.int64)
        t = torch.arange(T, device=DEV)
        mask = ((bits & ((1 << t) - 1)) | (1 << t)).to(torch.int32)
    kp, vp, table, req = _pool_from_cache(kc, vc, S, page, seed=B + T)
    ref = ops.verify_attention(q, kc, vc, starts, tree_mask=mask, split_keys=split)
    got = ops.verify_attention_paged(q, kp, vp, starts, table, req_rows=req, page_size=page, tree_mask=mask,
                                     max_kv=S, split_keys=split)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(got, ref)


def test_paged_kv_write_equals_contiguous():
    from tri_sds_b200 import ops
    from tri_sds_b200.model import precompute_rope
    B, T, S = 4, 5, 256
    g = torch.Generator(device=DEV).manual_seed(5)
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * D, device=DEV, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    cos, sin = precompute_rope(D, S, 1e6, DEV)
    starts = torch.randint(0, S - T, (B,), device=DEV, generator=g).to(torch.int32)
    pos = (starts.unsqueeze(1) + torch.arange(T, device=DEV)).reshape(-1).to(torch.int32)
    kc = torch.zeros(B, Hkv, S, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q1 = torch.empty(B * T, Hq * D, dtype=torch.bfloat16, device=DEV)
    ops.qk_norm_rope_kv(qkv, qn, kn, cos, sin, pos, starts, q1, kc, vc, B, T, Hq, Hkv)
    pool_rows = 3 * B * T
    loc = torch.randperm(pool_rows, device=DEV, generator=g)[:B * T].to(torch.int64)
    kp = torch.zeros(pool_rows, Hkv, D, dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    q2 = torch.empty_like(q1)
    ops.qk_norm_rope_kv_paged(qkv, qn, kn, cos, sin, pos, loc, q2, kp, vp, Hq, Hkv)
    torch.cuda.synchronize()
    ops.check_status()
    assert torch.equal(q1, q2)
    for b in range(B):
        for t in range(T):
            r = int(loc[b * T + t])
            p = int(starts[b]) + t
            assert torch.equal(kp[r], kc[b, :, p]) and torch.equal(vp[r], vc[b, :, p])


def test_paged_tree_commit_moves_table_entries():
    import ctypes

    from tri_sds_b200 import _lib
    from tri_sds_b200.ops import _p
    B, depth, NN, N, ld = 3, 5, 26, 256, 64
    g = torch.Generator().manual_seed(9)
    table = torch.randint(0, 10_000, (B + 1, ld), generator=g).to(torch.int32)
    req = torch.tensor([2, 0, 3], dtype=torch.int64)
    lengths = torch.tensor([10, 0, 30], dtype=torch.int32)
    acc = torch.tensor([3, 0, 5], dtype=torch.int32)
    path = torch.zeros(B, depth + 1, dtype=torch.int32)
    path[0, :3] = torch.tensor([2, 7, 19])
    path[2, :5] = torch.tensor([1, 4, 5, 11, 25])
    hidden = torch.randn(B, NN, N, generator=g).to(torch.bfloat16)
    want = table.clone()
    kept_want = torch.full((B, depth + 2), -1, dtype=torch.int64)
    for b in range(B):
        row, L, a = int(req[b]), int(lengths[b]), int(acc[b])
        for j in range(a):
            fr, to = L + int(path[b, j]), L + 1 + j
            want[row, fr], want[row, to] = want[row, to].clone(), want[row, fr].clone()
        kept_want[b, :a + 1] = want[row, L:L + a + 1].to(torch.int64)
    d = {k: v.to(DEV) for k, v in dict(table=table, req=req, lengths=lengths, acc=acc, path=path,
                                        hidden=hidden).items()}
    kept = torch.zeros(B, depth + 2, dtype=torch.int64, device=DEV)
    root = torch.zeros(B, N, dtype=torch.bfloat16, device=DEV)
    st = _lib.load().tsds_tree_commit_paged(_p(d["table"]), ld, _p(d["req"]), _p(d["lengths"]), _p(d["path"]),
                                            _p(d["acc"]), depth, _p(kept), _p(d["hidden"]), NN - 1, N, _p(root),
                                            B, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(d["table"].cpu(), want)
    assert torch.equal(kept.cpu(), kept_want)
    assert torch.equal(d["lengths"].cpu(), lengths + acc + 1)
    for b in range(B):
        a = int(acc[b])
        last = int(path[b, a - 1]) if a > 0 else 0
        assert torch.equal(root[b].cpu(), hidden[b, last])


def test_paged_attention_reports_a_row_outside_the_pool():
    from tri_sds_b200 import _lib, ops
    B, T, S = 1, 5, 128
    g = torch.Generator(device=DEV).manual_seed(3)
    kc = torch.randn(B, Hkv, S, D, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(B, T, Hq, D, device=DEV, generator=g).to(torch.bfloat16)
    starts = torch.tensor([40], dtype=torch.int32, device=DEV)
    kp, vp, table, req = _pool_from_cache(kc, vc, S, 1, seed=1)
    table[int(req[0]), 17] = kp.shape[0] + 5   # a key below the sequence's end, past the pool
    ops.verify_attention_paged(q, kp, vp, starts, table, req_rows=req, page_size=1, max_kv=S)
    torch.cuda.synchronize()
    st = int(ops._scratch.status_word(q.device).item())
    ops._scratch.status_word(q.device).zero_()
    assert st == 10, _lib.load().tsds_status_string(st).decode()   # TSDS_E_INDEX


def _engines(page, weights, B, greedy, use_graph):
    """An EAGLE engine on a contiguous target and one on a paged target
    (scattered pool rows, shuffled table rows), same weights."""
    from dataclasses import replace

    from oracle import qwen as oq
    from tri_sds_b200 import ops
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.paged import PagedKV
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    wt, we = weights
    small = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=len(wt["layers"]),
                 vocab=1000)
    shape = QwenShape(**small)
    out = []
    for paged in (False, True):
        kv = PagedKV.allocate(shape.n_layers, B, 128, 2, 128, DEV, page_size=page, seed=page) if paged else None
        tgt = QwenModel(shape, batch=B, max_seq=128, max_rows=B * 26, device=DEV, weights=wt, kv=kv)
        head = EagleHead(tgt, B, weights=we)
        out.append(EagleEngine(tgt, head, greedy=greedy, use_graph=use_graph))
    return oq.QwenShape(**small), out


@pytest.mark.parametrize("page,greedy,use_graph,mirror", [(1, False, False, True), (64, False, True, True),
                                                          (1, True, True, True), (1, False, True, False),
                                                          (64, True, False, False)])
def test_eagle_on_paged_kv_equals_contiguous(page, greedy, use_graph, mirror):
    """The whole EAGLE cycle with the target's KV in token pools (the table
    rewritten at every commit instead of K/V rows moved) emits the same
    tokens and accept lengths as the contiguous cache, cycle for cycle, and
    the committed positions hold the same K/V: with acceptance forced above
    zero (a head mirroring a one-layer target whose attention output is
    zeroed), and with random two-layer weights (attention in play)."""
    import sys
    sys.path.insert(0, __file__.rsplit("/", 1)[0])
    from oracle import eagle as oe
    from oracle import qwen as oq
    from test_gpu_eagle import SMALL, _mirror_weights
    B, P = 2, 10
    if mirror:
        weights = _mirror_weights()
    else:
        shape = oq.QwenShape(**SMALL)
        weights = (oq.random_qwen_weights(shape, seed=3, std=0.08), oe.random_eagle_weights(shape, seed=4, std=0.08))
    oshape, (ref, pag) = _engines(page, weights, B, greedy, use_graph)
    prompt = torch.randint(0, oshape.vocab, (B, P), generator=torch.Generator().manual_seed(7))
    for eng in (ref, pag):
        eng.prepare(prompt)
    g = torch.Generator().manual_seed(8)
    total = 0
    for cycle in range(6):
        U = (torch.rand(B, 6, 5, generator=g) * 0.05).to(DEV)
        outs = []
        for eng in (ref, pag):
            toks, acc = eng.step(None if greedy else U)
            torch.cuda.synchronize()
            outs.append((toks.clone(), acc.clone()))
        ref.target.check_status()
        pag.target.check_status()
        assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1]), cycle
        total += int(outs[0][1].sum())
        assert torch.equal(ref.target.lengths, pag.target.lengths)
    assert total > 0 or not mirror
    kv = pag.target.kv
    for b in range(B):
        n = int(ref.target.lengths[b])
        for layer in range(len(kv.k_pools)):
            k, v = kv.gather(layer, b, n)
            assert torch.equal(k, ref.target.k_cache[layer, b, :, :n]), (b, layer)
            assert torch.equal(v, ref.target.v_cache[layer, b, :, :n]), (b, layer)
    # the kept rows of the last commit are the table's entries at the committed positions
    kept = pag.kept_rows.cpu()
    for b in range(B):
        a = int(outs[1][1][b])
        n = int(pag.target.lengths[b])
        req = int(kv.req_rows[b])
        assert kept[b, :a + 1].tolist() == kv.table[req, n - a - 1:n].cpu().long().tolist()


def test_chain_spec_on_paged_kv_equals_contiguous():
    """The chain engine (a one-layer draft, K=4 greedy) with the target's KV
    in token pools (one row per token, scattered) emits what it emits on the
    contiguous cache, and greedy autoregressive decoding on the paged target
    emits the same tokens: the commit of a chain is a length update, the
    rejected rows' table entries are rewritten by the next forward."""
    from oracle import qwen as oq
    from tri_sds_b200 import ops
    from tri_sds_b200.engine import AutoregressiveEngine, SpecEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.paged import PagedKV
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    small = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)
    wt = oq.random_qwen_weights(oq.QwenShape(**small), seed=3, std=0.08)
    wd = {**wt, "layers": wt["layers"][:1]}
    B, P, K, n_new = 2, 9, 4, 24
    prompt = torch.randint(0, small["vocab"], (B, P), generator=torch.Generator().manual_seed(4))
    outs = []
    for paged in (False, True):
        kv = PagedKV.allocate(2, B, 128, 2, 128, DEV, page_size=1, seed=6) if paged else None
        tgt = QwenModel(QwenShape(**small), batch=B, max_seq=128, max_rows=B * (K + 1), device=DEV, weights=wt,
                        kv=kv)
        drf = QwenModel(QwenShape(**{**small, "n_layers": 1}), batch=B, max_seq=128, max_rows=B * 2, device=DEV,
                        weights=wd)
        outs.append(SpecEngine(tgt, drf, K).generate(prompt, n_new)[0])
    assert torch.equal(outs[0], outs[1])
    kv = PagedKV.allocate(2, B, 128, 2, 128, DEV, page_size=64, seed=7)
    ar_model = QwenModel(QwenShape(**small), batch=B, max_seq=128, max_rows=B, device=DEV, weights=wt, kv=kv)
    ar = AutoregressiveEngine(ar_model).generate(prompt, n_new)
    assert torch.equal(outs[1], ar)

"""The tcgen05 variant of verify attention (tsds_set_attention_tc) on the GPU.

Against the fp32 torch reference of the same op and against the default
kernel, for causal and tree masks, one and two 128-row query blocks, single
splits that run the online softmax over many 128-key tiles (no combine pass),
many short splits (with the combine pass), splits past the last key, and the
32B-shape verify configurations (B=8 over 4096 keys; the EAGLE tree, 26 rows
per sequence x 8 q heads per kv head), and the prompt prefill on it."""

import pytest
import torch

from oracle import qwen as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2


@pytest.fixture()
def ops():
    from tri_sds_b200 import ops as _ops
    _ops.set_attention_tc(True)
    assert _ops.attention_tc()
    yield _ops
    _ops.set_attention_tc(False)


def _case(B, T, Hq, Hkv, S, starts, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hq, 128, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, 128, generator=g).to(torch.bfloat16)
    return q, kc, vc, torch.tensor(starts, dtype=torch.int32)


def _ref_f32(q, kc, vc, starts, tree_mask=None, mask_origin=-1):
    """softmax(q k^T / sqrt(D)) v over the visible keys, in fp32."""
    B, T, Hq, D = q.shape
    G = Hq // kc.shape[1]
    out = torch.zeros(B, T, Hq, D)
    for b in range(B):
        st = int(starts[b])
        L = st + T
        base = st if mask_origin < 0 else mask_origin
        k = kc[b, :, :L].float().repeat_interleave(G, 0)
        v = vc[b, :, :L].float().repeat_interleave(G, 0)
        s = torch.einsum("thd,hkd->thk", q[b].float(), k) * D ** -0.5
        key = torch.arange(L)
        for t in range(T):
            if tree_mask is None:
                vis = key <= st + t
            else:
                rel = key - base
                bits = (int(tree_mask[b, t]) & 0xFFFFFFFF) >> rel.clamp(0, 31)
                vis = (rel < 0) | ((rel < 32) & ((bits & 1) == 1))
            s[t, :, ~vis] = float("-inf")
        out[b] = torch.einsum("thk,hkd->thd", torch.softmax(s, -1), v)
    return out


def _run(ops, q, kc, vc, st, **kw):
    out = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), **kw)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("split_keys", [128, 256, 512, 4096])
@pytest.mark.parametrize("B,T,starts,S", [(1, 5, [4091], 4096), (2, 5, [100, 517], 1024), (3, 1, [0, 63, 64], 256),
                                          (1, 16, [300], 512), (2, 5, [0, 1], 128)])
def test_tc_attention_vs_f32(ops, B, T, starts, S, split_keys):
    q, kc, vc, st = _case(B, T, 64, 8, S, starts)
    got = _run(ops, q, kc, vc, st, split_keys=min(split_keys, S)).cpu().float()
    assert (got - _ref_f32(q, kc, vc, st)).abs().max().item() <= TOL


@pytest.mark.parametrize("split_keys", [128, 512])
def test_tc_attention_kv4096_b8(ops, split_keys):
    """The isolated verify-attention configuration at its largest batch."""
    B, T, S = 8, 5, 4096
    q, kc, vc, st = _case(B, T, 64, 8, S, [S - T] * B, seed=13)
    got = _run(ops, q, kc, vc, st, split_keys=split_keys).cpu().float()
    assert (got - _ref_f32(q, kc, vc, st)).abs().max().item() <= TOL


@pytest.mark.parametrize("split_keys", [128, 1024])
def test_tc_attention_eagle_tree_rows(ops, split_keys):
    """26 tree nodes x 8 q heads = 208 query rows per kv head (two 128-row
    blocks), masks anchored at mask_origin, a 512-token prompt."""
    B, T, S, start = 2, 26, 1024, 512
    q, kc, vc, st = _case(B, T, 64, 8, S, [start, start + 37], seed=21)
    g = torch.Generator().manual_seed(4)
    parent = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, T)]
    masks = []
    for t in range(T):
        m, j = 0, t
        while j >= 0:
            m |= 1 << j
            j = parent[j]
        masks.append(m)
    tm = torch.tensor([masks] * B, dtype=torch.int64).to(torch.int32)
    got = _run(ops, q, kc, vc, st, tree_mask=tm, split_keys=split_keys).cpu().float()
    assert (got - _ref_f32(q, kc, vc, st, tree_mask=tm)).abs().max().item() <= TOL


def test_tc_attention_vs_oracle(ops):
    """Against the reference's own path (repeat_interleave + SDPA with its mask)."""
    B, T, S = 2, 5, 128
    q, kc, vc, st = _case(B, T, 16, 4, S, [60, 60], seed=5)
    got = _run(ops, q, kc, vc, st).cpu()
    ref = oq.verify_attention(q.transpose(1, 2), kc, vc, st).transpose(1, 2)
    assert (got.float() - ref.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("split_keys", [128, 2048])
def test_tc_attention_decode_equals_verify_bitwise(ops, split_keys):
    """A query's output does not depend on how many tokens share the call."""
    B, T, S = 2, 5, 2048
    q, kc, vc, st = _case(B, T, 64, 8, S, [1500, 700], seed=9)
    qd, kd, vd, sd = q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV)
    full = ops.verify_attention(qd, kd, vd, sd, split_keys=split_keys)
    for t in range(T):
        one = ops.verify_attention(qd[:, t:t + 1].contiguous(), kd, vd, sd + t, split_keys=split_keys)
        assert torch.equal(one[:, 0], full[:, t]), t


def test_tc_attention_chain_mask_equals_causal(ops):
    B, T, S = 2, 7, 512
    q, kc, vc, st = _case(B, T, 64, 8, S, [200, 333], seed=11)
    chain = torch.tensor([[(1 << (t + 1)) - 1 for t in range(T)]] * B, dtype=torch.int32)
    a = _run(ops, q, kc, vc, st)
    b = _run(ops, q, kc, vc, st, tree_mask=chain)
    assert torch.equal(a, b)


def test_tc_attention_close_to_default_kernel(ops):
    B, T, S = 2, 5, 1024
    q, kc, vc, st = _case(B, T, 64, 8, S, [900, 17], seed=3)
    tc = _run(ops, q, kc, vc, st).cpu().float()
    ops.set_attention_tc(False)
    ref = _run(ops, q, kc, vc, st).cpu().float()
    ops.set_attention_tc(True)
    assert (tc - ref).abs().max().item() <= TOL


def _tree_masks(B, T, seed):
    g = torch.Generator().manual_seed(seed)
    parent = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, T)]
    masks = []
    for t in range(T):
        m, j = 0, t
        while j >= 0:
            m |= 1 << j
            j = parent[j]
        masks.append(m)
    return torch.tensor([masks] * B, dtype=torch.int64).to(torch.int32)


@pytest.mark.parametrize("B,T,starts,S,tree", [(1, 26, [512], 1024, True), (2, 26, [300, 700], 896, True),
                                               (2, 5, [100, 517], 640, False), (3, 1, [0, 63, 200], 256, False)])
def test_tc_cluster_combine_equals_combine_pass(ops, B, T, starts, S, tree):
    """Mode 2: the 2 to 8 key splits of a row block as one cluster, combined
    through distributed shared memory - the same bits as the combine pass."""
    q, kc, vc, st = _case(B, T, 64, 8, S, starts, seed=S + T)
    tm = _tree_masks(B, T, seed=T) if tree else None
    one = _run(ops, q, kc, vc, st, tree_mask=tm)
    ops.set_attention_tc(2)
    two = _run(ops, q, kc, vc, st, tree_mask=tm)
    ops.set_attention_tc(1)
    assert torch.equal(one, two)
    assert (two.cpu().float() - _ref_f32(q, kc, vc, st, tree_mask=tm)).abs().max().item() <= TOL


@pytest.mark.parametrize("B,P,Hq", [(1, 512, 16), (2, 300, 8)])
def test_tc_prefill_attention_matches_f32(ops, B, P, Hq):
    """The prompt prefill's attention call (every prompt row of the batch,
    causal from row 0, one split of the whole prompt) against the fp32
    reference."""
    q, kc, vc, st = _case(B, P, Hq, 2, P + 64, [0] * B, seed=P)
    got = _run(ops, q, kc, vc, st, max_kv=P, split_keys=(P + 127) // 128 * 128)
    assert (got.cpu().float() - _ref_f32(q, kc, vc, st)).abs().max().item() <= TOL


@pytest.mark.parametrize("B,P", [(1, 512), (2, 300)])
def test_tc_prefill_matches_sdpa(ops, B, P):
    """Prompt prefill with its attention on the tcgen05 kernel against the
    same prefill on SDPA: layer 0's K/V cache (written before any attention)
    equal, and the final logits as close to the fp32 oracle's as SDPA's are
    (two bf16 attention implementations round P differently, and two layers
    of random weights carry that into the logits by a few bf16 ulps either
    way), with the argmax equal wherever the oracle's top two are apart."""
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    kw = dict(hidden=512, n_heads=16, n_kv_heads=2, head_dim=128, intermediate=1024, n_layers=2, vocab=1000)
    oshape = oq.QwenShape(**kw)
    w = oq.random_qwen_weights(oshape, seed=P, std=0.05)
    m = QwenModel(QwenShape(**kw), batch=B, max_seq=P + 64, max_rows=B * 5, device=DEV, weights=w)
    prompt = torch.randint(0, kw["vocab"], (B, P), generator=torch.Generator().manual_seed(B))
    h_tc = m.prefill(prompt)
    lg_tc = m.logits_of(h_tc.reshape(-1, kw["hidden"])).float().cpu()
    k0_tc = m.k_cache[0].clone()
    ops.set_attention_tc(False)
    h_ref = m.prefill(prompt)
    lg_sdpa = m.logits_of(h_ref.reshape(-1, kw["hidden"])).float().cpu()
    ops.set_attention_tc(True)
    assert torch.equal(k0_tc, m.k_cache[0])
    ora = oq.QwenOracle(oshape, w, batch=B, max_seq=P + 64, dtype=torch.float32)
    lg_f32, _ = ora.forward(prompt)
    lg_f32 = lg_f32.float().reshape(B * P, -1)
    err_tc = (lg_tc - lg_f32).abs().max().item()
    err_sdpa = (lg_sdpa - lg_f32).abs().max().item()
    assert err_tc <= 1.5 * err_sdpa + 1e-2, (err_tc, err_sdpa)
    top2 = lg_f32.topk(2, -1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * err_sdpa + 2e-2
    assert torch.equal(lg_tc.argmax(-1)[clear], lg_f32.argmax(-1)[clear])


def test_tc_attention_in_the_model(ops):
    """EAGLE greedy decoding with the tcgen05 attention equals greedy
    autoregressive decoding (small shape), up to bf16 near-ties of the
    target's own logits."""
    from oracle import eagle as oe
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.engine import AutoregressiveEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    kw = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)
    B, n_new = 2, 20
    oshape, shape = oq.QwenShape(**kw), QwenShape(**kw)
    wt = oq.random_qwen_weights(oshape, seed=0, std=0.08)
    we = oe.random_eagle_weights(oshape, seed=1, std=0.08)
    prompt = torch.randint(0, oshape.vocab, (B, 10), generator=torch.Generator().manual_seed(2))
    ops.set_attention_tc(2)   # with the clustered combine (max_seq 256: two splits)
    tgt = QwenModel(shape, batch=B, max_seq=256, max_rows=B * 26, device=DEV, weights=wt)
    eng = EagleEngine(tgt, EagleHead(tgt, B, weights=we), greedy=True)
    spec, _ = eng.generate(prompt, n_new)
    ar = AutoregressiveEngine(QwenModel(shape, batch=B, max_seq=256, max_rows=B, device=DEV, weights=wt)).generate(
        prompt, n_new)
    for b in range(B):
        diff = (spec[b] != ar[b]).nonzero()
        if diff.numel() == 0:
            continue
        i = int(diff[0])
        ora = oq.QwenOracle(oshape, wt, batch=1, max_seq=256)
        lg, _ = ora.forward(torch.cat([prompt[b], ar[b, :i]]).unsqueeze(0))
        last = lg[0, -1].float()
        assert abs((last[int(ar[b, i])] - last[int(spec[b, i])]).item()) <= 2e-2, (b, i)

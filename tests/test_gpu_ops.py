"""GPU parity of each C-ABI op against the CPU oracle / a torch fp32 reference."""
import pytest
import torch

from oracle import qwen as oq

pytestmark = pytest.mark.gpu

DEV = "cuda"


# tcgen05 accumulates in fp32 inside the tensor core with truncating
# alignment (like cuBLAS): allow one more bf16 ulp and a small absolute term
# than for the fp32-FMA paths.
TC_SLACK = {"ulps": 1.0, "abs": 2e-3}
LINEAR_PATH = {"name": "gemv"}


def _ulp_close(got: torch.Tensor, ref: torch.Tensor, ulps: float = 1.0, frac_exact: float = 0.98):
    """bf16 tensors agree to `ulps` bf16 ulps everywhere, and mostly exactly."""
    g, r = got.float().cpu(), ref.float().cpu()
    ulp = torch.clamp(r.abs(), min=1e-30) * 2.0 ** -7
    tc = LINEAR_PATH["name"] == "tcgen05"
    extra_ulps, extra_abs = (TC_SLACK["ulps"], TC_SLACK["abs"]) if tc else (0.0, 0.0)
    bad = (g - r).abs() > (ulps + extra_ulps) * ulp + 1e-6 + extra_abs
    assert not bad.any(), f"{int(bad.sum())} elements beyond {ulps} ulp; max abs diff {(g - r).abs().max().item()}"
    exact = (g == r).float().mean().item()
    assert exact >= frac_exact, exact


@pytest.fixture(scope="module", params=["gemv", "tcgen05"])
def ops(request):
    """Every op test runs with the linear layers / LM head on the CUDA-core
    GEMV (rows <= 8) and on the tcgen05 GEMM."""
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(8 if request.param == "gemv" else 0)
    LINEAR_PATH["name"] = request.param
    yield _ops
    LINEAR_PATH["name"] = "gemv"
    _ops.set_gemv_max_rows(0)


def test_rms_norm(ops):
    g = torch.Generator().manual_seed(0)
    for rows, n in [(1, 2560), (5, 5120), (40, 2560), (3, 128)]:
        x = torch.randn(rows, n, generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16)
        got = ops.rms_norm(x.to(DEV), w.to(DEV))
        _ulp_close(got, oq.rms_norm(x, w))


@pytest.mark.parametrize("M", [1, 2, 5, 8, 13, 40])
def test_linear_family(ops, M):
    g = torch.Generator().manual_seed(M)
    K, n_out = 2560, 768
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * n_out, K, generator=g)).to(torch.bfloat16)
    res = torch.randn(M, n_out, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.float().T   # fp32 reference of the same op
    got = ops.linear(x.to(DEV), w[:n_out].contiguous().to(DEV)).cpu().float()
    assert (got - ref[:, :n_out]).abs().max() <= 2e-2 * ref.abs().max()
    _ulp_close(got, ref[:, :n_out].to(torch.bfloat16), ulps=1.0, frac_exact=0.95)
    got_r = ops.linear_residual(x.to(DEV), w[:n_out].contiguous().to(DEV), res.to(DEV)).cpu().float()
    ref_r = (res.float() + ref[:, :n_out].to(torch.bfloat16).float()).to(torch.bfloat16).float()
    # one bf16 ulp of the product may move the sum by that much (cancellation)
    # plus the rounding of the sum itself
    tol = (ref[:, :n_out].abs() + ref_r.abs()) * 2.0 ** -7 + 1e-6
    if LINEAR_PATH["name"] == "tcgen05":
        tol = tol * 2 + TC_SLACK["abs"]
    assert ((got_r - ref_r).abs() <= tol).all()
    assert (got_r == ref_r).float().mean() >= 0.9
    got_s = ops.linear_swiglu(x.to(DEV), w.to(DEV)).cpu()
    gte, up = ref[:, :n_out].to(torch.bfloat16), ref[:, n_out:].to(torch.bfloat16)
    ref_s = torch.nn.functional.silu(gte) * up
    _ulp_close(got_s, ref_s, ulps=2.0, frac_exact=0.9)


def test_reference_named_wrappers(ops):
    """fused_qwen_decode.py names, reference [in, out] weight layout."""
    g = torch.Generator().manual_seed(7)
    B, N, I = 3, 512, 1024
    x = torch.randn(B, N, generator=g).to(torch.bfloat16)
    w_gu_t = (0.05 * torch.randn(N, 2 * I, generator=g)).to(torch.bfloat16)   # [in, out] like gate_up_w_t
    w_d_t = (0.05 * torch.randn(I, N, generator=g)).to(torch.bfloat16)
    h = ops.fused_gateup_silu(x.to(DEV), w_gu_t.to(DEV)).cpu()
    gu = (x.float() @ w_gu_t.float()).to(torch.bfloat16)
    _ulp_close(h, torch.nn.functional.silu(gu[:, :I]) * gu[:, I:], ulps=2.0, frac_exact=0.9)
    y = ops.fused_down_residual(h.to(DEV), w_d_t.to(DEV), x.to(DEV)).cpu()
    _ulp_close(y, (x.float() + (h.float() @ w_d_t.float()).to(torch.bfloat16).float()).to(torch.bfloat16),
               ulps=1.0, frac_exact=0.9)


def test_qk_norm_rope_kv(ops):
    g = torch.Generator().manual_seed(3)
    B, T, Hq, Hkv, D, S = 2, 5, 8, 2, 128, 64
    qkv = torch.randn(B * T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    cos, sin = oq.precompute_rope(D, S, 1e6, torch.bfloat16)
    starts = torch.tensor([7, 20], dtype=torch.int32)
    pos = (starts.unsqueeze(1) + torch.arange(T)).reshape(-1).to(torch.int32)
    kc = torch.zeros(B, Hkv, S, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B * T, Hq * D, dtype=torch.bfloat16, device=DEV)
    ops.qk_norm_rope_kv(qkv.to(DEV), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV), pos.to(DEV),
                        starts.to(DEV), q_out, kc, vc, B, T, Hq, Hkv)
    q = oq.rms_norm(qkv[:, :Hq * D].reshape(B, T, Hq, D), qn).transpose(1, 2)
    k = oq.rms_norm(qkv[:, Hq * D:(Hq + Hkv) * D].reshape(B, T, Hkv, D), kn).transpose(1, 2)
    v = qkv[:, (Hq + Hkv) * D:].reshape(B, T, Hkv, D).transpose(1, 2)
    pos2 = pos.reshape(B, T).long()
    q = oq.apply_rope(q, cos, sin, pos2).transpose(1, 2).reshape(B * T, Hq * D)
    k = oq.apply_rope(k, cos, sin, pos2)
    _ulp_close(q_out, q, ulps=1.0, frac_exact=0.97)
    for b in range(B):
        s0 = int(starts[b])
        _ulp_close(kc[b, :, s0:s0 + T], k[b], ulps=1.0, frac_exact=0.97)
        assert torch.equal(vc[b, :, s0:s0 + T].cpu(), v[b])
    assert kc[0, :, :7].abs().sum().item() == 0  # rows outside the new tokens untouched


def _attn_case(B, T, Hq, Hkv, S, starts, seed=0):
    g = torch.Generator().manual_seed(seed)
    D = 128
    q = torch.randn(B, T, Hq, D, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    return q, kc, vc, torch.tensor(starts, dtype=torch.int32)


def _attn_ref_f32(q, kc, vc, starts, tree_mask=None):
    """fp32 torch reference: softmax(q k^T / sqrt(D)) v over the visible keys."""
    B, T, Hq, D = q.shape
    G = Hq // kc.shape[1]
    out = torch.zeros(B, T, Hq, D)
    for b in range(B):
        st = int(starts[b])
        L = st + T
        k = kc[b, :, :L].float().repeat_interleave(G, 0)
        v = vc[b, :, :L].float().repeat_interleave(G, 0)
        s = torch.einsum("thd,hkd->thk", q[b].float(), k) * D ** -0.5
        key = torch.arange(L)
        for t in range(T):
            if tree_mask is None:
                vis = key <= st + t
            else:
                rel = (key - st).clamp(min=0)
                vis = (key < st) | (((int(tree_mask[b, t]) >> rel) & 1) == 1)
            s[t, :, ~vis] = float("-inf")
        out[b] = torch.einsum("thk,hkd->thd", torch.softmax(s, -1), v)
    return out


@pytest.mark.parametrize("B,T,starts,S", [(1, 5, [4091], 4096), (2, 5, [100, 517], 1024), (3, 1, [0, 63, 64], 256),
                                          (1, 16, [300], 512), (2, 5, [0, 1], 64)])
def test_verify_attention_vs_f32(ops, B, T, starts, S):
    q, kc, vc, st = _attn_case(B, T, 64, 8, S, starts)
    got = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV)).cpu().float()
    ref = _attn_ref_f32(q, kc, vc, st)
    assert (got - ref).abs().max().item() <= 1e-2


@pytest.mark.parametrize("split_keys", [1024, 512, 256, 128, 64])
def test_verify_attention_kv4096_b8(ops, split_keys):
    """The isolated verify-attention configuration at its largest batch: B=8,
    KV length 4096, 5 new tokens, 64/8 heads.  128-key splits give 32 splits
    (the combine pass's batched-load path at its limit), 64-key splits 64
    (its streaming path)."""
    B, T, S = 8, 5, 4096
    q, kc, vc, st = _attn_case(B, T, 64, 8, S, [S - T] * B, seed=13)
    got = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), split_keys=split_keys).cpu().float()
    ref = _attn_ref_f32(q, kc, vc, st)
    assert (got - ref).abs().max().item() <= 1e-2


def test_verify_attention_vs_oracle(ops):
    """Against the reference's own path (repeat_interleave + SDPA with its mask)."""
    B, T, S = 2, 5, 128
    q, kc, vc, st = _attn_case(B, T, 16, 4, S, [60, 60], seed=5)
    got = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV)).cpu()
    ref = oq.verify_attention(q.transpose(1, 2), kc, vc, st).transpose(1, 2)
    assert (got.float() - ref.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("split_keys", [128, 512, 64])
def test_verify_attention_decode_equals_verify_bitwise(ops, split_keys):
    """A query's output does not depend on how many tokens share the call
    (its row block, the grid, the number of splits in use)."""
    B, T, S = 2, 5, 2048
    q, kc, vc, st = _attn_case(B, T, 64, 8, S, [1500, 700], seed=9)
    qd, kd, vd, sd = q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV)
    full = ops.verify_attention(qd, kd, vd, sd, split_keys=split_keys)
    for t in range(T):
        one = ops.verify_attention(qd[:, t:t + 1].contiguous(), kd, vd, sd + t, split_keys=split_keys)
        assert torch.equal(one[:, 0], full[:, t]), t


@pytest.mark.parametrize("split_keys", [128, 256])
def test_verify_attention_tree_rows_32b_heads(ops, split_keys):
    """The EAGLE tree verify's shape: 26 rows per sequence x 8 q heads per kv
    head (208 rows, several row blocks), a branching tree mask, 32B heads."""
    B, T, S = 2, 26, 1024
    q, kc, vc, st = _attn_case(B, T, 64, 8, S, [512, 700], seed=21)
    g = torch.Generator().manual_seed(22)
    parent = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, T)]
    masks = []
    for t in range(T):
        m, j = 0, t
        while j >= 0:
            m |= 1 << j
            j = parent[j]
        masks.append(m)
    tm = torch.tensor([masks] * B, dtype=torch.int64).to(torch.int32)
    got = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), tree_mask=tm.to(DEV),
                               split_keys=split_keys).cpu().float()
    ref = _attn_ref_f32(q, kc, vc, st, tree_mask=tm)
    assert (got - ref).abs().max().item() <= 1e-2


def test_verify_attention_tree_mask(ops):
    B, T, S = 2, 7, 512
    q, kc, vc, st = _attn_case(B, T, 64, 8, S, [200, 333], seed=11)
    # chain-shaped mask == causal, bit for bit
    chain = torch.tensor([[(1 << (t + 1)) - 1 for t in range(T)]] * B, dtype=torch.int32)
    a = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV))
    b = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), tree_mask=chain.to(DEV))
    assert torch.equal(a, b)
    # a branching tree: node parents [-1, 0, 0, 1, 1, 2, 5]
    parent = [-1, 0, 0, 1, 1, 2, 5]
    masks = []
    for t in range(T):
        m, j = 0, t
        while j >= 0:
            m |= 1 << j
            j = parent[j]
        masks.append(m)
    tm = torch.tensor([masks, masks], dtype=torch.int32)
    got = ops.verify_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), st.to(DEV), tree_mask=tm.to(DEV)).cpu().float()
    ref = _attn_ref_f32(q, kc, vc, st, tree_mask=tm)
    assert (got - ref).abs().max().item() <= 1e-2


def test_attention_gqa_reference_signature(ops):
    """attention.py:299-318 calling convention: q [B,Hq,1,D], one kv_len."""
    B, S = 2, 300
    q, kc, vc, _ = _attn_case(B, 1, 64, 8, S, [0, 0], seed=13)
    qh = q.transpose(1, 2).contiguous()  # [B, Hq, 1, D]
    kv_len = torch.tensor([257], dtype=torch.int32)
    got = ops.attention_gqa(qh.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV), 8).cpu().float()
    ref = _attn_ref_f32(q, kc, vc, torch.tensor([256, 256])).transpose(1, 2)
    assert (got - ref).abs().max().item() <= 1e-2


@pytest.mark.parametrize("M", [1, 3, 8, 11])
def test_lm_head_argmax(ops, M):
    g = torch.Generator().manual_seed(M)
    K, V = 1024, 50000
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(V, K, generator=g)).to(torch.bfloat16)
    idx, logits = ops.lm_head_argmax(x.to(DEV), w.to(DEV), return_logits=True)
    idx, logits = idx.cpu(), logits.cpu()
    ref = (x.float() @ w.float().T)
    _ulp_close(logits, ref.to(torch.bfloat16), ulps=1.0, frac_exact=0.9)
    # the pick is torch.argmax of the kernel's own bf16 logits (lowest index on ties)
    assert torch.equal(idx, logits.float().argmax(-1))


def test_accept_greedy_matches_oracle(ops):
    from oracle.spec import greedy_accept
    g = torch.Generator().manual_seed(1)
    B, K = 64, 4
    y = torch.randint(0, 3, (B, K + 1), generator=g)
    d = torch.where(torch.rand(B, K, generator=g) < 0.7, y[:, :K], torch.randint(0, 3, (B, K), generator=g))
    n_ref, tok_ref = greedy_accept(d, y)
    tl = torch.randint(10, 100, (B,), generator=g, dtype=torch.int32)
    last = torch.randint(0, 9, (B,), generator=g)
    cur = torch.randint(0, 9, (B,), generator=g)
    tl_d, last_d, cur_d = tl.to(DEV), last.to(DEV), cur.to(DEV)
    n, tok = ops.accept_greedy(d.to(DEV), y.to(DEV), tl_d, last_d, cur_d)
    assert torch.equal(n.cpu(), n_ref) and torch.equal(tok.cpu(), tok_ref)
    assert torch.equal(tl_d.cpu(), tl + n_ref + 1)
    nn = n_ref.long()
    exp_last = torch.where(nn == 0, cur, d[torch.arange(B), (nn - 1).clamp(min=0)])
    assert torch.equal(last_d.cpu(), exp_last)
    assert torch.equal(cur_d.cpu(), y[torch.arange(B), nn])

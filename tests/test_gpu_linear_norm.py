"""tsds_linear_residual_norm: the residual projection and the RMSNorm that
reads its output in one launch (the first CTAs normalise the rows once every
CTA has stored its part) against tsds_linear_residual + tsds_rms_norm - bit
for bit, for the output and the normalised rows - across the stream-K and
data-parallel schedules, CTA pairs, the row counts of decode / tree verify /
B=8 verify, more rows than one launch takes, and back-to-back launches on one
workspace (the tail's header words are reset by every launch)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture()
def lib_ops():
    from tri_sds_b200 import _lib
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(0)
    yield _lib, _ops
    lib = _lib.load()
    lib.tsds_set_gemm_dp_rows(_lib.GEMM_DP_ROWS_DEFAULT)
    lib.tsds_set_gemm_dp_slack(_lib.GEMM_DP_SLACK_DEFAULT)
    lib.tsds_set_gemm_pair_rows(0)


def _case(M, n_out, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.02 * torch.randn(n_out, K, generator=g)).to(torch.bfloat16).to(DEV)
    res = torch.randn(M, n_out, generator=g).to(torch.bfloat16).to(DEV)
    nw = (1.0 + 0.1 * torch.randn(n_out, generator=g)).to(torch.bfloat16).to(DEV)
    return x, w, res, nw


def _check(ops, M, n_out, K, seed, eps=1e-6):
    x, w, res, nw = _case(M, n_out, K, seed)
    ref_out = ops.linear_residual(x, w, res.clone())
    ref_norm = ops.rms_norm(ref_out, nw, eps)
    out, norm = ops.linear_residual_norm(x, w, res.clone(), nw, eps)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(norm, ref_norm)
    # in place, as the model runs it (out = res = the residual stream)
    xs = res.clone()
    _, norm2 = ops.linear_residual_norm(x, w, xs, nw, eps, out=xs)
    torch.cuda.synchronize()
    assert torch.equal(xs, ref_out) and torch.equal(norm2, ref_norm)
    # the fp32 reference of the norm, loosely (the arithmetic is the separate kernel's)
    r = ref_out.float()
    exp = (r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps) * nw.float())
    assert (norm.float() - exp).abs().max().item() <= 2e-2 * exp.abs().max().item() + 1e-2


# (M, n_out, K): the 32B O and 4B O/down shapes and a small one at decode / tree
# verify / B=8 verify row counts and the one-launch maximum; the 32B down
# projection at the two verify row counts
CASES = [(M, n, k) for M in (1, 4, 26, 40, 208, 256) for n, k in ((5120, 8192), (2560, 4096), (1024, 512))] + \
        [(26, 5120, 25600), (208, 5120, 25600)]


@pytest.mark.parametrize("M,n_out,K", CASES)
def test_residual_norm_equals_the_two_launches(lib_ops, M, n_out, K):
    _, ops = lib_ops
    _check(ops, M, n_out, K, seed=M * 31 + n_out)


@pytest.mark.parametrize("M", [26, 208])
def test_residual_norm_data_parallel_and_pairs(lib_ops, M):
    lib, ops = lib_ops
    L = lib.load()
    L.tsds_set_gemm_dp_rows(1)
    L.tsds_set_gemm_dp_slack(1000)    # whole tiles per CTA at every M
    _check(ops, M, 5120, 8192, seed=7 + M)
    L.tsds_set_gemm_dp_rows(0)
    L.tsds_set_gemm_pair_rows(1)      # CTA pairs
    _check(ops, M, 5120, 8192, seed=9 + M)


def test_residual_norm_more_rows_than_one_launch(lib_ops):
    _, ops = lib_ops
    _check(ops, 300, 1024, 512, seed=3)   # the two steps apart beyond 256 rows


def test_residual_norm_back_to_back_on_one_workspace(lib_ops):
    """Launches alternating with plain GEMMs on the shared workspace stay
    exact (the tail's counters are left at zero by each launch)."""
    _, ops = lib_ops
    x, w, res, nw = _case(26, 5120, 8192, seed=11)
    ref_out = ops.linear_residual(x, w, res.clone())
    ref_norm = ops.rms_norm(ref_out, nw)
    for i in range(6):
        out, norm = ops.linear_residual_norm(x, w, res.clone(), nw)
        ops.linear(x, w)   # another epilogue on the same workspace in between
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out) and torch.equal(norm, ref_norm), i


def test_model_with_and_without_fused_norms_is_identical():
    """A chain verify forward (causal, 3 layers, 6 rows) with the RMSNorms
    applied by the residual projections - the final norm included - equals
    the plan with separate RMSNorm launches, logits and argmax bit for bit."""
    from oracle import qwen as oq
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    dims = dict(hidden=512, n_heads=8, n_kv_heads=2, head_dim=128, intermediate=1024, n_layers=3, vocab=2000)
    shape = QwenShape(**dims)
    wt = oq.random_qwen_weights(oq.QwenShape(**dims), seed=5, std=0.05)
    B, T = 1, 6
    outs = []
    for fuse in (False, True):
        m = QwenModel(shape, B, 64, B * T, device=DEV, weights=wt)
        m.fuse_norm = fuse
        ids = torch.randint(0, shape.vocab, (B, T), generator=torch.Generator().manual_seed(1)).to(DEV)
        am = torch.zeros(B * T, dtype=torch.int64, device=DEV)
        logits = torch.zeros(B * T, shape.vocab, dtype=torch.bfloat16, device=DEV)
        pl = m.forward_plan(ids.contiguous(), 1, B, T, m.lengths, 0, am, 1, logits_out=logits)
        names = [n for n, _, _ in pl.calls]
        assert ("tsds_linear_residual_norm" in names) == fuse
        pl.run()
        torch.cuda.synchronize()
        m.check_status()
        outs.append((logits.clone(), am.clone(), names.count("tsds_rms_norm")))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert outs[0][2] == 2 * shape.n_layers + 1 and outs[1][2] == 1

"""The tcgen05 GEMM's data-parallel schedule (tsds_set_gemm_dp_rows: whole
weight tiles per CTA, no split tiles) vs torch fp32 references and vs the
stream-K schedule.  The two schedules sum a split tile's k-blocks in a
different order, so they agree to bf16 rounding, not bit for bit."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture()
def dp_ops():
    from tri_sds_b200 import _lib
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(0)
    _lib.load().tsds_set_gemm_dp_rows(1)   # every M with a whole tile per CTA
    yield _ops
    _lib.load().tsds_set_gemm_dp_rows(_lib.GEMM_DP_ROWS_DEFAULT)


def _data(M, n_out, K, seed, rows_mult=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(rows_mult * n_out, K, generator=g)).to(torch.bfloat16)
    return x, w


def _close_bf16(got, ref_f32, frac_exact=0.95):
    g = got.float().cpu()
    r = ref_f32.float()
    tol = r.abs() * 2.0 ** -6 + 2e-3
    assert ((g - r).abs() <= tol).all(), (g - r).abs().max().item()
    assert (g == r.to(torch.bfloat16).float()).float().mean().item() >= frac_exact


def _applies(M, n_out, K, swiglu=False):
    """Whether the launch takes the data-parallel schedule (the library's own
    planning, tsds_tc_gemm_plan, under the switches the fixture set)."""
    import ctypes

    from tri_sds_b200 import _lib
    out = (ctypes.c_int32 * 6)()
    assert _lib.load().tsds_tc_gemm_plan(2 if swiglu else 0, M, n_out, K, out) == 0
    return out[3] == 1


# (M, n_out, K) where the data-parallel schedule applies; ragged last tiles:
# 592 tiles (2 per CTA at two CTAs per SM, 4 at one) and the LM head's 1187
# (8 or 9 per CTA at one CTA per SM)
CASES = [(1, 75700, 1024), (26, 75700, 1024), (136, 75700, 1024), (208, 75700, 1024), (136, 151936, 256),
         (208, 151936, 256)]


@pytest.mark.parametrize("M,n_out,K", CASES)
def test_dp_linear(dp_ops, M, n_out, K):
    assert _applies(M, n_out, K)
    x, w = _data(M, n_out, K, seed=M * 7 + n_out)
    got = dp_ops.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(got, x.float() @ w.float().T)


@pytest.mark.parametrize("M", [136, 208])
def test_dp_residual_swiglu(dp_ops, M):
    n_res, n_out, K = 56832, 25600, 1024      # 444 residual tiles, 400 SwiGLU tiles: 2 or 3 per CTA
    assert _applies(M, n_res, K) and _applies(M, n_out, K, swiglu=True)
    xr, wr = _data(M, n_res, K, seed=13)
    res = torch.randn(M, n_res, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    got_r = dp_ops.linear_residual(xr.to(DEV), wr.to(DEV), res.to(DEV)).cpu().float()
    exp_r = (res.float() + (xr.float() @ wr.float().T).to(torch.bfloat16).float()).to(torch.bfloat16).float()
    assert (got_r - exp_r).abs().max().item() <= 2e-2
    x, w = _data(M, n_out, K, seed=11, rows_mult=2)
    ref = x.float() @ w.float().T
    got_s = dp_ops.linear_swiglu(x.to(DEV), w.to(DEV)).cpu().float()
    g, u = ref[:, :n_out].to(torch.bfloat16).float(), ref[:, n_out:].to(torch.bfloat16).float()
    exp_s = (torch.nn.functional.silu(g).to(torch.bfloat16).float() * u)
    assert (got_s - exp_s).abs().max().item() <= 2e-2 * max(1.0, exp_s.abs().max().item())


def test_dp_lm_head_argmax(dp_ops):
    """The LM head's argmax epilogue under the data-parallel schedule: the
    argmax is that of the kernel's own bf16 logits (lowest index on ties)."""
    M, V, K = 208, 151936, 512
    assert _applies(M, V, K)
    x, w = _data(M, V, K, seed=3)
    idx, logits = dp_ops.lm_head_argmax(x.to(DEV), w.to(DEV), return_logits=True)
    torch.cuda.synchronize()
    _close_bf16(logits, x.float() @ w.float().T)
    assert torch.equal(idx.cpu(), logits.float().argmax(-1).cpu())


def test_dp_and_stream_k_agree_on_a_qwen3_32b_projection(dp_ops):
    """gate/up of the 32B shape at M = 208 (the B=8 tree verify): the two
    schedules agree to bf16 rounding."""
    from tri_sds_b200 import _lib
    M, I, N = 208, 25600, 5120
    assert _applies(M, I, N, swiglu=True)
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * I, N, device=DEV, generator=g)).to(torch.bfloat16)
    got_dp = dp_ops.linear_swiglu(x, w)
    _lib.load().tsds_set_gemm_dp_rows(0)
    got_sk = dp_ops.linear_swiglu(x, w)
    torch.cuda.synchronize()
    d = (got_dp.float() - got_sk.float()).abs()
    assert d.max().item() <= 2.0 ** -7 * max(1.0, got_sk.float().abs().max().item())
    assert (d == 0).float().mean().item() >= 0.95

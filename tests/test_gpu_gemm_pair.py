"""The tcgen05 GEMM on CTA pairs (tsds_set_gemm_pair_rows: two SMs per 256-row
weight tile, tcgen05 cta_group::2) vs torch fp32 references and vs the
one-CTA kernel."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture()
def pair_ops():
    from tri_sds_b200 import _lib
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(0)
    _lib.load().tsds_set_gemm_pair_rows(1)   # every M on pairs
    yield _ops
    _lib.load().tsds_set_gemm_pair_rows(0)


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


# n_out not a multiple of 256 in two of them: the pair's second half runs past the weights
SHAPES = [(768, 2560), (5120, 1024), (1000, 512), (10240, 5120)]


@pytest.mark.parametrize("M", [1, 16, 26, 40, 100, 208, 256])
@pytest.mark.parametrize("n_out,K", SHAPES)
def test_pair_linear(pair_ops, M, n_out, K):
    x, w = _data(M, n_out, K, seed=M * 7 + n_out)
    got = pair_ops.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(got, x.float() @ w.float().T)


@pytest.mark.parametrize("M", [26, 208])
def test_pair_residual_swiglu_f32(pair_ops, M):
    from tri_sds_b200 import _lib
    n_out, K = 1000, 2560
    x, w = _data(M, n_out, K, seed=11, rows_mult=2)
    res = torch.randn(M, n_out, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    got_r = pair_ops.linear_residual(x.to(DEV), w[:n_out].contiguous().to(DEV), res.to(DEV)).cpu().float()
    exp_r = (res.float() + ref[:, :n_out].to(torch.bfloat16).float()).to(torch.bfloat16).float()
    assert (got_r - exp_r).abs().max().item() <= 2e-2
    got_s = pair_ops.linear_swiglu(x.to(DEV), w.to(DEV)).cpu().float()
    g, u = ref[:, :n_out].to(torch.bfloat16).float(), ref[:, n_out:].to(torch.bfloat16).float()
    exp_s = (torch.nn.functional.silu(g).to(torch.bfloat16).float() * u)
    assert (got_s - exp_s).abs().max().item() <= 2e-2 * max(1.0, exp_s.abs().max().item())
    ws = torch.zeros(_lib.query("tsds_linear_workspace_bytes", M, n_out, K), dtype=torch.uint8, device=DEV)
    out = torch.empty(M, n_out, dtype=torch.float32, device=DEV)
    xd, wd = x.to(DEV), w[:n_out].contiguous().to(DEV)
    _lib.call("tsds_linear_f32", pair_ops._p(xd), K, pair_ops._p(wd), pair_ops._p(out), n_out, M, n_out, K,
              pair_ops._p(ws), ws.numel(), pair_ops._stream())
    torch.cuda.synchronize()
    assert (out.cpu() - ref[:, :n_out]).abs().max().item() <= 2e-3 + 2.0 ** -8 * ref.abs().max().item()
    assert int(ws[:4].view(torch.int32)[0]) == 0


def test_pair_and_single_agree_on_a_qwen3_32b_projection(pair_ops):
    """gate/up of the 32B shape at M = 208 (the B=8 tree verify): pair and
    one-CTA kernels agree to bf16 rounding."""
    from tri_sds_b200 import _lib
    M, I, N = 208, 25600, 5120
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(M, N, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * I, N, device=DEV, generator=g)).to(torch.bfloat16)
    got_pair = pair_ops.linear_swiglu(x, w)
    _lib.load().tsds_set_gemm_pair_rows(0)
    got_one = pair_ops.linear_swiglu(x, w)
    torch.cuda.synchronize()
    d = (got_pair.float() - got_one.float()).abs()
    assert d.max().item() <= 2.0 ** -7 * max(1.0, got_one.float().abs().max().item())
    assert (d == 0).float().mean().item() >= 0.95

"""The split-K variant of the CUDA-core GEMV (tsds_set_gemv_splitk: a CTA per
few weight rows, its 256 threads sweeping K, partials summed across warps
in a fixed order) against torch fp32 references of the same ops, and
against the one-warp-per-rows GEMV."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture()
def sk_ops():
    from tri_sds_b200 import _lib
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(8)
    _lib.load().tsds_set_gemv_splitk(1)
    yield _ops
    _lib.load().tsds_set_gemv_splitk(0)
    _ops.set_gemv_max_rows(0)


def _bf16_close(got, ref_f32, eps, ulps=1.0, frac_exact=0.95):
    """bf16 outputs against the rounded fp32 reference: one ulp of the
    larger of the two (a sum just below a power of two may round up to it),
    plus eps, the bound on the fp32 sums' order difference (a sum that
    cancels to near zero keeps an absolute error of that size)."""
    g, r = got.float().cpu(), ref_f32.to(torch.bfloat16).float()
    bad = (g - r).abs() > ulps * torch.clamp(torch.maximum(g.abs(), r.abs()), min=1e-30) * 2.0 ** -7 + eps + 1e-6
    assert not bad.any(), (g - r).abs().max().item()
    assert (g == r).float().mean().item() >= frac_exact


def _acc_eps(x, w):
    """How far two fp32 sums of x @ w.T in different orders may lie apart:
    2^-20 of the sum of |x_k w_k|, i.e. 16 fp32 ulps of it.  The worst case
    grows with K; blocked and tree orders (both sides here) stay near
    log2(K) ulps, and 32B-shape sums measured on the CPU differ by about
    1/60 of this bound."""
    return 2.0 ** -20 * (x.float().abs() @ w.float().abs().T)


def _swiglu_interval(g, u, eg, eu):
    """The range of bf16(bf16(silu(bf16(g'))) * bf16(u')) over accumulations
    g' within g +- eg and u' within u +- eu: the two roundings of a sum that
    lies near a bf16 boundary, amplified by silu's slope, bound the result,
    so the kernel is held to that interval plus one ulp of the product."""
    bf = torch.bfloat16
    outs = []
    for gg in (g - eg, g + eg):
        for uu in (u - eu, u + eu):
            s = torch.nn.functional.silu(gg.to(bf).float()).to(bf).float()
            outs.append((s * uu.to(bf).float()).to(bf).float())
    st = torch.stack(outs)
    return st.min(0).values, st.max(0).values


# (n_out, K): the 4B-shape O / down projections (the narrowest), a ragged
# n_out (the last CTA's rows run past the weights), K below one 256-chunk
# sweep and K of the 32B down projection
SHAPES = [(2560, 4096), (2560, 9728), (777, 2560), (1000, 1024), (5120, 25600)]


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("n_out,K", SHAPES)
def test_splitk_linear_family(sk_ops, M, n_out, K):
    from tri_sds_b200 import _lib
    g = torch.Generator().manual_seed(M * 31 + n_out)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(2 * n_out, K, generator=g)).to(torch.bfloat16)
    res = torch.randn(M, n_out, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    xd, wd = x.to(DEV), w.to(DEV)
    w1 = wd[:n_out].contiguous()
    eps = _acc_eps(x, w[:n_out])
    _bf16_close(sk_ops.linear(xd, w1), ref[:, :n_out], eps)
    got_r = sk_ops.linear_residual(xd, w1, res.to(DEV)).cpu().float()
    exp_r = (res.float() + ref[:, :n_out].to(torch.bfloat16).float()).to(torch.bfloat16).float()
    tol = (ref[:, :n_out].abs() + exp_r.abs()) * 2.0 ** -7 + eps + 1e-6
    assert ((got_r - exp_r).abs() <= tol).all()
    got_s = sk_ops.linear_swiglu(xd, wd).cpu().float()
    lo, hi = _swiglu_interval(ref[:, :n_out], ref[:, n_out:], _acc_eps(x, w[:n_out]), _acc_eps(x, w[n_out:]))
    ulp = torch.clamp(torch.maximum(lo.abs(), hi.abs()), min=1e-30) * 2.0 ** -7 + 1e-6
    bad = (got_s < lo - ulp) | (got_s > hi + ulp)
    assert not bad.any(), (got_s - torch.clamp(got_s, lo, hi)).abs().max().item()
    # fp32 output (tensor-parallel partials): the unrounded sum
    out = torch.empty(M, n_out, dtype=torch.float32, device=DEV)
    _lib.call("tsds_linear_f32", sk_ops._p(xd), K, sk_ops._p(w1), sk_ops._p(out), n_out, M, n_out, K, None, 0,
              sk_ops._stream())
    torch.cuda.synchronize()
    assert (out.cpu() - ref[:, :n_out]).abs().max().item() <= 1e-4 * max(1.0, ref.abs().max().item())


def test_splitk_and_warp_gemv_agree(sk_ops):
    """The two GEMV variants sum in different orders: equal to one bf16 ulp."""
    from tri_sds_b200 import _lib
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4, 5120, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.02 * torch.randn(10240, 5120, generator=g)).to(torch.bfloat16).to(DEV)
    a = sk_ops.linear(x, w)
    _lib.load().tsds_set_gemv_splitk(0)
    b = sk_ops.linear(x, w)
    torch.cuda.synchronize()
    d = (a.float() - b.float()).abs()
    assert (d <= b.float().abs() * 2.0 ** -7 + 1e-6).all()
    assert (d == 0).float().mean().item() >= 0.95

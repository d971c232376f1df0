"""tcgen05 persistent GEMM (linear family + LM head) vs torch fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture()
def ops():
    from tri_sds_b200 import ops as _ops
    _ops.set_gemv_max_rows(0)  # every call below takes the tcgen05 path
    yield _ops
    _ops.set_gemv_max_rows(0)


def _data(M, n_out, K, seed, rows_mult=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(rows_mult * n_out, K, generator=g)).to(torch.bfloat16)
    return x, w


def _close_bf16(got, ref_f32, frac_exact=0.95):
    """got (bf16) within two bf16 ulps (+2e-3 absolute: the tensor core's fp32
    accumulation truncates while aligning addends) of the fp32 reference,
    and mostly equal to its rounding."""
    g = got.float().cpu()
    r = ref_f32.float()
    tol = r.abs() * 2.0 ** -6 + 2e-3
    assert ((g - r).abs() <= tol).all(), (g - r).abs().max().item()
    assert (g == r.to(torch.bfloat16).float()).float().mean().item() >= frac_exact


# (n_out, K): stream-K splits tiles across CTAs for all of these on 148 SMs
SHAPES = [(768, 2560), (5120, 1024), (1000, 512), (384, 8192), (10240, 5120)]


@pytest.mark.parametrize("M", [1, 5, 16, 17, 40, 100, 256])
@pytest.mark.parametrize("n_out,K", SHAPES[:4])
def test_tc_linear(ops, M, n_out, K):
    x, w = _data(M, n_out, K, seed=M * 7 + n_out)
    got = ops.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    _close_bf16(got, x.float() @ w.float().T)


def test_tc_linear_large_shape_and_chunked_rows(ops):
    x, w = _data(300, 10240, 5120, seed=3)     # 300 rows: chunks of 256 + 44
    got = ops.linear(x.to(DEV), w.to(DEV))
    _close_bf16(got, x.float() @ w.float().T)


@pytest.mark.parametrize("M", [5, 40])
def test_tc_residual_and_swiglu(ops, M):
    n_out, K = 1000, 2560
    x, w = _data(M, n_out, K, seed=11, rows_mult=2)
    res = torch.randn(M, n_out, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    got_r = ops.linear_residual(x.to(DEV), w[:n_out].contiguous().to(DEV), res.to(DEV)).cpu().float()
    ref_r = (res.float() + ref[:, :n_out].to(torch.bfloat16).float()).to(torch.bfloat16).float()
    tol = (ref[:, :n_out].abs() + ref_r.abs()) * 2.0 ** -7 + 1e-5
    assert ((got_r - ref_r).abs() <= tol).all()
    got_s = ops.linear_swiglu(x.to(DEV), w.to(DEV)).cpu().float()
    g, u = ref[:, :n_out].to(torch.bfloat16), ref[:, n_out:].to(torch.bfloat16)
    ref_s = (torch.nn.functional.silu(g) * u).float()
    tol = ref_s.abs() * 2.0 ** -6 + 1e-4
    assert ((got_s - ref_s).abs() <= tol).all(), (got_s - ref_s).abs().max().item()


def test_tc_row_result_independent_of_M(ops):
    """A row's output is bit-identical whether it is computed alone or among 40 rows."""
    n_out, K = 5120, 8192
    x, w = _data(40, n_out, K, seed=21)
    wd = w.to(DEV)
    full = ops.linear(x.to(DEV), wd)
    for m in (0, 7, 39):
        one = ops.linear(x[m:m + 1].contiguous().to(DEV), wd)
        assert torch.equal(one[0], full[m]), m


@pytest.mark.parametrize("M", [1, 5, 40])
def test_tc_lm_head_argmax(ops, M):
    K, V = 2560, 50000
    x, w = _data(M, V, K, seed=M)
    idx, logits = ops.lm_head_argmax(x.to(DEV), w.to(DEV), return_logits=True)
    idx, logits = idx.cpu(), logits.cpu()
    _close_bf16(logits, x.float() @ w.float().T, frac_exact=0.9)
    assert torch.equal(idx, logits.float().argmax(-1))


def test_tc_repeated_calls_reuse_workspace(ops):
    """Counters left by one launch are ready for the next (no re-zeroing)."""
    x, w = _data(5, 5120, 1024, seed=4)
    xd, wd = x.to(DEV), w.to(DEV)
    first = ops.linear(xd, wd)
    for _ in range(5):
        assert torch.equal(ops.linear(xd, wd), first)


def test_lm_head_varying_M_shares_one_workspace():
    """Calls with different M (both GEMV and tcgen05 paths) on one workspace:
    the tile counters sit at a fixed offset no other data ever overwrites."""
    from tri_sds_b200 import ops as o
    o.set_gemv_max_rows(4)  # mix both paths on one workspace
    K, V = 1024, 30000
    g = torch.Generator().manual_seed(99)
    w = (0.05 * torch.randn(V, K, generator=g)).to(torch.bfloat16).to(DEV)
    for M in (40, 5, 1, 3, 8, 17, 2, 40, 11):
        x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
        idx, logits = o.lm_head_argmax(x, w, return_logits=True)
        ref = (x.float() @ w.float().T).cpu()
        lg = logits.cpu().float()
        assert ((lg - ref).abs() <= ref.abs() * 2.0 ** -6 + 2e-3).all(), M
        assert torch.equal(idx.cpu(), lg.argmax(-1)), M
    o.set_gemv_max_rows(0)

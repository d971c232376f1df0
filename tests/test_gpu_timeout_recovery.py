"""Recovery from a device wait that gave up (tcgen05 GEMM, C ABI).

With the wait limit lowered to 1 ns every bounded wait of the kernel gives
up at once: the launch records TSDS_E_TIMEOUT in the workspace's status
word and its CTAs unwind (in-flight copies and MMAs drained, TMEM freed),
leaving split-tile counters behind.  The host's status check then zeroes
the workspace header (status word + counters).  With the limit restored,
the next launch on the same workspace must equal a launch on a fresh
workspace bit for bit - the residual epilogue (split tiles summed by all
contributors) and the SwiGLU epilogue (last-arriver reduction) alike - and
leave the header zero again."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _call(lib, epi, x, w, res, out, ws, nb, s):
    from tri_sds_b200 import ops
    M, K = x.shape
    if epi == "residual":
        n_out = w.shape[0]
        return lib.tsds_linear_residual(ops._p(x), K, ops._p(w), ops._p(res), ops._p(out), n_out, M, n_out, K,
                                        ops._p(ws), nb, s)
    n_out = w.shape[0] // 2
    return lib.tsds_linear_swiglu(ops._p(x), K, ops._p(w), ops._p(out), n_out, M, n_out, K, ops._p(ws), nb, s)


@pytest.mark.parametrize("epi,n_out,K", [("residual", 5120, 8192), ("swiglu", 25600, 5120)])
def test_next_launch_after_a_timeout_is_correct(epi, n_out, K):
    from tri_sds_b200 import _lib, ops
    from tri_sds_b200.model import raise_status
    lib = _lib.load()
    ops.set_gemv_max_rows(0)
    M = 26
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    rows = n_out if epi == "residual" else 2 * n_out
    w = (0.02 * torch.randn(rows, K, device=DEV, generator=g)).to(torch.bfloat16)
    res = torch.randn(M, n_out, device=DEV, generator=g).to(torch.bfloat16)
    nb = _lib.query("tsds_linear_workspace_bytes", M, n_out, K)
    hb = _lib.query("tsds_linear_workspace_header_bytes")
    s = ops._stream()
    fresh = torch.zeros(nb, dtype=torch.uint8, device=DEV)
    ref = torch.empty(M, n_out, dtype=torch.bfloat16, device=DEV)
    assert _call(lib, epi, x, w, res, ref, fresh, nb, s) == 0
    ws = torch.zeros(nb, dtype=torch.uint8, device=DEV)
    out = torch.empty_like(ref)
    limit = lib.tsds_get_wait_limit_ns()
    try:
        lib.tsds_set_wait_limit_ns(1)
        assert _call(lib, epi, x, w, res, out, ws, nb, s) == 0
    finally:
        lib.tsds_set_wait_limit_ns(limit)
    torch.cuda.synchronize()
    word = ws[:4].view(torch.int32)
    st = int(word.item())
    assert st == 5, st   # TSDS_E_TIMEOUT
    # a launch that gives up mid-way leaves some tiles' arrivals counted;
    # stand in for that with counts in every counter (host writes)
    ws[64:hb].view(torch.int32).fill_(1)
    with pytest.raises(RuntimeError, match="status 5"):
        raise_status(word, st, ws[:hb])
    assert int(ws[:hb].count_nonzero()) == 0
    for _ in range(2):
        out.fill_(0)
        assert _call(lib, epi, x, w, res, out, ws, nb, s) == 0
        torch.cuda.synchronize()
        assert int(word.item()) == 0
        assert torch.equal(out, ref)
        assert int(ws[:hb].count_nonzero()) == 0   # every launch leaves its counters zero

"""The fused-layer kernel on the GPU (tsds_fused_layer: O -> RMSNorm -> gate/up
-> down -> RMSNorm -> q/k/v with QK-norm + RoPE + KV write in one launch).

* Qwen3-4B-shape layers: where the fused kernel's grid equals the per-op
  GEMMs' (tsds_fused_layer_grid vs tsds_tc_gemm_plan), the fused plan
  reproduces the per-op plan bit for bit (hidden state, q, K and V caches),
  since both split and sum every tile the same way and round identically;
  where the grids differ (one fused CTA per SM against the GEMMs' two at
  small M), to bf16 rounding and the logit tolerance;
* the small shape of the other GPU tests: logits within the bf16 tolerance
  of the oracle;
* EAGLE greedy decoding with fused layers equals greedy autoregressive
  decoding.
"""
import pytest
import torch

from oracle import eagle as oe
from oracle import qwen as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)
Q4B = dict(hidden=2560, n_heads=32, n_kv_heads=8, head_dim=128, intermediate=9728, n_layers=2, vocab=1000)


def _models(kw, B, max_rows, max_seq, seed):
    from tri_sds_b200 import ops
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    oshape = oq.QwenShape(**kw)
    w = oq.random_qwen_weights(oshape, seed=seed, std=0.02)
    ms = [QwenModel(QwenShape(**kw), batch=B, max_seq=max_seq, max_rows=max_rows, device=DEV, weights=w,
                    fused_layers=f) for f in (False, True)]
    return oshape, w, ms


def _verify(m, ids, B, T, vocab):
    am = torch.zeros(B * T, dtype=torch.int64, device=DEV)
    logits = torch.zeros(B * T, vocab, dtype=torch.bfloat16, device=DEV)
    m.forward_plan(ids.to(DEV).contiguous(), 1, B, T, m.lengths, 0, am, 1, logits_out=logits).run()
    torch.cuda.synchronize()
    m.check_status()
    if m.fused_layers:
        assert int(m.fused_ws[:4].view(torch.int32)[0]) == 0   # no bounded wait gave up
    return logits, am


@pytest.mark.parametrize("B,T", [(1, 5), (8, 5), (1, 26), (8, 26)])
def test_fused_equals_per_op_bitwise_qwen3_4b_shape(B, T):
    _bitwise_case(B, T)


@pytest.mark.parametrize("B,T", [(1, 26), (8, 26)])
def test_fused_equals_per_op_bitwise_on_cta_pairs(B, T):
    """Both plans' GEMMs on CTA pairs (the per-op GEMM and the fused
    kernel's phases alike): still bit for bit."""
    from tri_sds_b200 import _lib
    _lib.load().tsds_set_gemm_pair_rows(1)
    try:
        _bitwise_case(B, T)
    finally:
        _lib.load().tsds_set_gemm_pair_rows(0)


@pytest.mark.parametrize("B,T", [(1, 26), (8, 26)])
def test_fused_equals_per_op_bitwise_data_parallel(B, T):
    """Both plans' GEMMs under the data-parallel schedule where it applies
    (the per-op GEMM and the fused kernel's phases make the same choice):
    still bit for bit."""
    from tri_sds_b200 import _lib
    _lib.load().tsds_set_gemm_dp_rows(1)
    _lib.load().tsds_set_gemm_dp_slack(100)
    try:
        _bitwise_case(B, T)
    finally:
        _lib.load().tsds_set_gemm_dp_rows(_lib.GEMM_DP_ROWS_DEFAULT)
        _lib.load().tsds_set_gemm_dp_slack(_lib.GEMM_DP_SLACK_DEFAULT)


def _bitwise_case(B, T):
    S = 1024
    oshape, w, (ref, fus) = _models(Q4B, B, B * T, S, seed=B * 100 + T)
    g = torch.Generator().manual_seed(B + T)
    starts = torch.randint(0, S - T - 1, (B,), generator=g).to(torch.int32)
    ids = torch.randint(0, oshape.vocab, (B, T), generator=g)
    kpre = torch.randn(2, B, 8, S, 128, generator=g).to(torch.bfloat16)
    vpre = torch.randn(2, B, 8, S, 128, generator=g).to(torch.bfloat16)
    outs = []
    for m in (ref, fus):
        m.k_cache.copy_(kpre.to(DEV))
        m.v_cache.copy_(vpre.to(DEV))
        m.lengths.copy_(starts.to(DEV))
        logits, am = _verify(m, ids, B, T, oshape.vocab)
        outs.append((m.x[:B * T].clone(), m.q[:B * T].clone(), m.k_cache.clone(), m.v_cache.clone(), logits, am))
    if _same_split(B * T):
        for a, b, what in zip(outs[0], outs[1], ("hidden", "q", "k cache", "v cache", "logits", "argmax")):
            assert torch.equal(a, b), what
        return
    # a different grid splits the reductions differently: the two plans then
    # agree to bf16 rounding (hidden / q / caches), and their logits - each
    # within the 2e-2 bf16 tolerance of the oracle (test_fused_verify_matches_
    # oracle) - within twice that of each other
    for a, b, what in zip(outs[0][:4], outs[1][:4], ("hidden", "q", "k cache", "v cache")):
        a, b = a.float(), b.float()
        assert (a - b).abs().max().item() <= 3e-2 * max(1.0, a.abs().max().item()), what
    assert (outs[0][4].float() - outs[1][4].float()).abs().max().item() <= 4e-2


def _same_split(M):
    """True when the fused kernel's grid equals the per-op GEMMs' at M rows,
    so both plans split and sum every projection the same way."""
    import ctypes
    from tri_sds_b200 import _lib
    out = (ctypes.c_int32 * 8)()
    assert _lib.load().tsds_fused_layer_grid(M, out) == 0
    fused_p = out[0]
    same = True
    for epi, n, k in ((0, 6144, 2560), (1, 2560, 4096), (2, 9728, 2560), (1, 2560, 9728)):
        assert _lib.load().tsds_tc_gemm_plan(epi, M, n, k, out) == 0
        same = same and out[2] == fused_p
    return same


@pytest.mark.parametrize("B,T", [(1, 1), (2, 5), (2, 26)])
def test_fused_verify_matches_oracle(B, T):
    oshape, w, (ref, fus) = _models(SMALL, B, B * T, 128, seed=1)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, oshape.vocab, (B, 12), generator=g)
    step = torch.randint(0, oshape.vocab, (B, T), generator=g)
    ora = oq.QwenOracle(oshape, w, batch=B, max_seq=128)
    ora.forward(prompt)
    ora.lengths[:] = 12
    ref_logits, _ = ora.forward(step)
    for m in (ref, fus):
        m.prefill(prompt)
        logits, am = _verify(m, step, B, T, oshape.vocab)
        got = logits.cpu().float().reshape(B, T, -1)
        assert (got - ref_logits.float()).abs().max().item() <= 2e-2
        assert torch.equal(am.cpu(), logits.cpu().float().argmax(-1))


def test_fused_eagle_greedy_equals_autoregressive():
    from tri_sds_b200 import ops
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.engine import AutoregressiveEngine
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    B, n_new = 2, 20
    oshape, shape = oq.QwenShape(**SMALL), QwenShape(**SMALL)
    wt = oq.random_qwen_weights(oshape, seed=0, std=0.08)
    we = oe.random_eagle_weights(oshape, seed=1, std=0.08)
    prompt = torch.randint(0, oshape.vocab, (B, 10), generator=torch.Generator().manual_seed(2))
    tgt = QwenModel(shape, batch=B, max_seq=128, max_rows=B * 26, device=DEV, weights=wt, fused_layers=True)
    eng = EagleEngine(tgt, EagleHead(tgt, B, weights=we), greedy=True)
    assert eng.head.model.fused_layers
    spec, _ = eng.generate(prompt, n_new)
    ar_model = QwenModel(shape, batch=B, max_seq=128, max_rows=B, device=DEV, weights=wt, fused_layers=True)
    ar = AutoregressiveEngine(ar_model).generate(prompt, n_new)
    for b in range(B):   # equal up to the first bf16 near-tie of the target's own logits
        diff = (spec[b] != ar[b]).nonzero()
        if diff.numel() == 0:
            continue
        i = int(diff[0])
        ora = oq.QwenOracle(oshape, wt, batch=1, max_seq=128)
        lg, _ = ora.forward(torch.cat([prompt[b], ar[b, :i]]).unsqueeze(0))
        last = lg[0, -1].float()
        assert abs((last[int(ar[b, i])] - last[int(spec[b, i])]).item()) <= 2e-2, (b, i)

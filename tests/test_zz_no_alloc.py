"""The allocation-free verify attention (tsds_verify_attention_noalloc).

It serves callers that may not allocate device memory (a plugin inside a
framework that reserved the GPU's memory, or code running under stream
capture): its scratch is a built-in device array instead of a caller
workspace.  Through the C ABI, two calls in a row must reproduce the
workspace entry point's output; the second call reuses the scratch the
first one left behind.  This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
_P = ctypes.c_void_p


def _p(t):
    return None if t is None else _P(t.data_ptr())


def _case(B, T, S, starts, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, 64, 128, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(B, 8, S, 128, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(B, 8, S, 128, generator=g).to(torch.bfloat16).to(DEV)
    st = torch.tensor(starts, dtype=torch.int32, device=DEV)
    return q, kc, vc, st


def test_noalloc_attention_matches_workspace_entry_point():
    from tri_sds_b200 import _lib
    lib = _lib.load()
    stream = _P(torch.cuda.current_stream().cuda_stream)
    split = 256
    cases = [(2, 5, 1024, [700, 1011], 1), (1, 1, 2048, [1999], 2)]
    for (B, T, S, starts, seed) in cases:  # two calls in a row, different shapes and data
        q, kc, vc, st = _case(B, T, S, starts, seed)
        nb = lib.tsds_attention_workspace_bytes(B, T, 64, 8, 128, S, split)
        assert 0 < nb <= lib.tsds_verify_attention_noalloc_limit()
        ws = torch.zeros(nb, dtype=torch.uint8, device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        assert lib.tsds_verify_attention(_p(q), _p(kc), _p(vc), _p(ref), _p(st), None, -1, B, T, 64, 8, 128, S, S, split,
                                         128 ** -0.5, _p(ws), nb, _p(status), stream) == 0
        assert lib.tsds_verify_attention_noalloc(_p(q), _p(kc), _p(vc), _p(got), _p(st), None, -1, B, T, 64, 8, 128, S, S,
                                                 split, 128 ** -0.5, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref)          # same kernels, same key splits: bit-identical
        host_status = ctypes.c_int32(-1)
        assert lib.tsds_verify_attention_noalloc_status(ctypes.byref(host_status)) == 0
        assert host_status.value == 0 and int(status.item()) == 0


def test_noalloc_attention_rejects_requests_beyond_its_scratch():
    from tri_sds_b200 import _lib
    lib = _lib.load()
    B, T, S, split = 8, 5, 4096, 64
    assert lib.tsds_attention_workspace_bytes(B, T, 64, 8, 128, S, split) > lib.tsds_verify_attention_noalloc_limit()
    rc = lib.tsds_verify_attention_noalloc(None, None, None, None, None, None, -1, B, T, 64, 8, 128, S, S, split,
                                           0.1, _P(torch.cuda.current_stream().cuda_stream))
    assert rc == 8  # TSDS_E_SCRATCH_LIMIT
    assert lib.tsds_status_string(rc) == b"request larger than the built-in scratch area"

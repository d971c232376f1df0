"""The C-ABI library loads and exports every symbol include/tsds.h declares (no GPU needed)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "tsds.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tsds_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding_table():
    from tri_sds_b200 import _lib
    assert _declared() == sorted(_lib.exported_symbols())


def test_library_exports_every_symbol():
    from tri_sds_b200 import _lib
    from tri_sds_b200.build import LIB, build
    if not os.path.exists(LIB):
        build()
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.tsds_abi_version() == 1
    assert lib.tsds_status_string(0) == b"ok"


def test_argument_validation_without_gpu():
    """Shape checks run on the host before any launch and return codes."""
    from tri_sds_b200 import _lib
    lib = _lib.load()
    assert lib.tsds_rms_norm(None, None, None, 0, 128, 128, 128, 1e-6, None) == 1          # INVALID
    assert lib.tsds_linear(None, 8, None, None, 8, 1, 8, 8, None, 0, None) == 1
    assert lib.tsds_qk_norm_rope_kv(None, None, None, None, None, None, None, None, None, None,
                                    1, 1, 8, 2, 64, 16, 16, 1e-6, None) == 6                 # UNSUPPORTED D
    assert lib.tsds_verify_attention(None, None, None, None, None, None, -1, 1, 4, 8, 2, 64, 64, 64, 64,
                                     0.1, None, 0, None, None) == 6                           # UNSUPPORTED D


def test_residual_norm_argument_validation_without_gpu():
    """tsds_linear_residual_norm's host checks: missing pointers, widths and
    strides off the 8-element grid, misaligned buffers, a missing
    workspace - all before any launch."""
    import ctypes
    from tri_sds_b200 import _lib
    lib = _lib.load()
    buf = ctypes.create_string_buffer(1 << 16)
    a = ctypes.addressof(buf)
    al = (a + 255) // 256 * 256      # 16-byte aligned host addresses (never dereferenced)
    P = ctypes.c_void_p
    def call(x=al, w=al, res=al, out=al, ldo=64, n_out=64, nw=al, nout=al, nld=64, ws=al, wsb=4096, M=2, K=64):
        return lib.tsds_linear_residual_norm(P(x), K, P(w), P(res), P(out), ldo, M, n_out, K, P(nw), P(nout), nld,
                                             ctypes.c_float(1e-6), P(ws), wsb, None)
    assert call(res=None) == 1             # INVALID: no residual
    assert call(nw=None) == 1              # INVALID: no norm weights
    assert call(n_out=60, ldo=64) == 1     # INVALID: width off the 8-element grid
    assert call(nld=60) == 1               # INVALID: norm_out stride below the width
    assert call(nout=al + 2) == 2          # ALIGN
    assert call(ws=None) == 4              # WORKSPACE: the one-launch path needs one


def test_attention_row_and_cache_limits_without_gpu():
    """tsds_verify_attention's size checks (host only, before any device
    call): the default kernel takes up to 1024 query rows per kv head, the
    tcgen05 variant up to 65536; cache rows B*Hkv*S must fit an int."""
    import ctypes
    from tri_sds_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(0x1000)   # aligned stand-ins: the checks under test come first

    def call(T, Hq=64, Hkv=8, B=1, S=4096, split=128):
        return lib.tsds_verify_attention(p, p, p, p, p, None, -1, B, T, Hq, Hkv, 128, S, S, split, 0.1, p, 1 << 30,
                                         p, None)

    try:
        lib.tsds_set_attention_tc(0)
        assert call(T=129) == 6                     # 1032 rows: UNSUPPORTED on the default kernel
        assert call(T=128, B=1 << 16, Hkv=8, S=4096) == 6   # 2^31 cache rows
        lib.tsds_set_attention_tc(1)
        assert lib.tsds_get_attention_tc() == 1
        assert call(T=129) not in (1, 2, 6)        # past the row checks (fails later: no device here)
        assert call(T=8193) == 6                    # 65544 rows
        assert call(T=129, split=64) == 6           # 64-key splits keep the default kernel and its limit
        lib.tsds_set_attention_tc(7)
        assert lib.tsds_get_attention_tc() == 2     # clamped
    finally:
        lib.tsds_set_attention_tc(0)


def test_tuning_switches_clamp_and_read_back():
    """The process-wide GEMM / GEMV switches keep their documented ranges and
    read back what was set (each restored afterwards)."""
    from tri_sds_b200 import _lib
    lib = _lib.load()
    try:
        for v, want in [(-3, 0), (0, 0), (128, 128)]:
            lib.tsds_set_gemm_dp_rows(v)
            assert lib.tsds_get_gemm_dp_rows() == want
            lib.tsds_set_gemm_pair_rows(v)
            assert lib.tsds_get_gemm_pair_rows() == want
        for v, want in [(-1, 0), (15, 15), (5000, 1000)]:
            lib.tsds_set_gemm_dp_slack(v)
            assert lib.tsds_get_gemm_dp_slack() == want
        for v, want in [(0, 0), (7, 1), (1, 1)]:
            lib.tsds_set_gemv_splitk(v)
            assert lib.tsds_get_gemv_splitk() == want
        for v, want in [(-2, 0), (3, 3), (99, 8)]:
            lib.tsds_set_gemv_max_rows(v)
            assert lib.tsds_get_gemv_max_rows() == want
    finally:
        lib.tsds_set_gemm_dp_rows(_lib.GEMM_DP_ROWS_DEFAULT)
        lib.tsds_set_gemm_pair_rows(0)
        lib.tsds_set_gemm_dp_slack(_lib.GEMM_DP_SLACK_DEFAULT)
        lib.tsds_set_gemv_splitk(0)
        lib.tsds_set_gemv_max_rows(0)


def test_gemm_plan_query_checks_its_arguments():
    import ctypes

    from tri_sds_b200 import _lib
    lib = _lib.load()
    out = (ctypes.c_int32 * 6)()
    assert lib.tsds_tc_gemm_plan(0, 26, 5120, 8192, out) == 0
    assert lib.tsds_tc_gemm_plan(7, 26, 5120, 8192, out) != 0      # no such epilogue
    assert lib.tsds_tc_gemm_plan(0, 0, 5120, 8192, out) != 0       # no rows
    assert lib.tsds_tc_gemm_plan(0, 257, 5120, 8192, out) != 0     # more rows than one launch takes
    assert lib.tsds_tc_gemm_plan(0, 26, 5120, 8192, None) != 0

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

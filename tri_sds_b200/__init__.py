"""tri_sds_b200: sm_100a speculative-decoding hot path with tri-sds's plugin API.

``create_plugin()`` registers ``TriSDSWorker`` in place of SGLang's
``StandaloneWorker`` exactly like the reference (tri_sds/__init__.py:1-10).
The device work runs in libtsds.so (hand-written CUDA for sm_100a) through
its C ABI (include/tsds.h).
"""
from __future__ import annotations

__version__ = "0.1.0"

STANDALONE_WORKER = "sglang.srt.speculative.standalone_worker.StandaloneWorker"


def create_plugin():
    """Register TriSDSWorker as a REPLACE hook (tri_sds/__init__.py:1-10)."""
    from .sglang_compat import HookRegistry, HookType
    from .worker import TriSDSWorker

    HookRegistry.register(STANDALONE_WORKER, TriSDSWorker, HookType.REPLACE)

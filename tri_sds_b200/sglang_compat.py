"""SGLang names the plugin boundary needs, or stand-ins when SGLang is absent.

The reference imports ``HookRegistry``/``HookType`` (tri_sds/__init__.py:2),
``ScheduleBatch`` and ``StandaloneWorker`` (tri_sds/worker.py:3-4) from
SGLang.  When SGLang is installed those are used; otherwise minimal
stand-ins with the same names keep the plugin importable and testable.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

try:  # pragma: no cover - SGLang is not part of this environment
    from sglang.srt.managers.schedule_batch import ScheduleBatch  # type: ignore
    from sglang.srt.plugins.hook_registry import HookRegistry, HookType  # type: ignore
    from sglang.srt.speculative.standalone_worker import StandaloneWorker  # type: ignore
    HAVE_SGLANG = True
except Exception:  # noqa: BLE001
    HAVE_SGLANG = False

    class HookType(enum.Enum):
        REPLACE = "replace"

    class HookRegistry:
        """Records registrations: target dotted path -> (replacement, hook type)."""
        hooks: dict = {}

        @classmethod
        def register(cls, target: str, replacement, hook_type: "HookType"):
            cls.hooks[target] = (replacement, hook_type)

        @classmethod
        def lookup(cls, target: str):
            return cls.hooks.get(target)

    @dataclass
    class ScheduleBatch:
        """The fields the spec worker reads: token ids [B, T] (or a list of
        the sequences' prompts, ragged), positions, seq_lens (real tokens
        per row of a padded [B, P] prompt) and reqs (requests, each with a
        ``rid``: the batch's identity)."""
        input_ids: object = None
        positions: object = None
        seq_lens: object = None
        reqs: list = field(default_factory=list)
        extra: dict = field(default_factory=dict)

    class StandaloneWorker:
        """Stand-in for SGLang's worker: the non-SDS path is SGLang's own."""

        def __init__(self, *args, **kwargs):
            self.args, self.kwargs = args, kwargs

        def forward_batch_generation(self, batch):
            raise NotImplementedError("SGLang's StandaloneWorker is not installed")

        def draft(self, batch):
            raise NotImplementedError("SGLang's StandaloneWorker is not installed")

        def verify(self, batch):
            raise NotImplementedError("SGLang's StandaloneWorker is not installed")

"""CPU oracle for the speculative-decoding hot path (test infrastructure).

This package restates, in plain PyTorch on the CPU, the reference's
algorithm for the path draft -> verify -> accept -> KV commit:

* ``qwen``  - the Qwen3 forward of ``tri_sds/triton_kernels/qwen_model.py``
  (weight packing, RoPE, the verify forward over the KV cache, final norm +
  LM head), with the RMSNorm of ``tri_sds/triton_kernels/norm.py:42-72``;
* ``spec``  - the spec loop, greedy acceptance and KV commit, which the
  reference delegates to SGLang (absent from the reference tree, so these
  semantics are written down here and pinned by properties, not by golden
  vectors of the reference);
* ``eagle`` - ``tri_sds/triton_kernels/eagle_head.py`` plus tree drafting
  and rejection sampling;
* ``gpt2``  - the GPT-2 path of ``tri_sds/triton_kernels/model.py``.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg import it.  The product path
(``tri_sds_b200``) never imports this package and fails loudly when its
CUDA library is missing.
"""

"""Ragged prompts (SGLang batches: prompts of different lengths) on the GPU.

A batch of prompts of lengths 3, 11 and 7, padded behind each prompt and
prefilled together, then decoded by EAGLE tree speculation, by chain
speculation with a draft model and autoregressively.  Every sequence must
continue exactly as the oracle continues its prompt alone (greedy), up to
the first bf16 near-tie of the oracle's own logits; the speculative engines
must equal the autoregressive one on the same ragged batch."""

import pytest
import torch

from oracle import eagle as oe
from oracle import qwen as oq
from oracle.spec import autoregressive

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)
LENGTHS = [3, 11, 7]


def _prompts():
    g = torch.Generator().manual_seed(31)
    seqs = [torch.randint(0, SMALL["vocab"], (n,), generator=g) for n in LENGTHS]
    P = max(LENGTHS)
    padded = torch.zeros(len(seqs), P, dtype=torch.int64)
    for b, x in enumerate(seqs):
        padded[b, :len(x)] = x
    return seqs, padded, torch.tensor(LENGTHS, dtype=torch.int32)


def _model(shape, w, B, rows):
    from tri_sds_b200.model import QwenModel
    return QwenModel(shape, batch=B, max_seq=128, max_rows=rows, device=DEV, weights=w)


def _near_tie_or_equal(oshape, w, prompt, ref, got, tol=2e-2):
    diff = (ref != got).nonzero()
    if diff.numel() == 0:
        return
    i = int(diff[0])
    logits, _ = oq.QwenOracle(oshape, w, batch=1, max_seq=128).forward(torch.cat([prompt, ref[:i]]).unsqueeze(0))
    last = logits[0, -1].float()
    margin = (last[int(ref[i])] - last[int(got[i])]).item()
    assert 0.0 <= margin <= tol, (i, margin)


def test_ragged_batch_decodes_like_each_prompt_alone():
    from tri_sds_b200 import ops
    from tri_sds_b200.eagle import EagleEngine, EagleHead
    from tri_sds_b200.engine import AutoregressiveEngine, SpecEngine
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    oshape, shape = oq.QwenShape(**SMALL), QwenShape(**SMALL)
    wt = oq.random_qwen_weights(oshape, seed=5, std=0.08)
    we = oe.random_eagle_weights(oshape, seed=6, std=0.08)
    wd = {**wt, "layers": wt["layers"][:1]}
    seqs, padded, n = _prompts()
    B, n_new, K = len(seqs), 16, 4
    ar = AutoregressiveEngine(_model(shape, wt, B, B)).generate(padded, n_new, n)
    tgt = _model(shape, wt, B, B * 26)
    eagle, _ = EagleEngine(tgt, EagleHead(tgt, B, weights=we), greedy=True).generate(padded, n_new, n)
    drf = _model(QwenShape(**{**SMALL, "n_layers": 1}), wd, B, B * 2)
    chain, _ = SpecEngine(_model(shape, wt, B, B * (K + 1)), drf, K).generate(padded, n_new, n)
    for b in range(B):
        ref = autoregressive(oq.QwenOracle(oshape, wt, batch=1, max_seq=128), seqs[b].unsqueeze(0), n_new)[0]
        _near_tie_or_equal(oshape, wt, seqs[b], ref, ar[b])
        # the speculative engines equal autoregressive decoding on the same batch
        _near_tie_or_equal(oshape, wt, seqs[b], ar[b], eagle[b])
        assert torch.equal(chain[b], ar[b]), b

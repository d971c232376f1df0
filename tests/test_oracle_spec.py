"""Properties of the oracle's chain spec cycle (greedy losslessness, acceptance rules)."""
import torch

from oracle.qwen import QwenOracle, QwenShape, random_qwen_weights
from oracle.spec import ChainSpecOracle, autoregressive, greedy_accept

TINY = QwenShape(hidden=64, n_heads=4, n_kv_heads=2, head_dim=16, intermediate=128, n_layers=2, vocab=97)


def test_greedy_accept_rules():
    d = torch.tensor([[5, 6, 7, 8], [1, 2, 3, 4], [9, 9, 9, 9], [3, 0, 0, 0]])
    y = torch.tensor([[5, 6, 0, 8, 1], [0, 2, 3, 4, 4], [9, 9, 9, 9, 7], [3, 1, 0, 0, 0]])
    n, tok = greedy_accept(d, y)
    assert n.tolist() == [2, 0, 4, 1]
    assert tok.tolist() == [[5, 6, 0, -1, -1], [0, -1, -1, -1, -1], [9, 9, 9, 9, 7], [3, 1, -1, -1, -1]]


def _spec_vs_ar(draft_weights, target_weights, B=2, P=7, n_new=12, k=4):
    tgt = QwenOracle(TINY, target_weights, batch=B, max_seq=64, dtype=torch.float32)
    drf = QwenOracle(TINY, draft_weights, batch=B, max_seq=64, dtype=torch.float32)
    prompt = torch.randint(0, TINY.vocab, (B, P), generator=torch.Generator().manual_seed(11))
    spec, acc = ChainSpecOracle(tgt, drf, k).generate(prompt, n_new)
    ar = autoregressive(QwenOracle(TINY, target_weights, batch=B, max_seq=64, dtype=torch.float32),
                        prompt, n_new)
    return spec, ar, acc


def test_spec_equals_autoregressive_self_draft():
    """Draft == target: every draft is accepted and the output is the
    target's own greedy continuation."""
    w = random_qwen_weights(TINY, seed=3, dtype=torch.float32, std=0.2)
    spec, ar, acc = _spec_vs_ar(w, w)
    assert torch.equal(spec, ar)
    assert int(acc.float().mean().round()) == 4


def test_spec_equals_autoregressive_independent_draft():
    """An unrelated draft changes only how many tokens each cycle keeps."""
    wt = random_qwen_weights(TINY, seed=3, dtype=torch.float32, std=0.2)
    wd = random_qwen_weights(TINY, seed=4, dtype=torch.float32, std=0.2)
    spec, ar, _ = _spec_vs_ar(wd, wt)
    assert torch.equal(spec, ar)

"""GPT-2 correctness config (CPU, fp32): the oracle vs the reference's own
batched forward, and greedy spec decoding vs greedy autoregressive decoding."""
import torch

from conftest import load_golden
from oracle.gpt2 import (GPT2_SMALL, GPT2ChainSpec, GPT2Oracle, GPT2Shape, draft_weights_from_target,
                         gpt2_autoregressive, random_gpt2_weights, weights_from_state_dict)


def test_gpt2_matches_reference_batched_forward():
    """At start 0 the cache-correct forward equals model.py:89-135 (and HF up to tanh-vs-erf GELU)."""
    fx = load_golden("gpt2_ref_f32.pt")
    cfg = fx["config"]
    shape = GPT2Shape(n_layer=cfg["n_layer"], n_embd=cfg["n_embd"], n_head=cfg["n_head"], n_inner=4 * cfg["n_embd"],
                      n_positions=cfg["n_positions"], vocab=cfg["vocab_size"])
    st = GPT2Oracle(shape, weights_from_state_dict(fx["state_dict"], shape.n_layer), batch=1)
    got = st.forward(fx["ids"])
    assert (got - fx["logits"]).abs().max().item() <= 1e-5
    assert (got - fx["hf_logits"]).abs().max().item() <= 1e-3
    assert (st.k[0][:, :, :10] - fx["k_cache0"]).abs().max().item() <= 1e-6


def test_gpt2_verify_over_cache_equals_full_prefill():
    shape = GPT2Shape(n_layer=2, n_embd=64, n_head=4, n_inner=256, n_positions=64, vocab=300)
    w = random_gpt2_weights(shape, seed=3, std=0.05)
    ids = torch.randint(0, 300, (2, 20), generator=torch.Generator().manual_seed(4))
    full = GPT2Oracle(shape, w, batch=2).forward(ids)
    st = GPT2Oracle(shape, w, batch=2)
    a = st.forward(ids[:, :15]); st.lengths[:] = 15
    b = st.forward(ids[:, 15:])
    assert (torch.cat([a, b], 1) - full).abs().max().item() <= 1e-5


def test_gpt2_small_spec_decode_token_for_token():
    """The GPT-2-small correctness config: 12L/768/12x64, N(0,0.02) weights
    from seed 0, draft = target layers 0-5, 128-token prompt from seed 1,
    K=4, 64 new tokens, fp32: greedy spec output == greedy autoregressive."""
    torch.set_num_threads(max(1, torch.get_num_threads()))
    w = random_gpt2_weights(GPT2_SMALL, seed=0)
    draft_shape = GPT2Shape(n_layer=6)
    prompt = torch.randint(0, GPT2_SMALL.vocab, (1, 128), generator=torch.Generator().manual_seed(1))
    tgt = GPT2Oracle(GPT2_SMALL, w, batch=1, max_seq=128 + 64 + 12)
    drf = GPT2Oracle(draft_shape, draft_weights_from_target(w, 6), batch=1, max_seq=128 + 64 + 12)
    spec, acc = GPT2ChainSpec(tgt, drf, 4).generate(prompt, 64)
    ar = gpt2_autoregressive(GPT2Oracle(GPT2_SMALL, w, batch=1, max_seq=128 + 64 + 12), prompt, 64)
    assert torch.equal(spec, ar)
    assert acc.float().mean().item() > 0.0  # the copied layers make acceptance non-trivial

"""The CPU oracle against golden vectors produced by the reference's own code.

Fixtures come from tests/golden/make_golden.py (reference modules imported
unmodified, with their two Triton ops restated in torch) and from HF
transformers for the Qwen3 QK-norm the reference lacks.
"""
import torch

from conftest import load_golden
from oracle.qwen import QwenOracle, QwenShape, qwen_model_forward


def _shape(cfg, qk_norm):
    return QwenShape(cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"],
                     cfg["head_dim"], cfg["intermediate_size"], cfg["num_hidden_layers"],
                     cfg["vocab_size"], rope_theta=cfg["rope_theta"], eps=cfg["rms_norm_eps"],
                     qk_norm=qk_norm)


def _run_ref_sequence(fx, dtype):
    st = QwenOracle(_shape(fx["config"], qk_norm=False), fx["weights"], batch=2, max_seq=64, dtype=dtype)
    out = {}
    for tag in ("prefill", "verify", "decode"):
        lg, hd = qwen_model_forward(fx[f"ids_{tag}"], st, return_hidden=True)
        out[tag] = (lg, hd)
    return st, out


def test_qwen_reference_path_bf16_bitexact():
    """Prefill (T=12) and verify (T=5, start 12) equal the reference bit for bit."""
    fx = load_golden("qwen_ref_bf16.pt")
    st, out = _run_ref_sequence(fx, torch.bfloat16)
    for tag in ("prefill", "verify"):
        assert torch.equal(out[tag][0], fx[f"logits_{tag}"]), tag
        assert torch.equal(out[tag][1], fx[f"hidden_{tag}"]), tag
    # T=1 decode: the reference routes through its GQA decode kernel
    # (attention.py:236-318); the oracle uses the same masked verify path.
    d = (out["decode"][0].float() - fx["logits_decode"].float()).abs().max().item()
    assert d <= 2e-2, d
    assert torch.equal(st.k_caches[-1][:, :, :17], fx["k_cache_last"][:, :, :17])
    assert torch.equal(st.v_caches[-1][:, :, :17], fx["v_cache_last"][:, :, :17])


def test_qwen_reference_path_bf16_bitexact_head_dim_128():
    """The same at the library kernels' head dim (128; 2 q heads, 1 kv head):
    the fixture the device is checked against directly."""
    fx = load_golden("qwen_ref_bf16_d128.pt")
    assert fx["config"]["head_dim"] == 128
    st, out = _run_ref_sequence(fx, torch.bfloat16)
    for tag in ("prefill", "verify"):
        assert torch.equal(out[tag][0], fx[f"logits_{tag}"]), tag
        assert torch.equal(out[tag][1], fx[f"hidden_{tag}"]), tag
    d = (out["decode"][0].float() - fx["logits_decode"].float()).abs().max().item()
    assert d <= 2e-2, d


def test_qwen_reference_path_f32():
    fx = load_golden("qwen_ref_f32.pt")
    st, out = _run_ref_sequence(fx, torch.float32)
    for tag in ("prefill", "verify", "decode"):
        d = (out[tag][0] - fx[f"logits_{tag}"]).abs().max().item()
        assert d <= 1e-5, (tag, d)
        d = (out[tag][1] - fx[f"hidden_{tag}"]).abs().max().item()
        assert d <= 1e-5, (tag, d)
    assert (st.k_caches[-1][:, :, :18] - fx["k_cache_last"]).abs().max() <= 1e-6


def test_qwen_qknorm_matches_hf_f32():
    """qk_norm=True reproduces HF Qwen3ForCausalLM (q_norm/k_norm before RoPE)."""
    fx = load_golden("qwen_hf_qknorm_f32.pt")
    st = QwenOracle(_shape(fx["config"], qk_norm=True), fx["weights"], batch=2, max_seq=64,
                    dtype=torch.float32)
    lg, _ = st.forward(fx["ids"])
    d = (lg - fx["logits"]).abs().max().item()
    assert d <= 1e-4, d


def test_qwen_qknorm_verify_equals_prefill_f32():
    """Splitting a sequence into prefill + verify chunks over the cache gives
    the same logits as one prefill (the cache, mask and positions agree)."""
    fx = load_golden("qwen_hf_qknorm_f32.pt")
    st = QwenOracle(_shape(fx["config"], qk_norm=True), fx["weights"], batch=2, max_seq=64,
                    dtype=torch.float32)
    ids = fx["ids"]
    l1, _ = st.forward(ids[:, :10]); st.lengths += 10
    l2, _ = st.forward(ids[:, 10:15]); st.lengths += 5
    l3, _ = st.forward(ids[:, 15:16]); st.lengths += 1
    l4, _ = st.forward(ids[:, 16:18])
    got = torch.cat([l1, l2, l3, l4], dim=1)
    assert (got - fx["logits"]).abs().max().item() <= 1e-4


def test_per_sequence_starts_and_tree_mask_match_chain():
    """Ragged per-sequence starts and a chain-shaped tree mask reproduce the
    shared-start chain path, sequence by sequence."""
    fx = load_golden("qwen_hf_qknorm_f32.pt")
    shape = _shape(fx["config"], qk_norm=True)
    ids = fx["ids"]
    ref = QwenOracle(shape, fx["weights"], batch=2, max_seq=64, dtype=torch.float32)
    full, _ = ref.forward(ids)
    st = QwenOracle(shape, fx["weights"], batch=2, max_seq=64, dtype=torch.float32)
    # sequence 0 prefilled 9 tokens, sequence 1 prefilled 12
    st.forward(ids[:, :12]); st.lengths = torch.tensor([9, 12])
    T = 5
    step = torch.stack([ids[0, 9:9 + T], ids[1, 12:12 + T]])
    mask = torch.tensor([[(1 << (t + 1)) - 1 for t in range(T)]] * 2, dtype=torch.int64)
    lg, _ = st.forward(step, tree_mask=mask,
                       positions=st.lengths.unsqueeze(1) + torch.arange(T).unsqueeze(0))
    assert (lg[0] - full[0, 9:9 + T]).abs().max() <= 1e-4
    assert (lg[1] - full[1, 12:12 + T]).abs().max() <= 1e-4

"""The device path against the reference's own outputs (tests/golden/
qwen_ref_bf16_d128.pt: the reference's Qwen path, QK-norm off, at the
kernels' head dim 128), with no oracle in between.  The CPU oracle
reproduces the same fixture bit for bit (test_oracle_golden.py), so this
pins the device to the reference directly: prefill (T=12), verify (T=5 over
the cache) and decode (T=1), B=2, logits within 2e-2 (bf16) and the argmax
equal wherever the reference's top two logits are more than 2e-2 apart."""

import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _argmax_agrees(got, ref, margin=2e-2):
    top2 = ref.float().topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > margin
    assert torch.equal(got.float().argmax(-1)[clear], ref.float().argmax(-1)[clear])


def test_device_matches_the_reference_path_at_head_dim_128():
    from tri_sds_b200 import ops
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    ops.set_gemv_max_rows(0)
    fx = load_golden("qwen_ref_bf16_d128.pt")
    c = fx["config"]
    shape = QwenShape(c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"],
                      c["intermediate_size"], c["num_hidden_layers"], c["vocab_size"], rope_theta=c["rope_theta"],
                      eps=c["rms_norm_eps"], qk_norm=False)
    B, V = 2, c["vocab_size"]
    m = QwenModel(shape, batch=B, max_seq=64, max_rows=B * 5, device=DEV, weights=fx["weights"], qk_norm=False)
    # prefill: the untimed set-up path (cuBLAS GEMMs, SDPA, the library's RMSNorm and QK-norm/RoPE/KV kernels)
    hidden = m.prefill(fx["ids_prefill"])
    lp = m.logits_of(hidden.reshape(-1, shape.hidden)).reshape(B, -1, V)
    torch.cuda.synchronize()
    assert (lp.float().cpu() - fx["logits_prefill"].float()).abs().max().item() <= 2e-2
    # verify (T=5) and decode (T=1) on the library's kernels
    for tag, T in (("verify", 5), ("decode", 1)):
        ids = fx[f"ids_{tag}"].to(DEV).contiguous()
        am = torch.zeros(B * T, dtype=torch.int64, device=DEV)
        logits = torch.zeros(B * T, V, dtype=torch.bfloat16, device=DEV)
        m.forward_plan(ids, 1, B, T, m.lengths, 0, am, 1, logits_out=logits).run()
        torch.cuda.synchronize()
        m.check_status()
        got = logits.cpu().float().reshape(B, T, V)
        ref = fx[f"logits_{tag}"].float()
        assert (got - ref).abs().max().item() <= 2e-2, tag
        _argmax_agrees(got, ref)
        hid = m.x[:B * T].cpu().float().reshape(B, T, -1)
        href = fx[f"hidden_{tag}"].float()
        assert (hid - href).abs().max().item() <= 5e-2 * href.abs().max().item(), tag
        m.lengths += T   # the reference commits every token of the step

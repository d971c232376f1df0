"""Generate the golden vectors under tests/golden/ from the reference itself.

Run where the reference checkout (read-only) is available, naming its
root in TSDS_REFERENCE:

    TSDS_REFERENCE=<path of the tri-sds checkout> python tests/golden/make_golden.py

The reference's Python modules are imported unmodified.  Its two
Triton-only ops cannot launch on a CPU, so they are replaced by torch
restatements before the model code runs:

* ``norm.rms_norm``          (norm.py:42-72)      -> fp32 stats, one cast;
* ``attention.attention_gqa`` (attention.py:236-318) -> fp32 softmax over
  the first ``kv_len`` cache rows, output cast to q's dtype.

Everything else - weight packing, RoPE, the verify mask, SDPA, the MLP,
the final norm and LM head (qwen_model.py), the EAGLE head and its chain
draft (eagle_head.py), and GPT-2's batched forward (model.py:89-135) -
is the reference's own code.  HF ``transformers`` supplies the Qwen3
QK-norm semantics that the reference lacks.

The fixtures are small (a few hundred KB each) and are committed; the
tests never read the reference checkout.
"""
from __future__ import annotations

import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TSDS_REFERENCE")


def _torch_rms_norm(x, weight, eps=1e-6):
    xf = x.float()
    ms = (xf * xf).sum(-1, keepdim=True) / x.shape[-1]
    rstd = 1.0 / torch.sqrt(ms + eps)
    return (xf * rstd * weight.float()).to(x.dtype)


def _torch_attention_gqa(q, k, v, kv_len, q_per_kv):
    B, Hq, Tq, D = q.shape
    assert Tq == 1
    n = int(kv_len.reshape(-1)[0])
    kf = k[:, :, :n, :].float().repeat_interleave(q_per_kv, dim=1)
    vf = v[:, :, :n, :].float().repeat_interleave(q_per_kv, dim=1)
    s = (q.float() @ kf.transpose(-1, -2)) * (D ** -0.5)
    p = torch.softmax(s, dim=-1)
    return (p @ vf).to(q.dtype)


def _import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "tri_sds")):
        raise SystemExit("set TSDS_REFERENCE to the root of the tri-sds checkout (the directory holding tri_sds/)")
    sys.path.insert(0, REF)
    import tri_sds.triton_kernels.qwen_model as rq
    import tri_sds.triton_kernels.eagle_head as re
    import tri_sds.triton_kernels.model as rm
    rq.rms_norm = _torch_rms_norm
    rq.attention_gqa = _torch_attention_gqa
    re.rms_norm = _torch_rms_norm
    return rq, re, rm


QWEN_CFG = dict(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                max_position_embeddings=64, rope_theta=1.0e6, rms_norm_eps=1e-6,
                tie_word_embeddings=False)


# the library's kernels take head dim 128 only: the same reference path at
# that head dim, for checking the device directly against the reference
QWEN_D128_CFG = dict(vocab_size=512, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                     num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                     max_position_embeddings=64, rope_theta=1.0e6, rms_norm_eps=1e-6,
                     tie_word_embeddings=False)


def _hf_qwen(dtype, seed=0, qk_norm_gain=None, cfg_dict=None):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(**(cfg_dict or QWEN_CFG))
    m = Qwen3ForCausalLM(cfg)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("norm.weight"):
                p.copy_(1.0 + 0.05 * torch.randn_like(p))
            else:
                p.copy_(0.02 * torch.randn_like(p))
    return m.to(dtype).eval()


def make_qwen(dtype, tag, cfg_dict=None):
    """Reference Qwen path (QK-norm off): prefill T=12, verify T=5, decode T=1, B=2."""
    rq, _, _ = _import_reference()
    cfg_dict = cfg_dict or QWEN_CFG
    m = _hf_qwen(dtype, cfg_dict=cfg_dict)
    V = cfg_dict["vocab_size"]
    st = rq.QwenModelState(m, max_seq_len=64)
    if dtype != torch.bfloat16:
        # qwen_model.py:38 fixes the cache / RoPE-table dtype to bf16; the fp32
        # fixture rebuilds both in fp32 with the reference's own precompute_rope.
        st.dtype = dtype
        st.cos, st.sin = rq.precompute_rope(st.D, st.max_seq_len, base=1.0e6, device="cpu", dtype=dtype)
    st.reset_cache(batch_size=2)
    g = torch.Generator().manual_seed(1)
    ids_prefill = torch.randint(0, V, (2, 12), generator=g)
    ids_verify = torch.randint(0, V, (2, 5), generator=g)
    ids_decode = torch.randint(0, V, (2, 1), generator=g)
    with torch.no_grad():
        lp, hp = rq.qwen_model_forward(ids_prefill, st, return_hidden=True)
        lv, hv = rq.qwen_model_forward(ids_verify, st, return_hidden=True)
        ld, hd = rq.qwen_model_forward(ids_decode, st, return_hidden=True)
    from oracle.qwen import weights_from_hf
    out = {
        "config": cfg_dict, "dtype": str(dtype),
        "weights": weights_from_hf(m),
        "ids_prefill": ids_prefill, "ids_verify": ids_verify, "ids_decode": ids_decode,
        "logits_prefill": lp, "hidden_prefill": hp,
        "logits_verify": lv, "hidden_verify": hv,
        "logits_decode": ld, "hidden_decode": hd,
        "k_cache_last": st.k_caches[-1][:, :, :18].clone(),
        "v_cache_last": st.v_caches[-1][:, :, :18].clone(),
    }
    torch.save(out, os.path.join(HERE, f"qwen_ref_{tag}.pt"))


def make_qwen_hf_qknorm():
    """HF Qwen3 (with q_norm/k_norm) over the same 18 tokens, fp32."""
    m = _hf_qwen(torch.float32, seed=2)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 512, (2, 18), generator=g)
    with torch.no_grad():
        out = m(input_ids=ids, output_hidden_states=True)
    from oracle.qwen import weights_from_hf
    torch.save({"config": QWEN_CFG, "weights": weights_from_hf(m), "ids": ids,
                "logits": out.logits.detach()}, os.path.join(HERE, "qwen_hf_qknorm_f32.pt"))


def make_eagle():
    """Reference EagleHead.forward + eagle_draft_decode (eagle_head.py:16-129)."""
    rq, re, _ = _import_reference()
    m = _hf_qwen(torch.float32, seed=4)
    st = rq.QwenModelState(m, max_seq_len=64)
    N, I = QWEN_CFG["hidden_size"], 192
    g = torch.Generator().manual_seed(5)
    sd = {
        "fc.weight": 0.02 * torch.randn(2 * N, N, generator=g),      # stored [in, out]
        "fc.bias": 0.02 * torch.randn(N, generator=g),
        "attn.norm.weight": 1 + 0.05 * torch.randn(N, generator=g),
        "attn.q_proj.weight": 0.02 * torch.randn(N, N, generator=g),  # stored [in, out]
        "attn.k_proj.weight": 0.02 * torch.randn(N, N, generator=g),
        "attn.v_proj.weight": 0.02 * torch.randn(N, N, generator=g),
        "attn.o_proj.weight": 0.02 * torch.randn(N, N, generator=g),  # stored [out, in]
        "ffn.norm.weight": 1 + 0.05 * torch.randn(N, generator=g),
        "ffn.gate_proj.weight": 0.02 * torch.randn(I, N, generator=g),
        "ffn.up_proj.weight": 0.02 * torch.randn(I, N, generator=g),
        "ffn.down_proj.weight": 0.02 * torch.randn(N, I, generator=g),
    }
    head = re.EagleHead(N, I, device="cpu", dtype=torch.float32)
    head.load_state_dict(sd)
    feats = torch.randn(2, 6, N, generator=g)
    toks = torch.randint(0, 512, (2, 6), generator=g)
    with torch.no_grad():
        fwd = head.forward(feats, st.embed_w[toks])
        last_hidden = torch.randn(2, 1, N, generator=g)
        last_token = torch.randint(0, 512, (2, 1), generator=g)
        d_tok, d_log = re.eagle_draft_decode(last_hidden, last_token, head, st, n_draft=4)
    from oracle.qwen import weights_from_hf
    tw = weights_from_hf(m)
    tw = {"embed": tw["embed"], "lm_head": tw["lm_head"], "norm": tw["norm"]}
    torch.save({"config": QWEN_CFG, "target_weights": tw, "state_dict": sd,
                "intermediate": I, "feats": feats, "toks": toks, "forward": fwd,
                "last_hidden": last_hidden, "last_token": last_token,
                "draft_tokens": torch.cat(d_tok, dim=1), "draft_logits": torch.stack(d_log, dim=1)},
               os.path.join(HERE, "eagle_ref_f32.pt"))


def make_gpt2():
    """Reference GPT-2 batched forward (model.py:16-135) at start 0, fp32."""
    _, _, rm = _import_reference()
    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(6)
    cfg = GPT2Config(vocab_size=300, n_positions=64, n_embd=64, n_layer=2, n_head=4)
    m = GPT2LMHeadModel(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("ln_1.weight") or n.endswith("ln_2.weight") or n.endswith("ln_f.weight"):
                p.copy_(1 + 0.05 * torch.randn_like(p))
            else:
                p.copy_(0.02 * torch.randn_like(p))
    sd = {n: p.detach().clone() for n, p in m.named_parameters()}
    blocks = []
    for i in range(cfg.n_layer):
        b = m.transformer.h[i]
        blocks.append((b.ln_1.weight, b.ln_1.bias, b.attn.c_attn.weight, b.attn.c_attn.bias,
                       b.attn.c_proj.weight, b.attn.c_proj.bias, b.ln_2.weight, b.ln_2.bias,
                       b.mlp.c_fc.weight, b.mlp.c_fc.bias, b.mlp.c_proj.weight, b.mlp.c_proj.bias))
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 300, (1, 10), generator=g)
    pos = torch.arange(10).unsqueeze(0)
    kc = [torch.zeros(1, 4, 64, 16) for _ in range(2)]
    vc = [torch.zeros(1, 4, 64, 16) for _ in range(2)]
    with torch.no_grad():
        logits = rm.model_forward(ids, pos, m.transformer.wte.weight, m.transformer.wpe.weight, blocks,
                                  m.transformer.ln_f.weight, m.transformer.ln_f.bias, kc, vc, 4)
        hf = m(input_ids=ids).logits
    torch.save({"config": cfg.to_dict(), "state_dict": sd, "ids": ids, "logits": logits,
                "hf_logits": hf, "k_cache0": kc[0][:, :, :10].clone()},
               os.path.join(HERE, "gpt2_ref_f32.pt"))


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    make_qwen(torch.bfloat16, "bf16")
    make_qwen(torch.float32, "f32")
    make_qwen(torch.bfloat16, "bf16_d128", QWEN_D128_CFG)
    make_qwen_hf_qknorm()
    make_eagle()
    make_gpt2()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))

"""CPU restatement of the reference's Qwen3 forward (test infrastructure).

Follows ``tri_sds/triton_kernels/qwen_model.py`` of the reference:

* weight packing ``QwenModelState.__init__`` (qwen_model.py:27-84): fused
  ``qkv_w_t = cat(q,k,v).T``, ``o_w_t``, ``gate_up_w_t = cat(gate,up).T``,
  ``down_w_t``;
* RoPE tables and rotation ``precompute_rope`` / ``apply_rope``
  (qwen_model.py:8-24): fp32 angles, bf16 tables, bf16 element-wise math;
* the verify / prefill layer ``_qwen_prefill`` (qwen_model.py:100-146),
  including the reference's additive mask (value 1.0 on visible keys, -inf
  elsewhere, qwen_model.py:124-129) and ``repeat_interleave`` of the cache;
* dispatch, final RMSNorm and LM head ``qwen_model_forward``
  (qwen_model.py:183-209);
* RMSNorm of ``norm.py:42-72``: fp32 statistics, ``x*rstd*w`` in fp32,
  a single cast to the output dtype.

Additions the reference lacks, each a flag or argument:

* ``qk_norm``: Qwen3's per-head q_norm / k_norm between the projection and
  RoPE (HF ``Qwen3Attention`` order).  The reference never loads them
  (qwen_model.py:46-84); ``qk_norm=False`` is the strict reference path.
  The norm itself uses the same single-cast RMSNorm as norm.py:42-72.
* per-sequence cache lengths ``starts[B]`` (the reference keeps one scalar
  ``_prefilled``, qwen_model.py:94,185);
* a tree mask: ``tree_mask[b, t]`` is a bitmask over the T new tokens, bit
  j set when new token j is visible to new token t (ancestor or self).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class QwenShape:
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    n_layers: int
    vocab: int
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6
    qk_norm: bool = True
    tie_embeddings: bool = False

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def q_per_kv(self) -> int:
        return self.n_heads // self.n_kv_heads


# Layer shapes of the two model families the workloads name.
QWEN3_32B = QwenShape(5120, 64, 8, 128, 25600, 64, 151936)
QWEN3_4B = QwenShape(2560, 32, 8, 128, 9728, 36, 151936, tie_embeddings=True)


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------

LAYER_KEYS = ("q", "k", "v", "o", "gate", "up", "down", "ln1", "ln2", "q_norm", "k_norm")


def random_qwen_weights(shape: QwenShape, seed: int, dtype=torch.bfloat16, std: float = 0.02,
                        gain_std: float = 0.02) -> dict:
    """Seeded random weights in HF layout ([out, in] matrices).

    Matrices are N(0, std); norm gains are N(1, gain_std).  Generated on the
    CPU so that the same seed gives the same tensors on every machine.
    """
    g = torch.Generator().manual_seed(seed)
    N, D, I = shape.hidden, shape.head_dim, shape.intermediate

    def mat(o, i):
        return (torch.randn(o, i, generator=g) * std).to(dtype)

    def gain(n):
        return (1.0 + torch.randn(n, generator=g) * gain_std).to(dtype)

    layers = []
    for _ in range(shape.n_layers):
        layers.append({
            "q": mat(shape.q_dim, N), "k": mat(shape.kv_dim, N), "v": mat(shape.kv_dim, N),
            "o": mat(N, shape.q_dim),
            "gate": mat(I, N), "up": mat(I, N), "down": mat(N, I),
            "ln1": gain(N), "ln2": gain(N), "q_norm": gain(D), "k_norm": gain(D),
        })
    embed = mat(shape.vocab, N)
    lm_head = embed if shape.tie_embeddings else mat(shape.vocab, N)
    return {"embed": embed, "lm_head": lm_head, "norm": gain(N), "layers": layers}


def weights_from_hf(hf_model) -> dict:
    """Collect an HF ``Qwen3ForCausalLM``'s parameters (qwen_model.py:46-84 names)."""
    p = dict(hf_model.named_parameters())
    cfg = hf_model.config
    layers = []
    for i in range(cfg.num_hidden_layers):
        lp = f"model.layers.{i}."
        layers.append({
            "q": p[lp + "self_attn.q_proj.weight"].detach(),
            "k": p[lp + "self_attn.k_proj.weight"].detach(),
            "v": p[lp + "self_attn.v_proj.weight"].detach(),
            "o": p[lp + "self_attn.o_proj.weight"].detach(),
            "gate": p[lp + "mlp.gate_proj.weight"].detach(),
            "up": p[lp + "mlp.up_proj.weight"].detach(),
            "down": p[lp + "mlp.down_proj.weight"].detach(),
            "ln1": p[lp + "input_layernorm.weight"].detach(),
            "ln2": p[lp + "post_attention_layernorm.weight"].detach(),
            "q_norm": p[lp + "self_attn.q_norm.weight"].detach(),
            "k_norm": p[lp + "self_attn.k_norm.weight"].detach(),
        })
    embed = p["model.embed_tokens.weight"].detach()
    lm_head = p["lm_head.weight"].detach() if "lm_head.weight" in p else embed
    return {"embed": embed, "lm_head": lm_head, "norm": p["model.norm.weight"].detach(),
            "layers": layers}


# ---------------------------------------------------------------------------
# element-wise pieces
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """norm.py:42-72: fp32 mean of squares, ``rstd = 1/sqrt(ms+eps)``,
    ``y = x*rstd*w`` in fp32, one cast to ``x.dtype``.  Any leading shape."""
    xf = x.float()
    ms = (xf * xf).sum(-1, keepdim=True) / x.shape[-1]
    rstd = 1.0 / torch.sqrt(ms + eps)
    return (xf * rstd * w.float()).to(x.dtype)


def precompute_rope(dim: int, max_len: int, base: float = 1.0e6, dtype=torch.bfloat16):
    """qwen_model.py:8-14: fp32 inverse frequencies and angles, tables cast to ``dtype``."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(max_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """qwen_model.py:17-24 rotate-half RoPE in the tables' dtype.

    ``x`` is [B, H, T, D]; ``pos`` is [T] (shared, as in the reference) or
    [B, T] (per sequence)."""
    half = x.shape[-1] // 2
    if pos.dim() == 1:
        c = cos[pos].view(1, 1, pos.shape[0], half)
        s = sin[pos].view(1, 1, pos.shape[0], half)
    else:
        c = cos[pos].view(pos.shape[0], 1, pos.shape[1], half)
        s = sin[pos].view(pos.shape[0], 1, pos.shape[1], half)
    x1 = x[..., :half]
    x2 = x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def chain_tree_mask(T: int) -> list[int]:
    """The causal mask among T new tokens as tree bitmasks: token t sees 0..t."""
    return [(1 << (t + 1)) - 1 for t in range(T)]


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     starts: torch.Tensor, tree_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of T new query tokens over the cache (qwen_model.py:121-131).

    q: [B, Hq, T, D] (RoPE applied); k_cache/v_cache: [B, Hkv, S, D] with the
    new tokens already written at rows ``starts[b] .. starts[b]+T-1``.
    Query t of sequence b sees every cached row below ``starts[b]`` plus the
    new rows its mask allows (causal: rows ``starts[b]..starts[b]+t``).
    Returns [B, Hq, T, D] in q's dtype.
    """
    B, Hq, T, D = q.shape
    q_per_kv = Hq // k_cache.shape[1]
    starts = [int(s) for s in starts]
    if tree_mask is None and all(s == starts[0] for s in starts):
        # the reference's own batched call, unchanged
        start = starts[0]
        kv_len = start + T
        k_full = k_cache[:, :, :kv_len, :].repeat_interleave(q_per_kv, dim=1)
        v_full = v_cache[:, :, :kv_len, :].repeat_interleave(q_per_kv, dim=1)
        if start > 0:
            s = torch.arange(kv_len)
            t = torch.arange(T).unsqueeze(1)
            mask = (s.unsqueeze(0) <= start + t).to(q.dtype)
            mask = mask.masked_fill(mask == 0, float("-inf"))
            return F.scaled_dot_product_attention(q, k_full, v_full, attn_mask=mask)
        return F.scaled_dot_product_attention(q, k_full, v_full, is_causal=True)
    outs = []
    for b in range(B):
        start = starts[b]
        kv_len = start + T
        k_full = k_cache[b:b + 1, :, :kv_len, :].repeat_interleave(q_per_kv, dim=1)
        v_full = v_cache[b:b + 1, :, :kv_len, :].repeat_interleave(q_per_kv, dim=1)
        s = torch.arange(kv_len).unsqueeze(0)
        t = torch.arange(T).unsqueeze(1)
        if tree_mask is None:
            vis = s <= start + t
        else:
            bits = tree_mask[b].to(torch.int64).unsqueeze(1)
            j = (s - start).clamp(min=0)
            vis = (s < start) | (((bits >> j) & 1) == 1)
        mask = vis.to(q.dtype).masked_fill(~vis, float("-inf"))
        outs.append(F.scaled_dot_product_attention(q[b:b + 1], k_full, v_full, attn_mask=mask))
    return torch.cat(outs, dim=0)


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------

class QwenOracle:
    """Model state: packed weights + per-layer KV cache + per-sequence lengths.

    Mirrors ``QwenModelState`` (qwen_model.py:27-97).  ``lengths[b]`` is the
    number of committed cache rows of sequence b.
    """

    def __init__(self, shape: QwenShape, weights: dict, batch: int, max_seq: int,
                 dtype=torch.bfloat16):
        self.shape = shape
        self.dtype = dtype
        self.batch = batch
        self.max_seq = max_seq
        cv = lambda t: t.to(dtype)  # noqa: E731
        self.embed_w = cv(weights["embed"])
        self.lm_head_w = cv(weights["lm_head"])
        self.norm_w = cv(weights["norm"])
        self.cos, self.sin = precompute_rope(shape.head_dim, max_seq, shape.rope_theta, dtype)
        self.qkv_w_t, self.o_w_t, self.gate_up_w_t, self.down_w_t = [], [], [], []
        self.norm1_w, self.norm2_w, self.q_norm_w, self.k_norm_w = [], [], [], []
        for L in weights["layers"]:
            self.norm1_w.append(cv(L["ln1"]))
            self.norm2_w.append(cv(L["ln2"]))
            self.q_norm_w.append(cv(L["q_norm"]))
            self.k_norm_w.append(cv(L["k_norm"]))
            self.qkv_w_t.append(torch.cat([cv(L["q"]), cv(L["k"]), cv(L["v"])], dim=0).T.contiguous())
            self.o_w_t.append(cv(L["o"]).T.contiguous())
            self.gate_up_w_t.append(torch.cat([cv(L["gate"]), cv(L["up"])], dim=0).T.contiguous())
            self.down_w_t.append(cv(L["down"]).T.contiguous())
        self.reset_cache()

    def reset_cache(self):
        """qwen_model.py:86-94, with per-sequence lengths."""
        s = self.shape
        self.k_caches = [torch.zeros(self.batch, s.n_kv_heads, self.max_seq, s.head_dim, dtype=self.dtype)
                         for _ in range(s.n_layers)]
        self.v_caches = [torch.zeros_like(k) for k in self.k_caches]
        self.lengths = torch.zeros(self.batch, dtype=torch.int64)

    # -- one decoder layer (qwen_model.py:104-144) --------------------------
    def layer(self, i: int, x: torch.Tensor, starts: torch.Tensor, positions: torch.Tensor,
              tree_mask: torch.Tensor | None) -> torch.Tensor:
        s = self.shape
        B, T, N = x.shape
        x_norm = rms_norm(x.reshape(B * T, N), self.norm1_w[i], s.eps).reshape(B, T, N)
        qkv = x_norm @ self.qkv_w_t[i]
        q = qkv[..., :s.q_dim].reshape(B, T, s.n_heads, s.head_dim)
        k = qkv[..., s.q_dim:s.q_dim + s.kv_dim].reshape(B, T, s.n_kv_heads, s.head_dim)
        v = qkv[..., s.q_dim + s.kv_dim:].reshape(B, T, s.n_kv_heads, s.head_dim)
        if s.qk_norm:
            q = rms_norm(q, self.q_norm_w[i], s.eps)
            k = rms_norm(k, self.k_norm_w[i], s.eps)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        q = apply_rope(q, self.cos, self.sin, positions)
        k = apply_rope(k, self.cos, self.sin, positions)
        for b in range(B):
            st = int(starts[b])
            self.k_caches[i][b, :, st:st + T, :] = k[b]
            self.v_caches[i][b, :, st:st + T, :] = v[b]
        attn = verify_attention(q, self.k_caches[i], self.v_caches[i], starts, tree_mask)
        attn_flat = attn.transpose(1, 2).reshape(B * T, s.q_dim)
        x = x + (attn_flat @ self.o_w_t[i]).reshape(B, T, N)
        x_norm2 = rms_norm(x.reshape(B * T, N), self.norm2_w[i], s.eps).reshape(B, T, N)
        gate_up = x_norm2 @ self.gate_up_w_t[i]
        hidden = F.silu(gate_up[..., :s.intermediate]) * gate_up[..., s.intermediate:]
        return x + hidden @ self.down_w_t[i]

    def forward(self, ids: torch.Tensor, starts: torch.Tensor | None = None,
                positions: torch.Tensor | None = None, tree_mask: torch.Tensor | None = None,
                embeds: torch.Tensor | None = None):
        """Run T new tokens per sequence; writes their K/V at rows
        ``starts[b]..starts[b]+T-1`` and returns (logits [B,T,V], hidden [B,T,N]).

        ``lengths`` is not changed: the caller commits.  ``positions`` default
        to ``starts[b] + t`` (chain); tree callers pass ``starts[b] + depth``.
        """
        B, T = ids.shape
        starts = self.lengths.clone() if starts is None else starts.to(torch.int64)
        if positions is None:
            positions = starts.unsqueeze(1) + torch.arange(T).unsqueeze(0)
        if bool((starts == starts[0]).all()) and tree_mask is None:
            positions_arg = positions[0]          # the reference's shared [T] positions
        else:
            positions_arg = positions
        x = self.embed_w[ids] if embeds is None else embeds.to(self.dtype)
        for i in range(self.shape.n_layers):
            x = self.layer(i, x, starts, positions_arg, tree_mask)
        hidden = x
        logits = self.logits(hidden)
        return logits, hidden

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Final RMSNorm + LM head (qwen_model.py:191-193)."""
        B, T, N = hidden.shape
        x_flat = rms_norm(hidden.reshape(B * T, N), self.norm_w, self.shape.eps)
        return (x_flat @ self.lm_head_w.T).reshape(B, T, -1)


def qwen_model_forward(input_ids: torch.Tensor, state: QwenOracle, return_hidden: bool = False):
    """qwen_model.py:183-209: one shared start position, advanced by T."""
    logits, hidden = state.forward(input_ids)
    state.lengths += input_ids.shape[1]
    return (logits, hidden) if return_hidden else logits


def greedy_argmax(logits: torch.Tensor) -> torch.Tensor:
    """``torch.argmax`` over the last axis: the lowest index wins a tie."""
    return logits.argmax(dim=-1)

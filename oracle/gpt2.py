"""CPU restatement of the reference's GPT-2 path (test infrastructure).

Follows ``tri_sds/triton_kernels/model.py:16-135`` (``model_forward`` and
``_prefill_batched``) and ``draft_step.py:13-85``: learned positions, pre-LN
blocks with LayerNorm eps 1e-5 (``norm.py:6-39``), Conv1D projections
(``x @ W + b`` with ``W`` stored ``[in, out]``), erf GELU (``F.gelu``,
``model.py:121``), tied LM head.

One deliberate difference, named here because the config asks for a
correctness check the reference path cannot pass: the reference's T>1 path
calls ``F.scaled_dot_product_attention(q, k, v, is_causal=True)`` over the
new tokens only (``model.py:113``), ignoring the cache, so a K+1-token verify
step after a prefill attends to nothing before it.  ``forward`` here writes
the new K/V at ``start..start+T-1`` and attends over the whole cache with
the offset causal mask; at ``start == 0`` the two coincide (checked against
the reference's own output in ``tests/test_oracle_gpt2.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class GPT2Shape:
    n_layer: int = 12
    n_embd: int = 768
    n_head: int = 12
    n_inner: int = 3072
    n_positions: int = 1024
    vocab: int = 50257
    eps: float = 1e-5


GPT2_SMALL = GPT2Shape()


def random_gpt2_weights(shape: GPT2Shape, seed: int, std: float = 0.02) -> dict:
    """N(0, std) matrices and embeddings, LayerNorm gains 1 and biases 0 (HF init)."""
    g = torch.Generator().manual_seed(seed)
    N, I = shape.n_embd, shape.n_inner

    def mat(*s):
        return torch.randn(*s, generator=g) * std

    blocks = []
    for _ in range(shape.n_layer):
        blocks.append({
            "ln_1.weight": torch.ones(N), "ln_1.bias": torch.zeros(N),
            "attn.c_attn.weight": mat(N, 3 * N), "attn.c_attn.bias": torch.zeros(3 * N),
            "attn.c_proj.weight": mat(N, N), "attn.c_proj.bias": torch.zeros(N),
            "ln_2.weight": torch.ones(N), "ln_2.bias": torch.zeros(N),
            "mlp.c_fc.weight": mat(N, I), "mlp.c_fc.bias": torch.zeros(I),
            "mlp.c_proj.weight": mat(I, N), "mlp.c_proj.bias": torch.zeros(N),
        })
    return {"wte": mat(shape.vocab, N), "wpe": mat(shape.n_positions, N), "ln_f.weight": torch.ones(N),
            "ln_f.bias": torch.zeros(N), "blocks": blocks}


def weights_from_state_dict(sd: dict, n_layer: int) -> dict:
    """HF ``GPT2LMHeadModel`` parameter names -> the dict used here."""
    blocks = []
    for i in range(n_layer):
        p = f"transformer.h.{i}."
        blocks.append({k: sd[p + k] for k in (
            "ln_1.weight", "ln_1.bias", "attn.c_attn.weight", "attn.c_attn.bias", "attn.c_proj.weight",
            "attn.c_proj.bias", "ln_2.weight", "ln_2.bias", "mlp.c_fc.weight", "mlp.c_fc.bias",
            "mlp.c_proj.weight", "mlp.c_proj.bias")})
    return {"wte": sd["transformer.wte.weight"], "wpe": sd["transformer.wpe.weight"],
            "ln_f.weight": sd["transformer.ln_f.weight"], "ln_f.bias": sd["transformer.ln_f.bias"],
            "blocks": blocks}


class GPT2Oracle:
    """GPT-2 with a per-layer KV cache ``[B, H, S, D]`` (draft_step.py:58-66)
    and per-sequence committed lengths."""

    def __init__(self, shape: GPT2Shape, weights: dict, batch: int, max_seq: int | None = None,
                 dtype=torch.float32):
        self.shape, self.w, self.batch, self.dtype = shape, weights, batch, dtype
        self.max_seq = max_seq or shape.n_positions
        self.reset_cache()

    def reset_cache(self):
        s = self.shape
        D = s.n_embd // s.n_head
        self.k = [torch.zeros(self.batch, s.n_head, self.max_seq, D, dtype=self.dtype) for _ in range(s.n_layer)]
        self.v = [torch.zeros_like(t) for t in self.k]
        self.lengths = torch.zeros(self.batch, dtype=torch.int64)

    def forward(self, ids: torch.Tensor, starts: torch.Tensor | None = None) -> torch.Tensor:
        """T new tokens at rows starts[b].. (model.py:37,89-135); returns logits [B, T, V]."""
        s = self.shape
        B, T = ids.shape
        N, H = s.n_embd, s.n_head
        D = N // H
        starts = self.lengths.clone() if starts is None else starts.to(torch.int64)
        pos = starts.unsqueeze(1) + torch.arange(T).unsqueeze(0)
        x = self.w["wte"][ids] + self.w["wpe"][pos]
        for i, blk in enumerate(self.w["blocks"]):
            xn = F.layer_norm(x, (N,), blk["ln_1.weight"], blk["ln_1.bias"], s.eps)
            qkv = xn @ blk["attn.c_attn.weight"] + blk["attn.c_attn.bias"]
            q, k, v = qkv.split(N, dim=-1)
            q = q.reshape(B, T, H, D).transpose(1, 2)
            k = k.reshape(B, T, H, D).transpose(1, 2)
            v = v.reshape(B, T, H, D).transpose(1, 2)
            outs = []
            for b in range(B):
                st = int(starts[b])
                self.k[i][b, :, st:st + T] = k[b]
                self.v[i][b, :, st:st + T] = v[b]
                L = st + T
                key = torch.arange(L).unsqueeze(0)
                vis = key <= st + torch.arange(T).unsqueeze(1)
                mask = torch.zeros(T, L, dtype=x.dtype).masked_fill(~vis, float("-inf"))
                outs.append(F.scaled_dot_product_attention(q[b:b + 1], self.k[i][b:b + 1, :, :L],
                                                           self.v[i][b:b + 1, :, :L], attn_mask=mask))
            attn = torch.cat(outs).transpose(1, 2).reshape(B, T, N)
            x = x + (attn @ blk["attn.c_proj.weight"] + blk["attn.c_proj.bias"])
            xn2 = F.layer_norm(x, (N,), blk["ln_2.weight"], blk["ln_2.bias"], s.eps)
            h = F.gelu(xn2 @ blk["mlp.c_fc.weight"] + blk["mlp.c_fc.bias"])
            x = x + (h @ blk["mlp.c_proj.weight"] + blk["mlp.c_proj.bias"])
        x = F.layer_norm(x, (N,), self.w["ln_f.weight"], self.w["ln_f.bias"], s.eps)
        return x @ self.w["wte"].T


def draft_weights_from_target(w: dict, n_layer: int) -> dict:
    """A draft sharing the target's embeddings and its first n_layer blocks."""
    return {**w, "blocks": w["blocks"][:n_layer]}


class GPT2ChainSpec:
    """The chain cycle of ``oracle/spec.py`` with GPT-2 models."""

    def __init__(self, target: GPT2Oracle, draft: GPT2Oracle, k: int):
        self.target, self.draft, self.k = target, draft, k

    def generate(self, prompt: torch.Tensor, n_new: int):
        t, d, K = self.target, self.draft, self.k
        B, P = prompt.shape
        t.reset_cache()
        d.reset_cache()
        logits = t.forward(prompt)
        t.lengths[:] = P
        if P > 1:
            d.forward(prompt[:, :P - 1])
        last, cur = prompt[:, -1].clone(), logits[:, -1].argmax(-1)
        out = [[int(cur[b])] for b in range(B)]
        accepts = []
        while min(len(o) for o in out) < n_new:
            L = t.lengths.clone()
            lg = d.forward(torch.stack([last, cur], 1), starts=L - 1)
            drafts = [lg[:, -1].argmax(-1)]
            for i in range(2, K + 1):
                lg = d.forward(drafts[-1].unsqueeze(1), starts=L + i - 1)
                drafts.append(lg[:, -1].argmax(-1))
            dr = torch.stack(drafts, 1)
            y = t.forward(torch.cat([cur.unsqueeze(1), dr], 1), starts=L).argmax(-1)
            match = (dr == y[:, :K]).to(torch.int64)
            n = torch.cumprod(match, 1).sum(1)
            accepts.append(n.clone())
            bi = torch.arange(B)
            for b in range(B):
                out[b].extend(int(x) for x in y[b, :int(n[b]) + 1])
            t.lengths = L + n + 1
            last = torch.where(n == 0, cur, dr[bi, (n - 1).clamp(min=0)])
            cur = y[bi, n]
        return torch.tensor([o[:n_new] for o in out]), torch.stack(accepts)


def gpt2_autoregressive(target: GPT2Oracle, prompt: torch.Tensor, n_new: int) -> torch.Tensor:
    B, P = prompt.shape
    target.reset_cache()
    logits = target.forward(prompt)
    target.lengths[:] = P
    tok = logits[:, -1].argmax(-1)
    out = [tok]
    for _ in range(n_new - 1):
        logits = target.forward(tok.unsqueeze(1))
        target.lengths += 1
        tok = logits[:, -1].argmax(-1)
        out.append(tok)
    return torch.stack(out, 1)

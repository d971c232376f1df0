"""Qwen3 model state on the GPU and its verify / decode forward.

The device-side counterpart of ``QwenModelState`` + ``qwen_model_forward``
(qwen_model.py:27-209).  Differences by design:

* weights stay in the HF ``[out, in]`` layout (the kernels stream rows of
  ``in``); q/k/v and gate/up are concatenated like the reference's packing
  (qwen_model.py:75-84) but not transposed;
* one KV-cache tensor ``[layers, B, Hkv, S, D]`` and per-sequence committed
  lengths on the device (the reference keeps one host scalar);
* a forward is a fixed *launch plan* - a list of C-ABI calls with every
  pointer bound - so one speculative cycle can be captured in a CUDA graph;
* Qwen3's QK-norm (HF order: projection -> q/k RMSNorm -> RoPE).

The prompt prefill (untimed set-up) runs through cuBLAS GEMMs and SDPA,
with the cache written by the same QK-norm/RoPE/KV kernel as the
verify path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _lib
from .shapes import QwenShape

_VP = ctypes.c_void_p


def _p(t):
    return None if t is None else _VP(t.data_ptr())


def precompute_rope(dim: int, max_len: int, base: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """qwen_model.py:8-14: fp32 angles on the host, bf16 tables."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(max_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return (freqs.cos().to(torch.bfloat16).to(device).contiguous(),
            freqs.sin().to(torch.bfloat16).to(device).contiguous())


@dataclass
class LayerWeights:
    w_qkv: torch.Tensor   # [q_dim + 2 kv_dim, N]
    w_o: torch.Tensor     # [N, q_dim]
    w_gu: torch.Tensor    # [2 I, N]
    w_d: torch.Tensor     # [N, I]
    ln1: torch.Tensor
    ln2: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


def pack_layer(L: dict, device) -> LayerWeights:
    bf = lambda t: t.to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    return LayerWeights(
        w_qkv=torch.cat([bf(L["q"]), bf(L["k"]), bf(L["v"])], dim=0).contiguous(),
        w_o=bf(L["o"]), w_gu=torch.cat([bf(L["gate"]), bf(L["up"])], dim=0).contiguous(), w_d=bf(L["down"]),
        ln1=bf(L["ln1"]), ln2=bf(L["ln2"]), q_norm=bf(L["q_norm"]), k_norm=bf(L["k_norm"]))


def random_layer_gpu(shape: QwenShape, gen: torch.Generator, device, std=0.02, gain_std=0.02) -> LayerWeights:
    """N(0, std) matrices and N(1, gain_std) gains drawn on the device."""
    N, I = shape.hidden, shape.intermediate

    def mat(o, i):
        return (torch.randn(o, i, device=device, generator=gen, dtype=torch.float32) * std).to(torch.bfloat16)

    def gain(n):
        return (1.0 + gain_std * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    return LayerWeights(w_qkv=mat(shape.qkv_dim, N), w_o=mat(N, shape.q_dim), w_gu=mat(2 * I, N),
                        w_d=mat(N, I), ln1=gain(N), ln2=gain(N), q_norm=gain(shape.head_dim),
                        k_norm=gain(shape.head_dim))


@dataclass
class Plan:
    """A bound sequence of C-ABI calls; ``run`` appends the stream."""
    calls: list = field(default_factory=list)

    def add(self, name: str, *args):
        self.calls.append((name, getattr(_lib.load(), name), args))

    def extend(self, other: "Plan"):
        self.calls.extend(other.calls)

    def run(self, stream=None):
        s = _VP(torch.cuda.current_stream().cuda_stream if stream is None else stream)
        lib = _lib.load()
        for name, fn, args in self.calls:
            st = fn(*args, s)
            if st != 0:
                raise RuntimeError(f"{name} failed: status {st} ({lib.tsds_status_string(st).decode()})")

    def kernel_count(self) -> int:
        return len(self.calls)


class QwenModel:
    """Weights, KV cache and activation buffers of one Qwen3-shaped model.

    ``max_rows`` bounds the token rows of one forward (B * T).
    """

    def __init__(self, shape: QwenShape, batch: int, max_seq: int, max_rows: int, device="cuda",
                 weights: dict | None = None, seed: int = 0, split_keys: int = 256, qk_norm: bool | None = None,
                 share_embeddings: "QwenModel | None" = None, rope_len: int | None = None):
        self.shape = shape
        self.batch = batch
        self.max_seq = max_seq
        self.max_rows = max_rows
        self.device = torch.device(device)
        self.split_keys = split_keys
        self.qk_norm = shape.qk_norm if qk_norm is None else qk_norm
        s = shape
        dev = self.device
        if weights is not None:
            self.layers = [pack_layer(L, dev) for L in weights["layers"]]
        else:
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed)
            self.layers = [random_layer_gpu(s, gen, dev) for _ in range(s.n_layers)]
        if share_embeddings is not None:
            # the EAGLE head runs on the target's embedding, final norm and LM head
            self.embed_w, self.lm_head_w, self.norm_w = (share_embeddings.embed_w, share_embeddings.lm_head_w,
                                                         share_embeddings.norm_w)
        elif weights is not None:
            self.embed_w = weights["embed"].to(dev, torch.bfloat16).contiguous()
            self.lm_head_w = (self.embed_w if weights["lm_head"] is weights["embed"]
                              else weights["lm_head"].to(dev, torch.bfloat16).contiguous())
            self.norm_w = weights["norm"].to(dev, torch.bfloat16).contiguous()
        else:
            self.embed_w = (torch.randn(s.vocab, s.hidden, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
            self.lm_head_w = self.embed_w if s.tie_embeddings else \
                (torch.randn(s.vocab, s.hidden, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
            self.norm_w = (1.0 + 0.02 * torch.randn(s.hidden, device=dev, generator=gen)).to(torch.bfloat16)
        # RoPE tables cover absolute positions (the EAGLE head's small cache
        # holds rows of a tree whose positions continue the sequence)
        self.rope_len = max_seq if rope_len is None else rope_len
        self.cos, self.sin = precompute_rope(s.head_dim, self.rope_len, s.rope_theta, dev)
        self.k_cache = torch.zeros(s.n_layers, batch, s.n_kv_heads, max_seq, s.head_dim, dtype=torch.bfloat16,
                                   device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=dev)   # committed rows per sequence
        M = max_rows
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(M, s.hidden, **bf)          # residual stream
        self.xn = torch.zeros(M, s.hidden, **bf)         # normed input of a projection
        self.qkv = torch.zeros(M, s.qkv_dim, **bf)
        self.q = torch.zeros(M, s.q_dim, **bf)
        self.attn = torch.zeros(M, s.q_dim, **bf)
        self.h = torch.zeros(M, s.intermediate, **bf)
        self.starts = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(M, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        T_max = max(1, M // batch)
        self.attn_ws_bytes = max(
            _lib.query("tsds_attention_workspace_bytes", batch, t, s.n_heads, s.n_kv_heads, s.head_dim, max_seq,
                       split_keys) for t in range(1, T_max + 1))
        self.attn_ws = torch.empty(max(self.attn_ws_bytes, 16), dtype=torch.uint8, device=dev)
        lin = [(s.qkv_dim, s.hidden), (s.hidden, s.q_dim), (s.intermediate, s.hidden), (s.hidden, s.intermediate)]
        self.lin_ws_bytes = max(_lib.query("tsds_linear_workspace_bytes", m, o, k) for o, k in lin
                                for m in range(1, M + 1))
        # zero-filled once: the tcgen05 tile counters live in these and every
        # launch leaves them zero again
        self.lin_ws = torch.zeros(max(self.lin_ws_bytes, 16), dtype=torch.uint8, device=dev)
        self.lm_ws_bytes = max(_lib.query("tsds_lm_head_workspace_bytes", m, s.vocab) for m in range(1, M + 1))
        self.lm_ws = torch.zeros(max(self.lm_ws_bytes, 16), dtype=torch.uint8, device=dev)

    # -- launch plans ---------------------------------------------------------
    def layers_plan(self, B: int, T: int, tree_mask: torch.Tensor | None = None, mask_origin: int = -1,
                    x: torch.Tensor | None = None, starts: torch.Tensor | None = None,
                    positions: torch.Tensor | None = None) -> Plan:
        """All decoder layers over rows x[0:B*T] (embedded already), with
        starts/positions already prepared.  ``x`` / ``starts`` /
        ``positions`` default to the model's own buffers; ``tree_mask`` +
        ``mask_origin`` select the attention mask (see tsds_verify_attention)."""
        s = self.shape
        M = B * T
        assert M <= self.max_rows and B == self.batch
        eps = s.eps
        pl = Plan()
        lw, lb = self.lin_ws, self.lin_ws_bytes
        qn = self.qk_norm
        xb = self.x if x is None else x
        st = self.starts if starts is None else starts
        ps = self.positions if positions is None else positions
        for i, L in enumerate(self.layers):
            kc, vc = self.k_cache[i], self.v_cache[i]
            pl.add("tsds_rms_norm", _p(xb), _p(L.ln1), _p(self.xn), M, s.hidden, s.hidden, s.hidden, eps)
            pl.add("tsds_linear", _p(self.xn), s.hidden, _p(L.w_qkv), _p(self.qkv), s.qkv_dim, M, s.qkv_dim,
                   s.hidden, _p(lw), lb)
            pl.add("tsds_qk_norm_rope_kv", _p(self.qkv), _p(L.q_norm) if qn else None,
                   _p(L.k_norm) if qn else None, _p(self.cos), _p(self.sin), _p(ps), _p(st),
                   _p(self.q), _p(kc), _p(vc), B, T, s.n_heads, s.n_kv_heads, s.head_dim, self.max_seq, self.rope_len,
                   eps)
            pl.add("tsds_verify_attention", _p(self.q), _p(kc), _p(vc), _p(self.attn), _p(st),
                   _p(tree_mask), mask_origin, B, T, s.n_heads, s.n_kv_heads, s.head_dim, self.max_seq,
                   self.max_seq, self.split_keys, float(s.head_dim ** -0.5), _p(self.attn_ws), self.attn_ws_bytes,
                   _p(self.status))
            pl.add("tsds_linear_residual", _p(self.attn), s.q_dim, _p(L.w_o), _p(xb), _p(xb), s.hidden, M,
                   s.hidden, s.q_dim, _p(lw), lb)
            pl.add("tsds_rms_norm", _p(xb), _p(L.ln2), _p(self.xn), M, s.hidden, s.hidden, s.hidden, eps)
            pl.add("tsds_linear_swiglu", _p(self.xn), s.hidden, _p(L.w_gu), _p(self.h), s.intermediate, M,
                   s.intermediate, s.hidden, _p(lw), lb)
            pl.add("tsds_linear_residual", _p(self.h), s.intermediate, _p(L.w_d), _p(xb), _p(xb), s.hidden,
                   M, s.hidden, s.intermediate, _p(lw), lb)
        return pl

    def head_plan(self, B: int, T: int, argmax_out: torch.Tensor, argmax_stride: int, last_only: bool,
                  logits_out: torch.Tensor | None = None, x: torch.Tensor | None = None) -> Plan:
        """Final RMSNorm + LM head + argmax over all rows, or only the last
        row of each sequence."""
        s = self.shape
        pl = Plan()
        xb = self.x if x is None else x
        rows, ld = (B, T * s.hidden) if last_only else (B * T, s.hidden)
        src = xb[T - 1:] if last_only else xb
        pl.add("tsds_rms_norm", _p(src), _p(self.norm_w), _p(self.xn), rows, s.hidden, ld, s.hidden, s.eps)
        pl.add("tsds_lm_head_argmax", _p(self.xn), s.hidden, _p(self.lm_head_w), _p(logits_out), _p(argmax_out),
               argmax_stride, rows, s.vocab, s.hidden, _p(self.lm_ws), self.lm_ws_bytes)
        return pl

    def forward_plan(self, ids: torch.Tensor, ids_stride: int, B: int, T: int, base: torch.Tensor, offset: int,
                     argmax_out: torch.Tensor, argmax_stride: int = 1, last_only: bool = False,
                     logits_out: torch.Tensor | None = None) -> Plan:
        """Chain forward of T tokens per sequence at rows base[b]+offset+t:
        bookkeeping, embedding, layers, final norm, LM head + argmax."""
        s = self.shape
        pl = Plan()
        pl.add("tsds_prep_chain", _p(base), offset, B, T, _p(self.starts), _p(self.positions))
        pl.add("tsds_embed", _p(ids), ids_stride, _p(self.embed_w), _p(self.x), B * T, s.hidden, s.vocab)
        pl.extend(self.layers_plan(B, T))
        pl.extend(self.head_plan(B, T, argmax_out, argmax_stride, last_only, logits_out))
        return pl

    # -- prefill (untimed set-up: cuBLAS + SDPA) -------------------------------
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Process a [B, P] prompt from row 0; returns the hidden states
        [B, P, N] (pre final norm) and sets lengths = P."""
        s = self.shape
        B, P = prompt.shape
        dev = self.device
        prompt = prompt.to(dev)
        x = self.embed_w[prompt].reshape(B * P, s.hidden)
        pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(B)
        starts = torch.zeros(B, dtype=torch.int32, device=dev)
        from . import ops
        q = torch.empty(B * P, s.q_dim, dtype=torch.bfloat16, device=dev)
        for i, L in enumerate(self.layers):
            xn = ops.rms_norm(x, L.ln1, s.eps)
            qkv = xn @ L.w_qkv.T
            ops.qk_norm_rope_kv(qkv, L.q_norm if self.qk_norm else None, L.k_norm if self.qk_norm else None,
                                self.cos, self.sin, pos, starts, q, self.k_cache[i], self.v_cache[i], B, P,
                                s.n_heads, s.n_kv_heads, s.eps)
            qh = q.reshape(B, P, s.n_heads, s.head_dim).transpose(1, 2)
            kh = self.k_cache[i][:, :, :P].repeat_interleave(s.q_per_kv, dim=1)
            vh = self.v_cache[i][:, :, :P].repeat_interleave(s.q_per_kv, dim=1)
            a = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True)
            a = a.transpose(1, 2).reshape(B * P, s.q_dim)
            x = x + a @ L.w_o.T
            xn = ops.rms_norm(x, L.ln2, s.eps)
            gu = xn @ L.w_gu.T
            h = F.silu(gu[:, :s.intermediate]) * gu[:, s.intermediate:]
            x = x + h @ L.w_d.T
        self.lengths.fill_(P)
        return x.reshape(B, P, s.hidden)

    def logits_of(self, hidden: torch.Tensor) -> torch.Tensor:
        """Final norm + full bf16 logits (set-up / tests only)."""
        from . import ops
        xn = ops.rms_norm(hidden.reshape(-1, self.shape.hidden).contiguous(), self.norm_w, self.shape.eps)
        return xn @ self.lm_head_w.T

    def check_status(self):
        st = int(self.status.item())
        if st != 0:
            self.status.zero_()
            raise RuntimeError(f"device status {st}: {_lib.load().tsds_status_string(st).decode()}")

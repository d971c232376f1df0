"""``torch.ops.tsds``: the spec path's operators as PyTorch custom ops.

``import tri_sds_b200.torch_ops`` registers them.  Each is a thin layer over
the C ABI (through ``tri_sds_b200.ops``): the kernels the engines run, for
callers that compose them in PyTorch code.  Tensors must be CUDA tensors of
the documented types; anything else raises (there is no CPU
implementation).  Weights are in the ``[out, in]`` layout.

=================  =========================================================
op                 reference code it stands for
=================  =========================================================
qkv_rope_fused     RMSNorm -> q/k/v -> QK-norm + RoPE -> KV write
                   (qwen_model.py:104-119; fused_qwen_decode.py:212-250)
verify_attention   GQA attention over the cache, causal or tree mask
                   (qwen_model.py:121-131; attention.py:236-318)
oproj_fused        x + attn @ W_o (qwen_model.py:133-134)
mlp_fused          x + down(silu(gate) * up) of RMSNorm(x) (:136-144)
lm_head_topk       final RMSNorm + LM head, logits + top-k + log-sum-exp
                   (qwen_model.py:191-193; eagle_head.py:119-121)
eagle_fc           fc over [feature | embedding(token)] + bias
                   (eagle_head.py:79-80, 113)
accept_greedy      greedy chain acceptance + length commit
accept_rejection   tree acceptance: rejection sampling at temperature 1 with
                   given uniforms, or greedy
kv_compact         KV rows of the accepted path -> consecutive rows, lengths
                   += accepted + 1, next root feature
allreduce_oneshot  x += sum over the TP ranks of their fp32 partials (the
                   all-reduce after O / down; no reference counterpart)
=================  =========================================================

``allreduce_oneshot`` is tensor parallelism's row-parallel all-reduce + residual
add over NVLink peer memory (a ``tp.PeerAllReduce`` group, registered with
``tp.register_peer_group``).  ``accept_rejection`` and
``kv_compact`` check their index arguments on the host before the launch
(a device-to-host copy, so they do not belong in a captured CUDA graph); the
engines call the C ABI directly with indices their own kernels produced.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _lib, ops


def _p(t):
    return ops._p(t)


def _s():
    return ops._stream()


def _in_range(t: Tensor, lo: int, hi: int, what: str) -> None:
    """Index tensors that a kernel follows without a bounds check are checked
    here, on the host (one device-to-host copy): lo <= t < hi."""
    if t.numel():
        ops._need(lo <= int(t.min()) and int(t.max()) < hi, f"{what} out of range [{lo}, {hi})")


@torch.library.custom_op("tsds::qkv_rope_fused", mutates_args=("k_cache", "v_cache"))
def qkv_rope_fused(x: Tensor, norm_w: Tensor, qkv_w: Tensor, q_norm_w: Optional[Tensor], k_norm_w: Optional[Tensor],
                   cos: Tensor, sin: Tensor, positions: Tensor, starts: Tensor, k_cache: Tensor, v_cache: Tensor,
                   n_heads: int, n_kv_heads: int, eps: float = 1e-6) -> Tensor:
    """x [B*T, N] bf16 -> q [B*T, n_heads*D]; k/v of token t of sequence b
    written to cache row starts[b] + t (caches [B, Hkv, S, D]); positions
    [B*T] and starts [B] int32."""
    B = starts.shape[0]
    ops._need(B > 0 and x.shape[0] % B == 0, "rows of x must be B * T")
    T = x.shape[0] // B
    D = k_cache.shape[-1]
    xn = ops.rms_norm(x, norm_w, eps)
    qkv = ops.linear(xn, qkv_w)
    q = torch.empty(x.shape[0], n_heads * D, dtype=x.dtype, device=x.device)
    ops.qk_norm_rope_kv(qkv, q_norm_w, k_norm_w, cos, sin, positions, starts, q, k_cache, v_cache, B, T, n_heads,
                        n_kv_heads, eps)
    return q


@torch.library.custom_op("tsds::verify_attention", mutates_args=())
def verify_attention(q: Tensor, k_cache: Tensor, v_cache: Tensor, starts: Tensor, tree_mask: Optional[Tensor] = None,
                     split_keys: int = 128) -> Tensor:
    """q [B, T, Hq, D] over caches [B, Hkv, S, D] whose rows starts[b].. hold
    the T new tokens; tree_mask [B, T] int32 bitmasks over the new tokens."""
    return ops.verify_attention(q, k_cache, v_cache, starts, tree_mask, split_keys=split_keys)


@torch.library.custom_op("tsds::oproj_fused", mutates_args=())
def oproj_fused(attn: Tensor, o_w: Tensor, x: Tensor) -> Tensor:
    """x + attn @ o_w^T with the reference's rounding (bf16 product, bf16 sum)."""
    return ops.linear_residual(attn, o_w, x)


@torch.library.custom_op("tsds::mlp_fused", mutates_args=())
def mlp_fused(x: Tensor, norm_w: Tensor, gate_up_w: Tensor, down_w: Tensor, eps: float = 1e-6) -> Tensor:
    """x + down(silu(gate) * up) of RMSNorm(x); gate_up_w = [gate; up]."""
    h = ops.linear_swiglu(ops.rms_norm(x, norm_w, eps), gate_up_w)
    return ops.linear_residual(h, down_w, x)


@torch.library.custom_op("tsds::lm_head_topk", mutates_args=())
def lm_head_topk(x: Tensor, norm_w: Tensor, lm_head_w: Tensor, k: int,
                 eps: float = 1e-6) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """-> (logits [M, V] bf16, top-k values [M, k] fp32 (desc, lowest index
    first on ties), their indices [M, k] int32, log-sum-exp [M] fp32);
    k in {1, 2, 4, 8}."""
    ops._need(k in (1, 2, 4, 8), "k must be 1, 2, 4 or 8")
    _, logits = ops.lm_head_argmax(ops.rms_norm(x, norm_w, eps), lm_head_w, return_logits=True)
    M, V = logits.shape
    vals = torch.empty(M, k, dtype=torch.float32, device=x.device)
    idx = torch.empty(M, k, dtype=torch.int32, device=x.device)
    lse = torch.empty(M, dtype=torch.float32, device=x.device)
    _lib.call("tsds_logits_topk", _p(logits), V, M, V, k, _p(vals), _p(idx), _p(lse), _s())
    return logits, vals, idx, lse


@torch.library.custom_op("tsds::eagle_fc", mutates_args=())
def eagle_fc(features: Tensor, token_ids: Tensor, embed_w: Tensor, fc_w: Tensor, fc_b: Tensor) -> Tensor:
    """[features | embed_w[token_ids]] @ fc_w^T + fc_b: features [M, N] bf16,
    token_ids [M] int64, fc_w [N, 2N]."""
    ops._bf16_cuda(features, embed_w, fc_w, fc_b)
    ops._cuda(torch.int64, token_ids)
    M, N = features.shape
    ops._need(fc_w.shape == (N, 2 * N) and fc_b.shape == (N,) and token_ids.shape == (M,) and N % 8 == 0 and
              embed_w.shape[1] == N and features.is_contiguous() and fc_w.is_contiguous(), "bad shapes")
    x2 = torch.empty(M, 2 * N, dtype=features.dtype, device=features.device)
    root_rows = torch.full((M,), -1, dtype=torch.int32, device=features.device)   # feature row m of `features`
    _lib.call("tsds_eagle_inputs", _p(features), None, _p(root_rows), _p(token_ids), _p(embed_w), _p(x2), M, 1, N,
              embed_w.shape[0], _s())
    out = torch.empty(M, N, dtype=features.dtype, device=features.device)
    ws, nb = ops._lin_ws(M, N, 2 * N, features.device)
    _lib.call("tsds_linear_bias", _p(x2), 2 * N, _p(fc_w), _p(fc_b), _p(out), N, M, N, 2 * N, _p(ws), nb, _s())
    return out


@torch.library.custom_op("tsds::accept_greedy", mutates_args=("lengths", "last", "cur"))
def accept_greedy(draft: Tensor, target_argmax: Tensor, lengths: Tensor, last: Tensor,
                  cur: Tensor) -> tuple[Tensor, Tensor]:
    """Longest prefix of draft [B, K] equal to the target's argmax [B, K+1];
    lengths += accepted + 1; last / cur for the next cycle.
    -> (accept_len [B] int32, tokens [B, K+1] int64, -1 padded)."""
    return ops.accept_greedy(draft, target_argmax, lengths, last, cur)


@torch.library.custom_op("tsds::accept_rejection", mutates_args=())
def accept_rejection(target_logits: Tensor, head_logits: Tensor, ids: Tensor, hrow: Tensor, children: Tensor,
                     uniforms: Optional[Tensor], target_argmax: Optional[Tensor],
                     depth: int, rule: int = 0) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Walk a verified tree of NN nodes per sequence: ids [B, NN] int64,
    children [B, NN, k] int32 (-1 padded), hrow [B, NN] int32 (head-logits
    row of each node's children), target_logits [B*NN, V] and head_logits
    [rows, V] bf16.  uniforms [B, depth+1, k+1] fp32 -> rejection sampling at
    temperature 1; None -> greedy on target_argmax [B*NN] int64.  rule 0:
    accept x if u q(x) < p(x), residual max(p - q, 0) (children drawn from
    q); rule 1: accept x if u < p(x), drop x from p (deterministic children,
    e.g. top-k; head_logits unread).
    -> (path [B, depth+1] int32 node indices, accept_len [B] int32,
    tokens [B, depth+2] int64 (accepted then the bonus, -1 padded), bonus [B])."""
    ops._bf16_cuda(target_logits, head_logits)
    ops._cuda(torch.int64, ids, target_argmax)
    ops._cuda(torch.int32, hrow, children)
    ops._cuda(torch.float32, uniforms)
    B, NN = ids.shape
    k = children.shape[-1]
    V = target_logits.shape[-1]
    ops._need(NN <= 32 and target_logits.shape[0] == B * NN, "bad shapes")
    ops._need(uniforms is not None or target_argmax is not None, "uniforms or target_argmax needed")
    ops._need(children.shape == (B, NN, k) and hrow.shape == (B, NN) and depth >= 1, "bad shapes")
    ops._need(uniforms is None or uniforms.shape == (B, depth + 1, k + 1), "uniforms must be [B, depth+1, k+1]")
    ops._need(target_argmax is None or target_argmax.numel() == B * NN, "target_argmax must be [B*NN]")
    ops._need(rule in (0, 1), "rule must be 0 (draft) or 1 (target-only)")
    _in_range(children, -1, NN, "children")
    if uniforms is not None and rule == 0:   # the head-logits row of every node that has children
        _in_range(hrow[children[..., 0] >= 0], 0, head_logits.shape[0], "hrow")
    dev = ids.device
    path = torch.empty(B, depth + 1, dtype=torch.int32, device=dev)
    acc = torch.empty(B, dtype=torch.int32, device=dev)
    tokens = torch.empty(B, depth + 2, dtype=torch.int64, device=dev)
    bonus = torch.empty(B, dtype=torch.int64, device=dev)
    _lib.call("tsds_accept_tree_rule", _p(target_logits), _p(target_argmax), _p(head_logits), _p(ids), _p(hrow),
              _p(children), _p(uniforms), int(rule), _p(path), _p(acc), _p(tokens), _p(bonus), B, NN - 1, V, k,
              depth, _s())
    return path, acc, tokens, bonus


@torch.library.custom_op("tsds::kv_compact", mutates_args=("k_cache", "v_cache", "lengths", "root_feat"))
def kv_compact(k_cache: Tensor, v_cache: Tensor, lengths: Tensor, path: Tensor, accept_len: Tensor, hidden: Tensor,
               root_feat: Tensor, depth: int) -> None:
    """For sequence b at committed length L: K/V rows L + path[b, j] ->
    L + 1 + j for j < accept_len[b], in every layer (caches
    [layers, B, Hkv, S, D]); the hidden state [B*NN, N] of the last accepted
    node -> root_feat [B, N]; lengths += accept_len + 1."""
    ops._bf16_cuda(k_cache, v_cache, hidden, root_feat)
    ops._cuda(torch.int32, lengths, path, accept_len)
    L, B, Hkv, S, D = k_cache.shape
    ops._need(v_cache.shape == k_cache.shape and k_cache.is_contiguous() and v_cache.is_contiguous() and
              hidden.is_contiguous(), "contiguous caches of one shape expected")
    ops._need(hidden.shape[0] % B == 0 and path.shape == (B, depth + 1), "bad shapes")
    NN, N = hidden.shape[0] // B, hidden.shape[1]
    ops._need(lengths.shape == (B,) and accept_len.shape == (B,) and root_feat.shape == (B, N) and N % 8 == 0,
              "bad shapes")
    _in_range(accept_len, 0, depth + 1, "accept_len")
    used = torch.arange(depth + 1, device=path.device) < accept_len.to(path.device)[:, None]
    _in_range(path[used], 0, NN, "path")   # entries past accept_len are -1
    _in_range(lengths, 0, S, "lengths")
    _lib.call("tsds_tree_commit", _p(k_cache), _p(v_cache), L, B, Hkv, S, D, _p(lengths), _p(path), _p(accept_len),
              depth, _p(hidden), NN - 1, N, _p(root_feat), _s())


@torch.library.custom_op("tsds::allreduce_oneshot", mutates_args=("x",))
def allreduce_oneshot(x: Tensor, partial: Tensor, group: int) -> None:
    """Tensor parallelism: x [M, N] bf16 = bf16(x + bf16(sum over the ranks of
    their fp32 partial [M, N])), the same on every rank, over NVLink peer
    memory (tsds_peer_allreduce_residual).  `group` is the id from
    tp.register_peer_group of a tp.PeerAllReduce; every rank makes the same
    sequence of calls with the same shapes."""
    from . import tp
    ops._bf16_cuda(x)
    ops._cuda(torch.float32, partial)
    peer = tp.peer_group(group)
    M, N = x.shape
    ops._need(partial.shape == (M, N) and x.is_contiguous() and M * N <= peer.max_elems and N % 4 == 0,
              "bad shapes")
    slot = peer.next_slot()
    peer.slot_tensor(slot, M * N).copy_(partial.reshape(-1))
    _lib.call("tsds_peer_allreduce_residual", _p(x), peer.bufs, peer.rank, peer.size, slot, M, N, peer.max_elems,
              _p(ops._scratch.status_word(x.device)), _s())


OPS = ("qkv_rope_fused", "verify_attention", "oproj_fused", "mlp_fused", "lm_head_topk", "eagle_fc", "accept_greedy",
       "accept_rejection", "kv_compact", "allreduce_oneshot")

"""Torch-facing ops over the C ABI, named after the reference's kernel wrappers.

Reference op (file:line)                                 -> here
  norm.rms_norm (norm.py:61-72)                             rms_norm
  attention.attention_gqa (attention.py:299-318)            attention_gqa
  qwen_model verify SDPA (qwen_model.py:121-131)            verify_attention
  fused_qwen_decode.fused_rmsnorm_qkv_rope (:124-149)       fused_rmsnorm_qkv_rope
  fused_qwen_decode.fused_oproj_residual (:179-204)         fused_oproj_residual
  fused_qwen_decode.fused_gateup_silu (:242-265)            fused_gateup_silu
  fused_qwen_decode.fused_down_residual (:293-309)          fused_down_residual
  LM head + argmax (qwen_model.py:192; eagle_head.py:120)   lm_head_argmax

Like the reference wrappers these allocate their outputs with torch and
launch on torch's current stream; errors raise (the reference asserts).
The ops share one scratch workspace per device and op kind.  Calls that
could overlap on the GPU (ops on different streams) must therefore not
run at the same time.  The engines give every model workspaces of its own.
Every op runs the sm_100a kernels of libtsds.so; there is no other path.
Weights may be given in the reference's transposed ``[in, out]`` layout
(``*_w_t`` arguments) or as the transposed view of an HF ``[out, in]``
weight; the kernels read ``[out, in]``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_VP = ctypes.c_void_p


def _p(t):
    return None if t is None else _VP(t.data_ptr())


def _stream():
    return _VP(torch.cuda.current_stream().cuda_stream)


def _need(cond, msg):
    if not cond:
        raise ValueError(msg)


def _bf16_cuda(*ts):
    for t in ts:
        if t is not None:
            _need(t.is_cuda and t.dtype == torch.bfloat16, "expected a bf16 CUDA tensor")


def _cuda(dtype, *ts):
    """Index / length tensors: on a CUDA device, of the kernel's integer type
    (a host pointer handed to a kernel would fault the device)."""
    for t in ts:
        if t is not None:
            _need(t.is_cuda and t.dtype == dtype, f"expected a {dtype} CUDA tensor")


class _Scratch:
    """Grow-only, zero-initialised workspaces (one per device and op kind:
    the tcgen05 tile counters of one op must not be overwritten by another's
    scratch data) and a status word, for the op-level API."""

    def __init__(self):
        self.buf = {}
        self.status = {}

    def get(self, nbytes: int, device, kind: str = "linear") -> torch.Tensor:
        key = (torch.device(device).index, kind)
        b = self.buf.get(key)
        if b is None or b.numel() < nbytes:
            b = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self.buf[key] = b
        return b

    def status_word(self, device) -> torch.Tensor:
        key = torch.device(device).index
        s = self.status.get(key)
        if s is None:
            s = torch.zeros(1, dtype=torch.int32, device=device)
            self.status[key] = s
        return s


_scratch = _Scratch()


def check_status(device=None) -> None:
    """Raise RuntimeError if an op-level kernel on `device` (default: the
    current one) recorded an error in its status word - a bounded device
    wait that gave up.  Synchronises the device.  The op-level workspaces'
    headers (status word + tile counters) and the status word are zeroed
    first, so later calls start afresh."""
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    torch.cuda.synchronize(dev)
    # the tcgen05 GEMM and LM-head workspaces carry a status word and tile
    # counters; the attention workspace holds split partials only
    hb = _lib.query("tsds_linear_workspace_header_bytes")
    hdr = {"linear": hb, "lm_head": hb}
    bad = 0
    for (d, kind), b in _scratch.buf.items():
        if d != dev or kind not in hdr:
            continue
        st = int(b[:4].view(torch.int32).item())
        if st:
            b[:min(hdr.get(kind, 4), b.numel())].zero_()
            bad = bad or st
    s = _scratch.status.get(dev)
    if s is not None and int(s.item()):
        bad = bad or int(s.item())
        s.zero_()
    if bad:
        raise RuntimeError(f"device status {bad}: {_lib.load().tsds_status_string(bad).decode()}")


def _out_in(w_t: torch.Tensor) -> torch.Tensor:
    """[in, out] weight argument -> contiguous [out, in] tensor."""
    if w_t.dim() == 2 and w_t.stride(0) == 1 and w_t.stride(1) == w_t.shape[0]:
        return w_t.t()  # a transposed view of a contiguous [out, in] weight
    return w_t.t().contiguous()


# ---------------------------------------------------------------------------

def set_gemv_max_rows(rows: int) -> None:
    """Largest row count served by the CUDA-core GEMV; above it the tcgen05
    GEMM runs (process-wide; 0 sends every linear layer to tcgen05)."""
    _lib.load().tsds_set_gemv_max_rows(int(rows))


def set_attention_tc(mode: int | bool) -> None:
    """Run verify attention on its tcgen05 variant (process-wide) for calls
    whose split_keys is a multiple of 128: 1 / True; 2: also combine 2 to 8
    key splits inside a thread-block cluster; 0 / False: the default kernel."""
    _lib.load().tsds_set_attention_tc(int(mode))


def attention_tc() -> int:
    return int(_lib.load().tsds_get_attention_tc())


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None):
    """norm.py:61-72 over the rows of a 2-D tensor."""
    _bf16_cuda(x, weight, out)
    _need(x.dim() == 2 and x.stride(1) == 1, "x must be [rows, n] with unit inner stride")
    rows, n = x.shape
    out = torch.empty_like(x) if out is None else out
    _lib.call("tsds_rms_norm", _p(x), _p(weight), _p(out), rows, n, x.stride(0), out.stride(0), float(eps),
              _stream())
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None):
    """table[ids] for a flat int64 id tensor."""
    _bf16_cuda(table, out)
    _cuda(torch.int64, ids)
    ids = ids.reshape(-1)
    _need(ids.dtype == torch.int64 and ids.is_cuda, "ids must be int64 CUDA")
    M = ids.numel()
    out = torch.empty(M, table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    _lib.call("tsds_embed", _p(ids), ids.stride(0), _p(table), _p(out), M, table.shape[1], table.shape[0], _stream())
    return out


def _lin_ws(M, n_out, K, device):
    nb = _lib.query("tsds_linear_workspace_bytes", M, n_out, K)
    return (_scratch.get(nb, device), nb) if nb else (None, 0)


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None):
    """x [M, K] @ w[n_out, K]^T -> bf16 [M, n_out]."""
    _bf16_cuda(x, w, out)
    M, K = x.shape
    n_out = w.shape[0]
    _need(w.shape[1] == K and w.is_contiguous(), "w must be contiguous [n_out, K]")
    out = torch.empty(M, n_out, dtype=x.dtype, device=x.device) if out is None else out
    ws, nb = _lin_ws(M, n_out, K, x.device)
    _lib.call("tsds_linear", _p(x), x.stride(0), _p(w), _p(out), out.stride(0), M, n_out, K, _p(ws), nb, _stream())
    return out


def linear_residual(x: torch.Tensor, w: torch.Tensor, res: torch.Tensor, out: torch.Tensor | None = None):
    """res + x @ w^T with the reference's rounding (bf16 product, bf16 sum)."""
    _bf16_cuda(x, w, res, out)
    M, K = x.shape
    n_out = w.shape[0]
    _need(w.shape[1] == K and w.is_contiguous() and res.shape == (M, n_out), "shape mismatch")
    out = torch.empty_like(res) if out is None else out
    _need(res.stride(0) == out.stride(0), "res and out must share a row stride")
    ws, nb = _lin_ws(M, n_out, K, x.device)
    _lib.call("tsds_linear_residual", _p(x), x.stride(0), _p(w), _p(res), _p(out), out.stride(0), M, n_out, K,
              _p(ws), nb, _stream())
    return out


def linear_residual_norm(x: torch.Tensor, w: torch.Tensor, res: torch.Tensor, norm_w: torch.Tensor,
                         eps: float = 1e-6, out: torch.Tensor | None = None, norm_out: torch.Tensor | None = None):
    """(res + x @ w^T, RMSNorm of that with norm_w): a decoder layer's residual
    add and the RMSNorm that reads it, in one launch; both bit for bit what
    linear_residual + rms_norm give."""
    _bf16_cuda(x, w, res, norm_w, out, norm_out)
    M, K = x.shape
    n_out = w.shape[0]
    _need(w.shape[1] == K and w.is_contiguous() and res.shape == (M, n_out), "shape mismatch")
    _need(norm_w.shape == (n_out,) and norm_w.is_contiguous(), "norm_w must be [n_out]")
    out = torch.empty_like(res) if out is None else out
    norm_out = torch.empty_like(res) if norm_out is None else norm_out
    _need(res.stride(0) == out.stride(0), "res and out must share a row stride")
    ws, nb = _lin_ws(M, n_out, K, x.device)
    _lib.call("tsds_linear_residual_norm", _p(x), x.stride(0), _p(w), _p(res), _p(out), out.stride(0), M, n_out, K,
              _p(norm_w), _p(norm_out), norm_out.stride(0), float(eps), _p(ws), nb, _stream())
    return out, norm_out


def linear_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor | None = None):
    """silu(x @ gate^T) * (x @ up^T) for w_gate_up = [gate; up] ([2I, K])."""
    _bf16_cuda(x, w_gate_up, out)
    M, K = x.shape
    _need(w_gate_up.shape[0] % 2 == 0 and w_gate_up.shape[1] == K and w_gate_up.is_contiguous(), "bad gate/up")
    I = w_gate_up.shape[0] // 2
    out = torch.empty(M, I, dtype=x.dtype, device=x.device) if out is None else out
    ws, nb = _lin_ws(M, I, K, x.device)
    _lib.call("tsds_linear_swiglu", _p(x), x.stride(0), _p(w_gate_up), _p(out), out.stride(0), M, I, K, _p(ws), nb,
              _stream())
    return out


def linear_f32(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None):
    """x @ w^T as an unrounded fp32 [M, n_out] partial: a row-parallel
    shard's product before the all-reduce over the tensor-parallel ranks."""
    _bf16_cuda(x, w)
    _cuda(torch.float32, out)
    M, K = x.shape
    n_out = w.shape[0]
    _need(w.shape[1] == K and w.is_contiguous(), "w must be contiguous [n_out, K]")
    out = torch.empty(M, n_out, dtype=torch.float32, device=x.device) if out is None else out
    ws, nb = _lin_ws(M, n_out, K, x.device)
    _lib.call("tsds_linear_f32", _p(x), x.stride(0), _p(w), _p(out), out.stride(0), M, n_out, K, _p(ws), nb,
              _stream())
    return out


def residual_add_f32(x: torch.Tensor, partial: torch.Tensor):
    """x = bf16(x + bf16(partial)) in place (qwen_model.py:133-134,143-144
    rounding) for the all-reduced fp32 partial of a row-parallel projection."""
    _bf16_cuda(x)
    _cuda(torch.float32, partial)
    _need(x.is_contiguous() and partial.is_contiguous() and partial.shape == x.shape, "x / partial mismatch")
    _lib.call("tsds_residual_add_f32", _p(x), _p(partial), x.shape[0], x.shape[1], _stream())
    return x


def fused_oproj_residual(attn_flat, o_w_t, x):
    """fused_qwen_decode.py:179-204: x + attn_flat @ o_w_t."""
    return linear_residual(attn_flat, _out_in(o_w_t), x)


def fused_gateup_silu(x_norm2, gate_up_w_t):
    """fused_qwen_decode.py:242-265: silu(x@W[:, :I]) * (x@W[:, I:])."""
    return linear_swiglu(x_norm2, _out_in(gate_up_w_t))


def fused_down_residual(hidden, down_w_t, x_residual):
    """fused_qwen_decode.py:293-309: x_residual + hidden @ down_w_t."""
    return linear_residual(hidden, _out_in(down_w_t), x_residual)


def qk_norm_rope_kv(qkv, q_norm_w, k_norm_w, cos, sin, positions, starts, q_out, k_cache, v_cache,
                    B, T, Hq, Hkv, eps=1e-6):
    """QK-norm + RoPE of the q/k heads of ``qkv`` [B*T, (Hq+2Hkv)*D]; q -> q_out,
    k/v -> the cache rows ``starts[b]+t``."""
    _bf16_cuda(qkv, q_norm_w, k_norm_w, cos, sin, q_out, k_cache, v_cache)
    _cuda(torch.int32, positions, starts)
    D = k_cache.shape[-1]
    S = k_cache.shape[-2]
    _lib.call("tsds_qk_norm_rope_kv", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin), _p(positions),
              _p(starts), _p(q_out), _p(k_cache), _p(v_cache), B, T, Hq, Hkv, D, S, cos.shape[0], float(eps),
              _stream())


def fused_rmsnorm_qkv_rope(x, norm1_w, qkv_w_t, q_out, k_cache, v_cache, cos, sin, pos, N, q_dim, kv_dim,
                           H_q, H_kv, D, q_norm_w=None, k_norm_w=None, eps=1e-6):
    """fused_qwen_decode.py:253-274: RMSNorm -> QKV -> RoPE -> KV write at
    scalar position ``pos`` for B single-token rows; q_out is [B, H_q, 1, D].
    ``q_norm_w`` / ``k_norm_w`` add Qwen3's QK-norm (absent in the reference)."""
    B = x.shape[0]
    xn = rms_norm(x, norm1_w, eps)
    qkv = linear(xn, _out_in(qkv_w_t))
    dev = x.device
    positions = torch.full((B,), int(pos), dtype=torch.int32, device=dev)
    qk_norm_rope_kv(qkv, q_norm_w, k_norm_w, cos, sin, positions, positions, q_out, k_cache, v_cache,
                    B, 1, H_q, H_kv, eps)


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, starts: torch.Tensor,
                     tree_mask: torch.Tensor | None = None, max_kv: int | None = None, split_keys: int = 128,
                     scale: float | None = None, out: torch.Tensor | None = None, mask_origin: int = -1):
    """Attention of q [B, T, Hq, D] over caches [B, Hkv, S, D] whose rows
    ``starts[b]..starts[b]+T-1`` hold the new tokens (qwen_model.py:121-131
    with per-sequence starts and an optional [B, T] tree bitmask)."""
    _bf16_cuda(q, k_cache, v_cache, out)
    B, T, Hq, D = q.shape
    Hkv, S = k_cache.shape[1], k_cache.shape[2]
    _need(q.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous(), "contiguous tensors expected")
    starts = starts.to(device=q.device, dtype=torch.int32).contiguous()
    if tree_mask is not None:
        tree_mask = tree_mask.to(device=q.device, dtype=torch.int32).contiguous()
    max_kv = S if max_kv is None else int(max_kv)
    scale = D ** -0.5 if scale is None else float(scale)
    out = torch.empty_like(q) if out is None else out
    nb = _lib.query("tsds_attention_workspace_bytes", B, T, Hq, Hkv, D, max_kv, split_keys)
    ws = _scratch.get(nb, q.device, "attention") if nb else None
    status = _scratch.status_word(q.device)
    _lib.call("tsds_verify_attention", _p(q), _p(k_cache), _p(v_cache), _p(out), _p(starts), _p(tree_mask),
              int(mask_origin), B, T, Hq, Hkv, D, S, max_kv, split_keys, scale, _p(ws), nb, _p(status), _stream())
    return out


def verify_attention_paged(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, starts: torch.Tensor,
                           token_table: torch.Tensor, req_rows: torch.Tensor | None = None, page_size: int = 1,
                           tree_mask: torch.Tensor | None = None, max_kv: int | None = None, split_keys: int = 1024,
                           scale: float | None = None, out: torch.Tensor | None = None, mask_origin: int = -1):
    """verify_attention over SGLang-style token pools: k_pool / v_pool
    [pool_rows, Hkv, D], position p of sequence b at pool row
    token_table[req_rows[b] (or b), p] (int32 [reqs, table_ld])."""
    _bf16_cuda(q, k_pool, v_pool, out)
    _cuda(torch.int32, token_table)
    _cuda(torch.int64, req_rows)
    B, T, Hq, D = q.shape
    pool_rows, Hkv = k_pool.shape[0], k_pool.shape[1]
    _need(q.is_contiguous() and k_pool.is_contiguous() and v_pool.is_contiguous() and token_table.is_contiguous(),
          "contiguous tensors expected")
    _need(v_pool.shape == k_pool.shape and k_pool.shape[2] == D, "pool shape mismatch")
    table_ld = token_table.shape[1]
    starts = starts.to(device=q.device, dtype=torch.int32).contiguous()
    if tree_mask is not None:
        tree_mask = tree_mask.to(device=q.device, dtype=torch.int32).contiguous()
    max_kv = table_ld if max_kv is None else int(max_kv)
    scale = D ** -0.5 if scale is None else float(scale)
    out = torch.empty_like(q) if out is None else out
    nb = _lib.query("tsds_attention_workspace_bytes", B, T, Hq, Hkv, D, max_kv, split_keys)
    ws = _scratch.get(nb, q.device, "attention") if nb else None
    status = _scratch.status_word(q.device)
    _lib.call("tsds_verify_attention_paged", _p(q), _p(k_pool), _p(v_pool), _p(out), _p(starts), _p(tree_mask),
              int(mask_origin), _p(token_table), table_ld, _p(req_rows), pool_rows, int(page_size), B, T, Hq, Hkv, D,
              max_kv, split_keys, scale, _p(ws), nb, _p(status), _stream())
    return out


def qk_norm_rope_kv_paged(qkv, q_norm_w, k_norm_w, cos, sin, positions, out_loc, q_out, k_pool, v_pool, Hq, Hkv,
                          eps=1e-6):
    """QK-norm + RoPE of the q/k heads of ``qkv`` [M, (Hq+2Hkv)*D]; q -> q_out,
    row m's k/v -> pool row out_loc[m] (SGLang's out_cache_loc)."""
    _bf16_cuda(qkv, q_norm_w, k_norm_w, cos, sin, q_out, k_pool, v_pool)
    _cuda(torch.int32, positions)
    _cuda(torch.int64, out_loc)
    M = qkv.shape[0]
    D = k_pool.shape[-1]
    status = _scratch.status_word(qkv.device)
    _lib.call("tsds_qk_norm_rope_kv_paged", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin), _p(positions),
              _p(out_loc), _p(q_out), _p(k_pool), _p(v_pool), M, Hq, Hkv, D, k_pool.shape[0], cos.shape[0],
              float(eps), _p(status), _stream())


def attention_gqa(q, k, v, kv_len, q_per_kv):
    """attention.py:299-318: q [B, Hq, 1, D] over the first ``kv_len`` cache
    rows (one length for the whole batch, a device int32 tensor)."""
    B, Hq, Tq, D = q.shape
    _need(Tq == 1, "GQA decode only")
    _need(Hq == k.shape[1] * q_per_kv, "q_per_kv mismatch")
    starts = (kv_len.reshape(1).to(torch.int32) - 1).expand(B).contiguous()
    o = verify_attention(q.reshape(B, 1, Hq, D).contiguous(), k, v, starts)
    return o.reshape(B, Hq, 1, D)


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, return_logits: bool = False, out: torch.Tensor | None = None):
    """argmax_v (x @ w^T) on bf16-rounded logits, lowest index on ties;
    optionally also the bf16 logits [M, V]."""
    _bf16_cuda(x, w)
    _cuda(torch.int64, out)
    M, K = x.shape
    V = w.shape[0]
    out = torch.empty(M, dtype=torch.int64, device=x.device) if out is None else out
    logits = torch.empty(M, V, dtype=torch.bfloat16, device=x.device) if return_logits else None
    nb = _lib.query("tsds_lm_head_workspace_bytes", M, V)
    ws = _scratch.get(nb, x.device, "lm_head")
    _lib.call("tsds_lm_head_argmax", _p(x), x.stride(0), _p(w), _p(logits), _p(out), out.stride(0), None, M, V, K,
              _p(ws), nb, _stream())
    return (out, logits) if return_logits else out


def accept_greedy(draft: torch.Tensor, target: torch.Tensor, target_len: torch.Tensor, last: torch.Tensor,
                  cur: torch.Tensor):
    """Greedy acceptance + commit (in place on target_len/last/cur);
    returns (accept_len [B] int32, tokens [B, K+1] int64 padded with -1)."""
    _cuda(torch.int64, draft, target, last, cur)
    _cuda(torch.int32, target_len)
    B, K = draft.shape
    acc = torch.empty(B, dtype=torch.int32, device=draft.device)
    tokens = torch.empty(B, K + 1, dtype=torch.int64, device=draft.device)
    _lib.call("tsds_accept_greedy", _p(draft), _p(target), _p(acc), _p(tokens), _p(target_len), _p(last), _p(cur),
              B, K, _stream())
    return acc, tokens

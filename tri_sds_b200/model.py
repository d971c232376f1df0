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

The prompt prefill (untimed set-up) runs through cuBLAS GEMMs and SDPA
(or the library's tcgen05 attention when that is switched on), with the
cache written by the same QK-norm/RoPE/KV kernel as the verify path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from dataclasses import replace

from . import _lib
from .paged import PagedKV  # noqa: F401  (QwenModel's kv argument)
from .shapes import QwenShape
from .tp import LocalComm, lm_exchange_layout, local_dims, shard_layer, vocab_shard

_VP = ctypes.c_void_p


def _p(t):
    return None if t is None else _VP(t.data_ptr())


# Remote bytes per rank above which the fused kernel's peer all-reduce runs
# two-shot (each rank reduces 1/tp of the elements and publishes them) rather
# than one-shot (every rank reads every partial): 2 MB, between B=1 at TP=4
# (1.6 MB one-shot) and TP=8 (3.7 MB) for the 32B hidden size.
TWO_SHOT_BYTES = 2 << 20


def raise_status(word, st: int, header=None, on_error=None):
    """Raise RuntimeError for a nonzero device status `st` read from `word`.
    The word - and `header`, the workspace bytes that hold it and the tile
    counters a launch that gave up may have left nonzero - is cleared so the
    next launch on the workspace starts afresh; `on_error()` runs first
    (e.g. to retire a peer group whose cross-rank epochs have drifted)."""
    if st != 0:
        if on_error is not None:
            on_error()
        (header if header is not None else word).zero_()
        raise RuntimeError(f"device status {st}: {_lib.load().tsds_status_string(st).decode()}")


class StatusWatch:
    """Reads a set of device status words together with a cycle's results:
    `copy()` queues their copies into pinned host memory on the current
    stream (after the cycle's kernels), `check()` - after the caller's
    synchronize - raises on the first nonzero one.  `regions` holds
    (word, header, on_error) triples as QwenModel.status_regions returns
    them, or bare status words."""

    def __init__(self, regions: list):
        self.regions = [r if isinstance(r, tuple) else (r, None, None) for r in regions]
        self.words = [r[0] for r in self.regions]
        self.host = torch.zeros(len(self.words), dtype=torch.int32,
                                pin_memory=bool(self.words) and self.words[0].is_cuda)

    def copy(self):
        for i, w in enumerate(self.words):
            self.host[i:i + 1].copy_(w, non_blocking=True)

    def check(self):
        for i, (w, header, on_error) in enumerate(self.regions):
            raise_status(w, int(self.host[i]), header, on_error)


def _fused_args(phases: list, rope: dict | None, peer, M: int, ws, ws_bytes: int) -> tuple:
    """tsds_fused_layer arguments (after the name) from phase dicts of
    pointers and sizes: a tsds_fused_phase array, a tsds_qk_rope and a
    tsds_peer_group (tp.PeerAllReduce), kept alive by the argument tuple."""
    arr = (_lib.FusedPhase * len(phases))(*[_lib.FusedPhase(**ph) for ph in phases])
    qr = ctypes.pointer(_lib.QkRope(**rope)) if rope is not None else None
    pg = None
    if peer is not None:
        pg = ctypes.pointer(_lib.PeerGroup(bufs=ctypes.cast(peer.bufs, ctypes.c_void_p), rank=peer.rank,
                                           tp=peer.size, max_elems=peer.max_elems))
        pg._bufs = peer.bufs
    return (arr, len(phases), M, qr, pg, ws, ws_bytes)


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
    """A bound sequence of C-ABI calls (``run`` appends the stream) and, for
    tensor parallelism, collective steps (Python callables on the current
    stream)."""
    calls: list = field(default_factory=list)
    # layers_plan(final_norm=True) that left the final RMSNorm of every row in xn
    final_normed: bool = False

    def add(self, name: str, *args):
        self.calls.append((name, getattr(_lib.load(), name), args))

    def add_py(self, name: str, fn):
        self.calls.append((name, None, fn))

    def extend(self, other: "Plan"):
        self.calls.extend(other.calls)

    def run(self, stream=None):
        s = _VP(torch.cuda.current_stream().cuda_stream if stream is None else stream)
        lib = _lib.load()
        for name, fn, args in self.calls:
            if fn is None:
                args()
                continue
            st = fn(*args, s)
            if st != 0:
                raise RuntimeError(f"{name} failed: status {st} ({lib.tsds_status_string(st).decode()})")

    def kernel_count(self) -> int:
        return sum(1 for c in self.calls if c[1] is not None)


class QwenModel:
    """Weights, KV cache and activation buffers of one Qwen3-shaped model.

    ``max_rows`` bounds the token rows of one forward (B * T).
    """

    def __init__(self, shape: QwenShape, batch: int, max_seq: int, max_rows: int, device="cuda",
                 weights: dict | None = None, seed: int = 0, split_keys: int = 1024, qk_norm: bool | None = None,
                 share_embeddings: "QwenModel | None" = None, rope_len: int | None = None,
                 tp_rank: int = 0, tp_size: int = 1, tp_layers: bool = True, tp_vocab: bool = True, comm=None,
                 peer=None, fused_layers: bool = False, share_weights: "QwenModel | None" = None,
                 kv: "PagedKV | None" = None):
        """``share_weights``: another model of the same shape and tensor-parallel
        layout whose layer weights, embedding, final norm and LM head this one
        uses (no copy): a second batch size over the same weights.
        ``kv``: paged KV memory in SGLang's layout (tri_sds_b200.paged.PagedKV:
        per-layer token pools + request-to-token table) used instead of the
        model's own contiguous cache; the default kernels' path only (no
        fused layers, no tcgen05 attention)."""
        self.shape = shape
        # tensor parallelism: layers and/or vocabulary sharded over tp_size ranks
        self.tp_rank = tp_rank
        self.layer_tp = tp_size if tp_layers else 1
        self.vocab_tp = share_embeddings.vocab_tp if share_embeddings is not None else (tp_size if tp_vocab else 1)
        if comm is None:
            comm = share_embeddings.comm if share_embeddings is not None else LocalComm()
        self.comm = comm
        # tp.PeerAllReduce: the row-parallel all-reduces run as this library's
        # peer-memory kernel instead of NCCL's (layers sharded only).  A
        # one-rank group (tp_size 1) runs the same kernels with nothing to
        # exchange: the peer paths on one GPU, bit for bit the plain plan.
        self.peer = peer
        if peer is not None:
            assert tp_layers and (peer.rank, peer.size) == (tp_rank, tp_size)
            assert peer.max_elems >= max_rows * shape.hidden
        # the vocab-parallel LM head exchanges candidates / logits through the
        # peer group's exchange region when it has one (the EAGLE head shares
        # the target's LM head and so its group)
        if share_embeddings is not None:
            self.lm_peer = share_embeddings.lm_peer
            self.lm_rows = share_embeddings.lm_rows
        else:
            vt = tp_size if tp_vocab else 1
            use = peer is not None and getattr(peer, "exchange_bytes", 0) > 0
            self.lm_peer = peer if use else None
            self.lm_rows = max_rows
            if use:
                assert peer.exchange_bytes >= lm_exchange_layout(max_rows, shape.vocab // vt)[2]
        if self.lm_peer is not None:
            assert max_rows <= self.lm_rows
        self.lshape = replace(shape, **local_dims(shape, self.layer_tp)) if self.layer_tp > 1 else shape
        self.vocab_local = shape.vocab // self.vocab_tp
        self.batch = batch
        self.max_seq = max_seq
        self.max_rows = max_rows
        self.device = torch.device(device)
        self.split_keys = split_keys
        self.qk_norm = shape.qk_norm if qk_norm is None else qk_norm
        s = shape
        ls = self.lshape
        dev = self.device
        if share_weights is not None:
            assert share_weights.shape == shape and share_weights.layer_tp == self.layer_tp
            assert share_weights.tp_rank == tp_rank and share_weights.vocab_tp == self.vocab_tp
            self.layers = share_weights.layers
        elif weights is not None:
            self.layers = [pack_layer(shard_layer(L, s, tp_rank, self.layer_tp), dev) for L in weights["layers"]]
        else:
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed)   # replicated tensors: the same on every rank
            lgen = torch.Generator(device=dev)
            lgen.manual_seed(seed + 7919 * (1 + tp_rank) if self.layer_tp > 1 else seed + 1)
            self.layers = [random_layer_gpu(ls, lgen, dev) for _ in range(s.n_layers)]
        if share_embeddings is not None or share_weights is not None:
            # the EAGLE head runs on the target's embedding, final norm and LM
            # head; a shared-weights model on the other model's
            src = share_embeddings if share_embeddings is not None else share_weights
            self.embed_w, self.lm_head_w, self.norm_w = src.embed_w, src.lm_head_w, src.norm_w
        elif weights is not None:
            self.embed_w = weights["embed"].to(dev, torch.bfloat16).contiguous()
            lm = self.embed_w if weights["lm_head"] is weights["embed"] else weights["lm_head"].to(dev, torch.bfloat16)
            self.lm_head_w = vocab_shard(lm, tp_rank, self.vocab_tp) if self.vocab_tp > 1 else lm.contiguous()
            self.norm_w = weights["norm"].to(dev, torch.bfloat16).contiguous()
        else:
            self.embed_w = (torch.randn(s.vocab, s.hidden, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
            if s.tie_embeddings:
                self.lm_head_w = vocab_shard(self.embed_w, tp_rank, self.vocab_tp) if self.vocab_tp > 1 \
                    else self.embed_w
            else:
                vgen = torch.Generator(device=dev)
                vgen.manual_seed(seed + 104729 * (1 + tp_rank))
                self.lm_head_w = (torch.randn(self.vocab_local, s.hidden, device=dev, generator=vgen) * 0.02
                                  ).to(torch.bfloat16)
            self.norm_w = (1.0 + 0.02 * torch.randn(s.hidden, device=dev, generator=gen)).to(torch.bfloat16)
        # RoPE tables cover absolute positions (the EAGLE head's small cache
        # holds rows of a tree whose positions continue the sequence)
        self.rope_len = max_seq if rope_len is None else rope_len
        self.cos, self.sin = precompute_rope(s.head_dim, self.rope_len, s.rope_theta, dev)
        self.kv = kv
        if kv is None:
            self.k_cache = torch.zeros(s.n_layers, batch, ls.n_kv_heads, max_seq, s.head_dim, dtype=torch.bfloat16,
                                       device=dev)
            self.v_cache = torch.zeros_like(self.k_cache)
        else:
            assert not fused_layers, "paged KV runs the per-op plan"
            assert len(kv.k_pools) == s.n_layers and kv.n_kv_heads == ls.n_kv_heads and kv.table_ld >= max_seq
            self.k_cache = self.v_cache = None
            self.out_loc = torch.zeros(max_rows, dtype=torch.int64, device=dev)   # the new tokens' pool rows
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=dev)   # committed rows per sequence
        M = max_rows
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(M, s.hidden, **bf)          # residual stream
        self.xn = torch.zeros(M, s.hidden, **bf)         # normed input of a projection
        self.qkv = torch.zeros(M, ls.qkv_dim, **bf)
        self.q = torch.zeros(M, ls.q_dim, **bf)
        self.attn = torch.zeros(M, ls.q_dim, **bf)
        self.h = torch.zeros(M, ls.intermediate, **bf)
        if self.layer_tp > 1:
            self.part = torch.zeros(M, s.hidden, dtype=torch.float32, device=dev)   # row-parallel partials
        if self.vocab_tp > 1:
            tpv = self.vocab_tp
            self.am_idx = torch.zeros(M, dtype=torch.int64, device=dev)
            self.am_val = torch.zeros(M, dtype=torch.float32, device=dev)
            self.am_idx_all = torch.zeros(tpv * M, dtype=torch.int64, device=dev)
            self.am_val_all = torch.zeros(tpv * M, dtype=torch.float32, device=dev)
            self.logits_local = None   # allocated on first use with full logits
        self.starts = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(M, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        T_max = max(1, M // batch)
        self.attn_ws_bytes = max(
            _lib.query("tsds_attention_workspace_bytes", batch, t, ls.n_heads, ls.n_kv_heads, s.head_dim, max_seq,
                       split_keys) for t in range(1, T_max + 1))
        self.attn_ws = torch.empty(max(self.attn_ws_bytes, 16), dtype=torch.uint8, device=dev)
        lin = [(ls.qkv_dim, s.hidden), (s.hidden, ls.q_dim), (ls.intermediate, s.hidden), (s.hidden, ls.intermediate)]
        self.lin_ws_bytes = max(_lib.query("tsds_linear_workspace_bytes", m, o, k) for o, k in lin
                                for m in range(1, M + 1))
        # zero-filled once: the tcgen05 tile counters live in these and every
        # launch leaves them zero again
        self.lin_ws = torch.zeros(max(self.lin_ws_bytes, 16), dtype=torch.uint8, device=dev)
        self.lm_ws_bytes = max(_lib.query("tsds_lm_head_workspace_bytes", m, self.vocab_local)
                               for m in range(1, M + 1))
        self.lm_ws = torch.zeros(max(self.lm_ws_bytes, 16), dtype=torch.uint8, device=dev)
        # fused-layer kernel (one launch for O -> norm -> gate/up -> down ->
        # norm -> q/k/v of consecutive layers, under tensor parallelism with
        # the peer all-reduces as phases); its own zero-filled workspace
        self.fused_layers = fused_layers and (self.layer_tp == 1 or peer is not None)
        # True: the per-op plan's residual GEMMs (O, down) also apply the
        # RMSNorm that follows them (tsds_linear_residual_norm: one launch,
        # the same bits as the two).  Off by default: measured slower on a
        # B200 (B=1 EAGLE cycle 59.0 vs 61.6 tok/s) - the GEMM's tail (every
        # CTA's fence and report, then a few CTAs normalising one row each
        # while the next projection's CTAs stream their first weight tiles)
        # costs more than the separate RMSNorm launch and its kernel boundary.
        self.fuse_norm = False
        if self.fused_layers:
            self.fused_ws_bytes = _lib.query("tsds_fused_layer_workspace_bytes", M)
            self.fused_ws = torch.zeros(self.fused_ws_bytes, dtype=torch.uint8, device=dev)

    # -- launch plans ---------------------------------------------------------
    def layers_plan(self, B: int, T: int, tree_mask: torch.Tensor | None = None, mask_origin: int = -1,
                    x: torch.Tensor | None = None, starts: torch.Tensor | None = None,
                    positions: torch.Tensor | None = None, final_norm: bool = False) -> Plan:
        """All decoder layers over rows x[0:B*T] (embedded already), with
        starts/positions already prepared.  ``x`` / ``starts`` /
        ``positions`` default to the model's own buffers; ``tree_mask`` +
        ``mask_origin`` select the attention mask (see tsds_verify_attention).
        Under tensor parallelism the O and down projections produce fp32
        partials that are all-reduced before the residual add.  Without it
        (``fuse_norm``) each O / down projection also applies the RMSNorm
        that reads its output - the layer's post-attention norm, the next
        layer's input norm and, with ``final_norm``, the final norm into
        ``xn``; the returned plan's ``final_normed`` then tells head_plan to
        skip its own."""
        s, ls = self.shape, self.lshape
        M = B * T
        assert M <= self.max_rows and B == self.batch
        eps = s.eps
        pl = Plan()
        lw, lb = self.lin_ws, self.lin_ws_bytes
        qn = self.qk_norm
        xb = self.x if x is None else x
        st = self.starts if starts is None else starts
        ps = self.positions if positions is None else positions
        tp = self.layer_tp > 1
        if self.fused_layers:
            return self._fused_layers_plan(B, T, tree_mask, mask_origin, xb, st, ps)
        n_peer = [0]

        def row_parallel(src, ld_src, w, k_in, norm_w=None):
            """The row-parallel projection + residual add; True when it also
            wrote RMSNorm(x) with norm_w into xn."""
            if not tp and self.peer is None:
                if norm_w is not None and self.fuse_norm:
                    pl.add("tsds_linear_residual_norm", _p(src), ld_src, _p(w), _p(xb), _p(xb), s.hidden, M, s.hidden,
                           k_in, _p(norm_w), _p(self.xn), s.hidden, eps, _p(lw), lb)
                    return True
                pl.add("tsds_linear_residual", _p(src), ld_src, _p(w), _p(xb), _p(xb), s.hidden, M, s.hidden, k_in,
                       _p(lw), lb)
                return False
            if self.peer is not None:
                # the partial goes straight into this rank's peer slot; calls alternate slots
                slot = n_peer[0] % 2
                n_peer[0] += 1
                pl.add("tsds_linear_f32", _p(src), ld_src, _p(w), self.peer.slot_ptr(slot), s.hidden, M, s.hidden,
                       k_in, _p(lw), lb)
                pl.add("tsds_peer_allreduce_residual", _p(xb), self.peer.bufs, self.tp_rank, self.layer_tp, slot, M,
                       s.hidden, self.peer.max_elems, _p(self.status))
                return False
            part = self.part[:M]
            pl.add("tsds_linear_f32", _p(src), ld_src, _p(w), _p(part), s.hidden, M, s.hidden, k_in, _p(lw), lb)
            pl.add_py("all_reduce", lambda part=part: self.comm.all_reduce(part))
            pl.add("tsds_residual_add_f32", _p(xb), _p(part), M, s.hidden)
            return False

        kv = self.kv
        if kv is not None:
            # the new tokens' pool rows (SGLang's out_cache_loc) from the table
            pl.add("tsds_table_rows", _p(kv.table), kv.table_ld, _p(kv.req_rows), _p(st), B, T, _p(self.out_loc))
        normed = False   # xn already holds this layer's input norm
        nl = len(self.layers)
        for i, L in enumerate(self.layers):
            if not normed:
                pl.add("tsds_rms_norm", _p(xb), _p(L.ln1), _p(self.xn), M, s.hidden, s.hidden, s.hidden, eps)
            pl.add("tsds_linear", _p(self.xn), s.hidden, _p(L.w_qkv), _p(self.qkv), ls.qkv_dim, M, ls.qkv_dim,
                   s.hidden, _p(lw), lb)
            if kv is None:
                kc, vc = self.k_cache[i], self.v_cache[i]
                pl.add("tsds_qk_norm_rope_kv", _p(self.qkv), _p(L.q_norm) if qn else None,
                       _p(L.k_norm) if qn else None, _p(self.cos), _p(self.sin), _p(ps), _p(st),
                       _p(self.q), _p(kc), _p(vc), B, T, ls.n_heads, ls.n_kv_heads, s.head_dim, self.max_seq,
                       self.rope_len, eps)
                pl.add("tsds_verify_attention", _p(self.q), _p(kc), _p(vc), _p(self.attn), _p(st),
                       _p(tree_mask), mask_origin, B, T, ls.n_heads, ls.n_kv_heads, s.head_dim, self.max_seq,
                       self.max_seq, self.split_keys, float(s.head_dim ** -0.5), _p(self.attn_ws),
                       self.attn_ws_bytes, _p(self.status))
            else:
                kp, vp = kv.k_pools[i], kv.v_pools[i]
                pl.add("tsds_qk_norm_rope_kv_paged", _p(self.qkv), _p(L.q_norm) if qn else None,
                       _p(L.k_norm) if qn else None, _p(self.cos), _p(self.sin), _p(ps), _p(self.out_loc),
                       _p(self.q), _p(kp), _p(vp), M, ls.n_heads, ls.n_kv_heads, s.head_dim, kv.pool_rows,
                       self.rope_len, eps, _p(self.status))
                pl.add("tsds_verify_attention_paged", _p(self.q), _p(kp), _p(vp), _p(self.attn), _p(st),
                       _p(tree_mask), mask_origin, _p(kv.table), kv.table_ld, _p(kv.req_rows), kv.pool_rows,
                       kv.page_size, B, T, ls.n_heads, ls.n_kv_heads, s.head_dim, self.max_seq, self.split_keys,
                       float(s.head_dim ** -0.5), _p(self.attn_ws), self.attn_ws_bytes, _p(self.status))
            if not row_parallel(self.attn, ls.q_dim, L.w_o, ls.q_dim, norm_w=L.ln2):
                pl.add("tsds_rms_norm", _p(xb), _p(L.ln2), _p(self.xn), M, s.hidden, s.hidden, s.hidden, eps)
            pl.add("tsds_linear_swiglu", _p(self.xn), s.hidden, _p(L.w_gu), _p(self.h), ls.intermediate, M,
                   ls.intermediate, s.hidden, _p(lw), lb)
            nxt = self.layers[i + 1].ln1 if i + 1 < nl else (self.norm_w if final_norm else None)
            normed = row_parallel(self.h, ls.intermediate, L.w_d, ls.intermediate, norm_w=nxt)
        assert n_peer[0] % 2 == 0   # the next plan run starts on slot 0 again
        pl.final_normed = bool(final_norm and normed)
        return pl

    def _fused_layers_plan(self, B: int, T: int, tree_mask, mask_origin: int, xb, st, ps) -> Plan:
        """layers_plan with the fused-layer kernel: per layer one attention
        launch and one fused launch [O (+res) -> norm -> gate/up -> down (+res) ->
        next layer's norm -> q/k/v (+QK-norm, RoPE, KV write)]; the first
        is [norm -> q/k/v] of layer 0.  Same rounding as the per-op
        plan.  Under tensor parallelism O and down store fp32 partials into
        this rank's peer slots (alternating) and a peer all-reduce phase
        adds their sum over the ranks to the residual."""
        s, ls = self.shape, self.lshape
        M = B * T
        eps = s.eps
        qn = self.qk_norm
        pl = Plan()
        N = s.hidden
        peer = self.peer
        # two-shot all-reduce once a rank would pull more than TWO_SHOT_BYTES
        # of the other ranks' partials in one shot (same bits either way)
        two_shot = peer is not None and M * N * 4 * (peer.size - 1) > TWO_SHOT_BYTES

        def row_parallel(src, K, w, slot):
            if peer is None:
                return [gemm(_lib.EPI_RESIDUAL, src, K, w, N, out=xb, res=xb)]
            part = dict(gemm(_lib.EPI_STORE_F32, src, K, w, N), out=peer.slot_ptr(slot), ldo=N)
            reduce = dict(kind=_lib.PHASE_PEER, epi=int(two_shot), x=None, ldx=0, K=N, w=None, n_out=slot, res_ld=0,
                          res=None, out=_p(xb), ldo=N, eps=0.0)
            return [part, reduce]

        def norm(w):
            return dict(kind=_lib.PHASE_NORM, epi=0, x=_p(xb), ldx=N, K=N, w=_p(w), n_out=0, res_ld=0, res=None,
                        out=_p(self.xn), ldo=N, eps=eps)

        def gemm(epi, x, K, w, n_out, out=None, res=None):
            return dict(kind=_lib.PHASE_GEMM, epi=epi, x=_p(x), ldx=K, K=K, w=_p(w), n_out=n_out,
                        res_ld=N if res is not None else 0, res=_p(res), out=_p(out),
                        ldo=n_out if out is not None else 0, eps=0.0)

        def qkv(i):
            L = self.layers[i]
            rope = dict(q_norm_w=_p(L.q_norm) if qn else None, k_norm_w=_p(L.k_norm) if qn else None,
                        cos=_p(self.cos), sin=_p(self.sin), positions=_p(ps), starts=_p(st), q_out=_p(self.q),
                        k_cache=_p(self.k_cache[i]), v_cache=_p(self.v_cache[i]), T=T, Hq=ls.n_heads,
                        Hkv=ls.n_kv_heads, S=self.max_seq, rope_len=self.rope_len, eps=eps)
            return [norm(L.ln1), gemm(_lib.EPI_QKROPE, self.xn, N, L.w_qkv, ls.qkv_dim)], rope

        phases, rope = qkv(0)
        pl.add("tsds_fused_layer", *_fused_args(phases, rope, peer, M, _p(self.fused_ws), self.fused_ws_bytes))
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            kc, vc = self.k_cache[i], self.v_cache[i]
            pl.add("tsds_verify_attention", _p(self.q), _p(kc), _p(vc), _p(self.attn), _p(st),
                   _p(tree_mask), mask_origin, B, T, ls.n_heads, ls.n_kv_heads, s.head_dim, self.max_seq,
                   self.max_seq, self.split_keys, float(s.head_dim ** -0.5), _p(self.attn_ws), self.attn_ws_bytes,
                   _p(self.status))
            phases = (row_parallel(self.attn, ls.q_dim, L.w_o, 0)
                      + [norm(L.ln2), gemm(_lib.EPI_SWIGLU, self.xn, N, L.w_gu, ls.intermediate, out=self.h)]
                      + row_parallel(self.h, ls.intermediate, L.w_d, 1))
            rope = None
            if i + 1 < n:
                nxt, rope = qkv(i + 1)
                phases += nxt
            pl.add("tsds_fused_layer", *_fused_args(phases, rope, peer, M, _p(self.fused_ws), self.fused_ws_bytes))
        return pl

    def head_plan(self, B: int, T: int, argmax_out: torch.Tensor, argmax_stride: int, last_only: bool,
                  logits_out: torch.Tensor | None = None, x: torch.Tensor | None = None,
                  normed: bool = False) -> Plan:
        """Final RMSNorm + LM head + argmax over all rows, or only the last
        row of each sequence (``normed``: xn already holds the final norm of
        all rows, from layers_plan(final_norm=True)).  With a vocab-parallel
        LM head each rank picks its shard's best (value, index), the
        candidates are all-gathered and merged (ties: lowest global index);
        full logits, when requested, are all-gathered and reassembled."""
        s = self.shape
        pl = Plan()
        xb = self.x if x is None else x
        rows, ld = (B, T * s.hidden) if last_only else (B * T, s.hidden)
        src = xb[T - 1:] if last_only else xb
        if not (normed and not last_only):
            pl.add("tsds_rms_norm", _p(src), _p(self.norm_w), _p(self.xn), rows, s.hidden, ld, s.hidden, s.eps)
        if self.vocab_tp == 1 and self.lm_peer is None:
            pl.add("tsds_lm_head_argmax", _p(self.xn), s.hidden, _p(self.lm_head_w), _p(logits_out), _p(argmax_out),
                   argmax_stride, None, rows, s.vocab, s.hidden, _p(self.lm_ws), self.lm_ws_bytes)
            return pl
        tpv, vl = self.vocab_tp, self.vocab_local
        if self.lm_peer is not None:
            # the shard's candidates / logits straight into this rank's exchange
            # region, gathered over peer memory (no NCCL)
            g = self.lm_peer
            val_off, log_off, _ = lm_exchange_layout(self.lm_rows, vl)
            want = logits_out is not None
            pl.add("tsds_lm_head_argmax", _p(self.xn), s.hidden, _p(self.lm_head_w),
                   g.exchange_at(log_off) if want else None, g.exchange_at(0), 1, g.exchange_at(val_off), rows, vl,
                   s.hidden, _p(self.lm_ws), self.lm_ws_bytes)
            pl.add("tsds_peer_lm_gather", g.bufs, g.rank, g.size, g.max_elems, g.exchange_bytes, rows, vl, val_off,
                   log_off if want else 0, _p(argmax_out), argmax_stride, _p(logits_out), _p(self.status))
            return pl
        loc = None
        if logits_out is not None:
            need = rows * vl
            if self.logits_local is None or self.logits_local.numel() < need:
                self.logits_local = torch.zeros(self.max_rows * vl, dtype=torch.bfloat16, device=self.device)
                self.logits_all = torch.zeros(tpv * self.max_rows * vl, dtype=torch.bfloat16, device=self.device)
            loc = self.logits_local[:need]
        pl.add("tsds_lm_head_argmax", _p(self.xn), s.hidden, _p(self.lm_head_w), _p(loc), _p(self.am_idx), 1,
               _p(self.am_val), rows, vl, s.hidden, _p(self.lm_ws), self.lm_ws_bytes)
        vi, vv = self.am_idx[:rows], self.am_val[:rows]
        ai, av = self.am_idx_all[:tpv * rows], self.am_val_all[:tpv * rows]
        pl.add_py("all_gather", lambda: (self.comm.all_gather(ai, vi), self.comm.all_gather(av, vv)))
        pl.add("tsds_argmax_merge", _p(av), _p(ai), rows, tpv, vl, _p(argmax_out), argmax_stride)
        if logits_out is not None:
            allb = self.logits_all[:tpv * rows * vl]
            pl.add_py("all_gather", lambda: self.comm.all_gather(allb, loc))
            pl.add("tsds_gather_shards", _p(allb), _p(logits_out), tpv, rows, vl)
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
        lp = self.layers_plan(B, T, final_norm=not last_only)
        pl.extend(lp)
        pl.extend(self.head_plan(B, T, argmax_out, argmax_stride, last_only, logits_out, normed=lp.final_normed))
        return pl

    # -- prefill (untimed set-up, on this library's kernels) ---------------------
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        """Process a [B, P] prompt from row 0; returns the hidden states
        [B, P, N] (pre final norm) and sets lengths = P.  Ragged prompts:
        ``lengths[b]`` (1..P) real tokens at the start of row b, the rest
        padding; the causal attention keeps every real token's state
        independent of the padding behind it, and lengths = lengths (the
        padding's cache rows lie past the sequence and are overwritten by the
        next forward).

        Every step runs on this library's kernels (qwen_model.py:100-146 at
        T = P): the embedding gather, RMSNorm, the tcgen05 GEMMs over row
        chunks of at most 256 (their epilogues: plain, SwiGLU, residual; the
        fp32 partial + all-reduce + residual add under tensor parallelism),
        QK-norm/RoPE/KV write, and the prompt's causal attention - the
        tcgen05 kernel in one call when it is switched on, else the verify
        kernel over query chunks of at most 1024 / (q heads per kv head)
        tokens, chunk c attending to the cache rows below it like a verify
        step that starts at c."""
        from . import ops
        s, ls = self.shape, self.lshape
        B, P = prompt.shape
        assert P <= self.max_seq, "prompt longer than the cache"
        if lengths is not None:
            lengths = torch.as_tensor(lengths).to(torch.int32)
            assert lengths.shape == (B,) and int(lengths.min()) >= 1 and int(lengths.max()) <= P, \
                "prompt lengths must be in 1..P"
        dev = self.device
        M = B * P
        bf = dict(dtype=torch.bfloat16, device=dev)
        x = ops.embed(prompt.to(dev, torch.int64).reshape(-1).contiguous(), self.embed_w)
        pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(B)
        starts = torch.zeros(B, dtype=torch.int32, device=dev)
        xn = torch.empty(M, s.hidden, **bf)
        qkv = torch.empty(M, ls.qkv_dim, **bf)
        q = torch.empty(M, ls.q_dim, **bf)
        a = torch.empty(M, ls.q_dim, **bf)
        h = torch.empty(M, ls.intermediate, **bf)
        part = torch.empty(M, s.hidden, dtype=torch.float32, device=dev) if self.layer_tp > 1 else None
        chunks = [(r, min(M, r + 256)) for r in range(0, M, 256)]

        def row_parallel(inp, w):
            """x += inp @ w^T (all-reduced over the tensor-parallel ranks)."""
            for r0, r1 in chunks:
                if part is None:
                    ops.linear_residual(inp[r0:r1], w, x[r0:r1], out=x[r0:r1])
                else:
                    ops.linear_f32(inp[r0:r1], w, out=part[r0:r1])
            if part is not None:
                self.comm.all_reduce(part)
                ops.residual_add_f32(x, part)

        G = ls.n_heads // ls.n_kv_heads
        Tc = max(1, 1024 // G)   # query tokens per call of the verify kernel
        kv = self.kv
        if kv is not None:
            loc = torch.empty(M, dtype=torch.int64, device=dev)
            _lib.call("tsds_table_rows", _p(kv.table), kv.table_ld, _p(kv.req_rows), _p(starts), B, P, _p(loc),
                      ops._stream())
        for i, L in enumerate(self.layers):
            ops.rms_norm(x, L.ln1, s.eps, out=xn)
            for r0, r1 in chunks:
                ops.linear(xn[r0:r1], L.w_qkv, out=qkv[r0:r1])
            qn_w, kn_w = (L.q_norm, L.k_norm) if self.qk_norm else (None, None)
            qv = q.view(B, P, ls.n_heads, s.head_dim)
            av = a.view(B, P, ls.n_heads, s.head_dim)
            if kv is not None:
                kp, vp = kv.k_pools[i], kv.v_pools[i]
                ops.qk_norm_rope_kv_paged(qkv, qn_w, kn_w, self.cos, self.sin, pos, loc, q, kp, vp, ls.n_heads,
                                          ls.n_kv_heads, s.eps)
                for c0 in range(0, P, Tc):
                    c1 = min(P, c0 + Tc)
                    st = torch.full((B,), c0, dtype=torch.int32, device=dev)
                    av[:, c0:c1] = ops.verify_attention_paged(
                        qv[:, c0:c1].contiguous(), kp, vp, st, kv.table, req_rows=kv.req_rows,
                        page_size=kv.page_size, max_kv=c1, split_keys=self.split_keys)
                row_parallel(a, L.w_o)
                ops.rms_norm(x, L.ln2, s.eps, out=xn)
                for r0, r1 in chunks:
                    ops.linear_swiglu(xn[r0:r1], L.w_gu, out=h[r0:r1])
                row_parallel(h, L.w_d)
                continue
            kc, vc = self.k_cache[i], self.v_cache[i]
            ops.qk_norm_rope_kv(qkv, qn_w, kn_w, self.cos, self.sin, pos, starts, q, kc, vc, B, P, ls.n_heads,
                                ls.n_kv_heads, s.eps)
            if ops.attention_tc():
                # every prompt row of a kv head in one call, one key split (no combine pass)
                ops.verify_attention(qv, kc, vc, starts, max_kv=P, split_keys=(P + 127) // 128 * 128, out=av)
            else:
                for c0 in range(0, P, Tc):
                    c1 = min(P, c0 + Tc)
                    st = torch.full((B,), c0, dtype=torch.int32, device=dev)
                    av[:, c0:c1] = ops.verify_attention(qv[:, c0:c1].contiguous(), kc, vc, st, max_kv=c1,
                                                        split_keys=self.split_keys)
            row_parallel(a, L.w_o)
            ops.rms_norm(x, L.ln2, s.eps, out=xn)
            for r0, r1 in chunks:
                ops.linear_swiglu(xn[r0:r1], L.w_gu, out=h[r0:r1])
            row_parallel(h, L.w_d)
        if lengths is None:
            self.lengths.fill_(P)
        else:
            self.lengths.copy_(lengths.to(dev))
        return x.reshape(B, P, s.hidden)

    @staticmethod
    def last_rows(hidden: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        """hidden[b, lengths[b] - 1] for every b (the last real token of
        ragged prompts; the last column without lengths)."""
        if lengths is None:
            return hidden[:, -1]
        idx = torch.as_tensor(lengths).to(device=hidden.device, dtype=torch.int64) - 1
        return hidden[torch.arange(hidden.shape[0], device=hidden.device), idx]

    def logits_of(self, hidden: torch.Tensor) -> torch.Tensor:
        """Final norm + full bf16 logits (set-up / tests only)."""
        from . import ops
        xn = ops.rms_norm(hidden.reshape(-1, self.shape.hidden).contiguous(), self.norm_w, self.shape.eps)
        loc = torch.cat([ops.lm_head_argmax(xn[r:r + 256], self.lm_head_w, return_logits=True)[1]
                         for r in range(0, xn.shape[0], 256)])
        if self.vocab_tp == 1:
            return loc
        allv = torch.empty(self.vocab_tp * loc.numel(), dtype=loc.dtype, device=loc.device)
        self.comm.all_gather(allv, loc.contiguous().reshape(-1))
        return allv.reshape(self.vocab_tp, *loc.shape).permute(1, 0, 2).reshape(loc.shape[0], -1)

    def status_regions(self) -> list:
        """(status word, header, on_error) for each place this model's
        kernels record errors (a bounded device wait that gave up): the
        attention / peer status word, and word 0 of the tcgen05 GEMM, LM-head
        and fused-layer workspaces, whose header (status + tile counters) is
        cleared with the word.  A model with a peer group retires the group
        on any error: the ranks' per-CTA epochs no longer agree."""
        hl = _lib.query("tsds_linear_workspace_header_bytes")
        on_error = self._retire_peer if self.peer is not None else None
        regs = [(self.status, None, on_error),
                (self.lin_ws[:4].view(torch.int32), self.lin_ws[:min(hl, self.lin_ws.numel())], on_error),
                (self.lm_ws[:4].view(torch.int32), self.lm_ws[:min(hl, self.lm_ws.numel())], on_error)]
        if self.fused_layers:
            hf = _lib.query("tsds_fused_layer_workspace_header_bytes")
            regs.append((self.fused_ws[:4].view(torch.int32), self.fused_ws[:min(hf, self.fused_ws.numel())],
                         on_error))
        return regs

    def status_words(self) -> list:
        """The device status words of status_regions (one int32 each)."""
        return [r[0] for r in self.status_regions()]

    def _retire_peer(self):
        self.peer.broken = True

    def ensure_usable(self):
        """Raise before a launch on a peer group retired by a device error."""
        if self.peer is not None and getattr(self.peer, "broken", False):
            raise RuntimeError("the peer all-reduce group was retired after a device wait gave up (its ranks' "
                               "epochs no longer agree): build a new PeerAllReduce on every rank")

    def check_status(self):
        """Raise if a kernel recorded an error in a status word (clears it
        and the counters beside it)."""
        for w, header, on_error in self.status_regions():
            raise_status(w, int(w.item()), header, on_error)

"""Tensor-parallel shard rules on CPU: 2, 4 and 8 gloo ranks, each holding the
tri_sds_b200.tp shards of an oracle layer, reproduce the unsharded layer
(fp32) after the all-reduces, and the vocab-parallel argmax merge picks the
full argmax (ties: lowest global index)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle.qwen import QwenOracle, QwenShape, apply_rope, random_qwen_weights, rms_norm

SHAPE = QwenShape(hidden=64, n_heads=8, n_kv_heads=4, head_dim=16, intermediate=128, n_layers=1, vocab=96)
# 8 ranks: one kv head per rank, as the 32B shape at tp = 8
SHAPE8 = QwenShape(hidden=64, n_heads=16, n_kv_heads=8, head_dim=16, intermediate=128, n_layers=1, vocab=96)


def _tp_layer(L, x, pos, shape, rank, tp, cos, sin):
    """One decoder layer with rank-local shards; prefill (causal) over x [1, T, N], fp32."""
    from tri_sds_b200.tp import shard_layer
    W = shard_layer(L, shape, rank, tp)
    s = shape
    hq, hk = s.n_heads // tp, s.n_kv_heads // tp
    T = x.shape[1]
    xn = rms_norm(x, L["ln1"])
    q = (xn @ W["q"].T).reshape(1, T, hq, s.head_dim)
    k = (xn @ W["k"].T).reshape(1, T, hk, s.head_dim)
    v = (xn @ W["v"].T).reshape(1, T, hk, s.head_dim)
    q = apply_rope(rms_norm(q, L["q_norm"]).transpose(1, 2), cos, sin, pos)
    k = apply_rope(rms_norm(k, L["k_norm"]).transpose(1, 2), cos, sin, pos)
    v = v.transpose(1, 2)
    rep = hq // hk
    a = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1), is_causal=True)
    part = a.transpose(1, 2).reshape(1, T, hq * s.head_dim) @ W["o"].T
    dist.all_reduce(part)
    x = x + part
    xn2 = rms_norm(x, L["ln2"])
    part = (F.silu(xn2 @ W["gate"].T) * (xn2 @ W["up"].T)) @ W["down"].T
    dist.all_reduce(part)
    return x + part


def _worker(rank, tp, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=tp)
    SHAPE = SHAPE8 if tp == 8 else globals()["SHAPE"]
    try:
        from tri_sds_b200.tp import vocab_shard
        w = random_qwen_weights(SHAPE, seed=5, dtype=torch.float32, std=0.2)
        ids = torch.randint(0, SHAPE.vocab, (1, 9), generator=torch.Generator().manual_seed(6))
        ora = QwenOracle(SHAPE, w, batch=1, max_seq=32, dtype=torch.float32)
        x = ora.embed_w[ids]
        pos = torch.arange(9)
        got = _tp_layer(w["layers"][0], x, pos, SHAPE, rank, tp, ora.cos, ora.sin)
        ref = ora.layer(0, x.clone(), torch.zeros(1, dtype=torch.int64), pos, None)
        err = (got - ref).abs().max().item()
        # vocab-parallel LM head: local argmax candidates, gathered, merged
        h = rms_norm(ref, ora.norm_w)[0]
        local = h @ vocab_shard(w["lm_head"], rank, tp).T
        lv, li = local.max(-1)
        vals = [torch.zeros_like(lv) for _ in range(tp)]
        idxs = [torch.zeros_like(li) for _ in range(tp)]
        dist.all_gather(vals, lv)
        dist.all_gather(idxs, li)
        shard = SHAPE.vocab // tp
        merged = []
        for m in range(h.shape[0]):
            best = min(range(tp), key=lambda r: (-float(vals[r][m]), int(idxs[r][m]) + r * shard))
            merged.append(int(idxs[best][m]) + best * shard)
        full = (h @ w["lm_head"].T).argmax(-1).tolist()
        q.put((rank, err, merged == full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_layer_and_vocab_parallel_argmax_match_unsharded(tp):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(daemon=True, target=_worker, args=(r, tp, port, q)) for r in range(tp)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=120) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():  # a rank stuck in teardown must not keep the session waiting
                p.terminate()
    for rank, err, ok in res:
        assert err <= 5e-5, (rank, err)  # fp32 sums over up to 8 rank partials
        assert ok, rank

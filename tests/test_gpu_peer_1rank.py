"""The peer-memory kernels on one GPU, as a one-rank group (tp = 1).

A one-rank tp.PeerAllReduce runs every peer path of the library with nothing
to exchange - the flag meetings meet only their own CTA, the sums run over
one partial - so its results equal the plain plan bit for bit:

* tsds_peer_allreduce_residual against x + bf16(partial), over alternating
  slots;
* torch.ops.tsds.allreduce_oneshot the same way;
* a verify forward of a 4B-shape model with the peer all-reduces, per-op and
  fused (one-shot and two-shot peer phases), with the LM head through the
  exchange region and tsds_peer_lm_gather, against the same model without a
  peer group: hidden state, q, caches, logits and argmax equal.
The two-rank forms are in test_gpu_tp.py."""

import pytest
import torch

from oracle import qwen as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
Q4B = dict(hidden=2560, n_heads=32, n_kv_heads=8, head_dim=128, intermediate=9728, n_layers=2, vocab=1000)


def _peer(max_elems, exchange_bytes=0):
    from tri_sds_b200.tp import PeerAllReduce
    return PeerAllReduce(0, 1, max_elems, exchange_bytes=exchange_bytes)


@pytest.mark.parametrize("M,N", [(1, 256), (26, 5120), (208, 5120)])
def test_allreduce_residual_one_rank(M, N):
    from tri_sds_b200 import _lib, ops
    peer = _peer(M * N)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(M)
    try:
        for call in range(4):
            slot = call % 2
            part = torch.randn(M, N, generator=g)
            x = torch.randn(M, N, generator=g).to(torch.bfloat16)
            peer.slot_tensor(slot, M * N).copy_(part.reshape(-1).to(DEV))
            xd = x.to(DEV)
            _lib.call("tsds_peer_allreduce_residual", ops._p(xd), peer.bufs, 0, 1, slot, M, N, peer.max_elems,
                      ops._p(status), ops._stream())
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            ref = (x.float() + part.to(torch.bfloat16).float()).to(torch.bfloat16)
            assert torch.equal(xd.cpu(), ref), call
    finally:
        torch.cuda.synchronize()
        peer.close()


def test_allreduce_oneshot_op_one_rank():
    import tri_sds_b200.torch_ops  # noqa: F401
    from tri_sds_b200 import tp
    M, N = 26, 2560
    peer = _peer(M * N)
    gid = tp.register_peer_group(peer)
    g = torch.Generator().manual_seed(3)
    try:
        for _ in range(3):
            part = torch.randn(M, N, generator=g)
            x = torch.randn(M, N, generator=g).to(torch.bfloat16)
            xd = x.to(DEV)
            torch.ops.tsds.allreduce_oneshot(xd, part.to(DEV), gid)
            torch.cuda.synchronize()
            assert torch.equal(xd.cpu(), (x.float() + part.to(torch.bfloat16).float()).to(torch.bfloat16))
    finally:
        torch.cuda.synchronize()
        peer.close()


@pytest.mark.parametrize("fused,two_shot", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("B,T", [(1, 26), (8, 26)])
def test_model_with_one_rank_peer_group_is_bitwise_plain(monkeypatch, fused, two_shot, B, T):
    import tri_sds_b200.model as model
    from tri_sds_b200 import ops
    from tri_sds_b200.model import QwenModel
    from tri_sds_b200.shapes import QwenShape
    from tri_sds_b200.tp import lm_exchange_layout
    if two_shot:
        monkeypatch.setattr(model, "TWO_SHOT_BYTES", -1)   # every peer phase two-shot, even with one rank
    ops.set_gemv_max_rows(0)
    S, rows = 1024, B * T
    oshape = oq.QwenShape(**Q4B)
    w = oq.random_qwen_weights(oshape, seed=B + T, std=0.02)
    peer = _peer(rows * Q4B["hidden"], exchange_bytes=lm_exchange_layout(rows, Q4B["vocab"])[2])
    try:
        plain = QwenModel(QwenShape(**Q4B), batch=B, max_seq=S, max_rows=rows, device=DEV, weights=w,
                          fused_layers=fused)
        viap = QwenModel(QwenShape(**Q4B), batch=B, max_seq=S, max_rows=rows, device=DEV, weights=w,
                         fused_layers=fused, tp_rank=0, tp_size=1, peer=peer)
        assert viap.lm_peer is peer and viap.fused_layers == fused
        g = torch.Generator().manual_seed(7)
        starts = torch.randint(0, S - T - 1, (B,), generator=g).to(torch.int32)
        ids = torch.randint(0, Q4B["vocab"], (B, T), generator=g)
        kpre = torch.randn(2, B, 8, S, 128, generator=g).to(torch.bfloat16)
        vpre = torch.randn(2, B, 8, S, 128, generator=g).to(torch.bfloat16)
        outs = []
        for m in (plain, viap):
            m.k_cache.copy_(kpre.to(DEV))
            m.v_cache.copy_(vpre.to(DEV))
            m.lengths.copy_(starts.to(DEV))
            am = torch.zeros(rows, dtype=torch.int64, device=DEV)
            logits = torch.zeros(rows, Q4B["vocab"], dtype=torch.bfloat16, device=DEV)
            m.forward_plan(ids.to(DEV).contiguous(), 1, B, T, m.lengths, 0, am, 1, logits_out=logits).run()
            torch.cuda.synchronize()
            m.check_status()
            outs.append((m.x[:rows].clone(), m.q[:rows].clone(), m.k_cache.clone(), m.v_cache.clone(), logits, am))
        for a, b, what in zip(outs[0], outs[1], ("hidden", "q", "k cache", "v cache", "logits", "argmax")):
            assert torch.equal(a, b), what
    finally:
        torch.cuda.synchronize()
        peer.close()

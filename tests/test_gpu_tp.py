"""Tensor parallelism on 2 GPUs: the TP=2 verify forward vs the oracle, and
greedy speculative decoding (chain draft and EAGLE tree, whose commit
compacts each rank's shard of the KV cache) == greedy autoregressive
decoding under TP=2, with the row-parallel all-reduces by NCCL or by the
library's peer-memory kernel (standalone, or as phases of the fused-layer
kernel), and the chain leg once more with the draft model tensor-parallel
over the same ranks.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import qwen as oq

pytestmark = pytest.mark.gpu
SMALL = dict(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, n_layers=2, vocab=1000)


def _worker(rank, port, q, allreduce):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120))
    try:
        from tri_sds_b200 import ops
        from tri_sds_b200.engine import AutoregressiveEngine, SpecEngine
        from tri_sds_b200.model import QwenModel
        from tri_sds_b200.shapes import QwenShape
        from tri_sds_b200.tp import Comm, PeerAllReduce
        ops.set_gemv_max_rows(0)
        dev = torch.device("cuda", rank)
        comm = Comm()
        # one set of peer buffers for every TP model here (their calls run in stream order)
        from tri_sds_b200.tp import lm_exchange_layout
        # with an exchange region: the vocab-parallel LM heads gather over peer memory too
        peer = (PeerAllReduce(rank, 2, 2 * 26 * SMALL["hidden"],
                              exchange_bytes=lm_exchange_layout(2 * 26, SMALL["vocab"] // 2)[2])
                if allreduce != "nccl" else None)
        fused = allreduce == "peer+fused"   # the all-reduces as phases of the fused-layer kernel
        oshape = oq.QwenShape(**SMALL)
        shape = QwenShape(**SMALL)
        w = oq.random_qwen_weights(oshape, seed=1, std=0.02)
        B, P, T = 2, 12, 5
        g = torch.Generator().manual_seed(2)
        prompt = torch.randint(0, oshape.vocab, (B, P), generator=g)
        step = torch.randint(0, oshape.vocab, (B, T), generator=g)
        m = QwenModel(shape, B, 128, B * T, device=dev, weights=w, tp_rank=rank, tp_size=2, comm=comm,
                      peer=peer, fused_layers=fused)
        m.prefill(prompt)
        logits = torch.zeros(B * T, oshape.vocab, dtype=torch.bfloat16, device=dev)
        am = torch.zeros(B * T, dtype=torch.int64, device=dev)
        m.forward_plan(step.to(dev), 1, B, T, m.lengths, 0, am, 1, logits_out=logits).run()
        torch.cuda.synchronize()
        out = {"logits": logits.cpu(), "am": am.cpu()}
        # greedy spec (target TP=2, draft replicated) vs greedy autoregressive (TP=2), CUDA graphs on
        wt = oq.random_qwen_weights(oshape, seed=3, std=0.08)
        wd = {**wt, "layers": wt["layers"][:1]}
        dshape = QwenShape(**{**SMALL, "n_layers": 1})
        K = 4
        tgt = QwenModel(shape, B, 128, B * (K + 1), device=dev, weights=wt, tp_rank=rank, tp_size=2, comm=comm,
                        peer=peer, fused_layers=fused)
        drf = QwenModel(dshape, B, 128, B * 2, device=dev, weights=wd, tp_size=2, tp_layers=False, tp_vocab=False)
        spec, _ = SpecEngine(tgt, drf, K).generate(prompt, 16)
        # the chain draft tensor-parallel over the same ranks (and peer group)
        tgt4 = QwenModel(shape, B, 128, B * (K + 1), device=dev, weights=wt, tp_rank=rank, tp_size=2,
                         comm=comm, peer=peer, fused_layers=fused)
        drf4 = QwenModel(dshape, B, 128, B * 2, device=dev, weights=wd, tp_rank=rank, tp_size=2, comm=comm,
                         peer=peer, fused_layers=fused)
        spec4, _ = SpecEngine(tgt4, drf4, K).generate(prompt, 16)
        out.update(spec_draft_tp=spec4)
        tgt2 = QwenModel(shape, B, 128, B, device=dev, weights=wt, tp_rank=rank, tp_size=2, comm=comm,
                         peer=peer, fused_layers=fused)
        ar = AutoregressiveEngine(tgt2).generate(prompt, 16)
        out.update(spec=spec, ar=ar)
        # EAGLE tree, greedy: the head replicated, the target TP=2
        from oracle import eagle as oe
        from tri_sds_b200.eagle import EagleEngine, EagleHead
        we = oe.random_eagle_weights(oshape, seed=4, std=0.08)
        tgt3 = QwenModel(shape, B, 128, B * 26, device=dev, weights=wt, tp_rank=rank, tp_size=2, comm=comm,
                         peer=peer, fused_layers=fused)
        eng = EagleEngine(tgt3, EagleHead(tgt3, B, weights=we), greedy=True)
        espec, _ = eng.generate(prompt, 16)
        out.update(espec=espec)
        # a CUDA graph holding NCCL calls must be gone before the process group
        eng.graph = None
        del eng
        torch.cuda.synchronize()
        for mdl in (m, tgt, tgt2, tgt3):
            mdl.check_status()
        if peer is not None:
            # the op-level all-reduce on a group of its own: x = 1 + (1 + 2) on both ranks
            import tri_sds_b200.torch_ops  # noqa: F401
            from tri_sds_b200.tp import register_peer_group
            op_peer = PeerAllReduce(rank, 2, 64 * 256)
            gid = register_peer_group(op_peer)
            xo = torch.ones(64, 256, dtype=torch.bfloat16, device=dev)
            for _ in range(3):   # both slots, then the first again
                xo.fill_(1.0)
                torch.ops.tsds.allreduce_oneshot(xo, torch.full((64, 256), float(rank + 1), device=dev), gid)
            torch.cuda.synchronize()
            out.update(op_allreduce=xo.cpu())
            dist.barrier()   # neither rank reads the other's buffers any more
            op_peer.close()
            peer.close()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("allreduce", ["nccl", "peer", "peer+fused"])
def test_tp2_verify_and_lossless_spec(allreduce):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(daemon=True, target=_worker, args=(r, port, q, allreduce)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=600) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():  # a rank stuck in teardown must not keep the session waiting
                p.terminate()
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
    # both ranks hold identical results
    assert torch.equal(res[0]["logits"], res[1]["logits"]) and torch.equal(res[0]["spec"], res[1]["spec"])
    oshape = oq.QwenShape(**SMALL)
    w = oq.random_qwen_weights(oshape, seed=1, std=0.02)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, oshape.vocab, (2, 12), generator=g)
    step = torch.randint(0, oshape.vocab, (2, 5), generator=g)
    ora = oq.QwenOracle(oshape, w, batch=2, max_seq=128)
    ora.forward(prompt)
    ora.lengths[:] = 12
    ref, _ = ora.forward(step)
    got = res[0]["logits"].float().reshape(2, 5, -1)
    assert (got - ref.float()).abs().max().item() <= 2e-2
    assert torch.equal(res[0]["am"], res[0]["logits"].float().argmax(-1))
    assert torch.equal(res[0]["spec"], res[0]["ar"])
    if "spec_draft_tp" in res[0]:
        assert torch.equal(res[0]["spec_draft_tp"], res[1]["spec_draft_tp"])
        assert torch.equal(res[0]["spec_draft_tp"], res[0]["ar"])
    assert torch.equal(res[0]["espec"], res[1]["espec"])
    assert torch.equal(res[0]["espec"], res[0]["ar"])
    if allreduce != "nccl":
        for r in (0, 1):
            assert torch.equal(res[r]["op_allreduce"], torch.full((64, 256), 4.0, dtype=torch.bfloat16))

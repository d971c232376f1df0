#!/usr/bin/env python
"""Benchmark: speculative decoding on a Qwen3-32B-shape target.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--mode eagle|chain]
                    [--impl tsds|reference]

One step = one speculative cycle over B sequences:

* ``--mode eagle`` (default): EAGLE draft head (fc 2x5120->5120 + one
  Qwen3-32B-shape decoder layer, the target's LM head), draft tree of depth
  5 with top-4 expansion pruned to 25 nodes, one target pass over the tree
  with the ancestor mask, rejection sampling at temperature 1 with seeded
  uniforms, KV compaction;
* ``--mode chain``: Qwen3-4B-shape draft model (36 layers), K=4 greedy
  chain, target verify over K+1 tokens, greedy acceptance.

Weights are random N(0, 0.02) (no checkpoints offline), prompts are 512
seeded uniform ids.  The metric is whole-job tokens/s (emitted tokens,
i.e. sum over sequences of accept_len + 1 per cycle).

N > 1 (torchrun): the target is tensor-parallel over the N GPUs (heads and
FFN sharded; after the O and down projections an all-reduce over NVLink peer
memory fused with the residual add, NCCL with ``--allreduce nccl``;
vocab-parallel LM head gathered over the same peer memory); the EAGLE head
is replicated, the chain draft model too unless
``--draft-tp`` shards it over the same ranks.  The ranks serve the
same B sequences, so the value is those tokens over the max-over-ranks time
(strong scaling).

``--impl reference`` times the reference's PyTorch algorithm on the host
CPU cores (the CPU oracle: a restatement of tri_sds/triton_kernels/
qwen_model.py), on a bounded sample of each cycle scaled to the full cycle.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="tsds", choices=["tsds", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--mode", default="eagle", choices=["eagle", "chain", "attention", "layer", "gemm"],
                    help="eagle / chain: the spec-decode cycle; attention: verify attention alone over a "
                         "--kv-len cache (B x (K+1) queries, 32B heads); layer: Qwen3-4B-shape decoder layers "
                         "alone over B x (K+1) rows; gemm: each projection of a layer alone over --rows rows, "
                         "back to back over several layers' weights")
    ap.add_argument("--rows", type=int, default=26, help="gemm mode: token rows M")
    ap.add_argument("--shape", default="32b", choices=["32b", "4b"], help="gemm mode: Qwen3-32B or -4B shape")
    ap.add_argument("--kv-len", type=int, default=4096, help="attention mode: keys per sequence")
    ap.add_argument("--greedy", action="store_true", help="eagle mode: greedy acceptance instead of sampling")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--sub-batch", type=int, default=8,
                    help="also measure this batch size over the same weights and report it as the line's "
                         "sub_batch record (0: off; skipped when equal to --batch)")
    # smaller depth for profiler captures only (never for reported numbers)
    ap.add_argument("--target-layers", type=int, default=None)
    ap.add_argument("--draft-layers", type=int, default=None)
    ap.add_argument("--fuse-norm", action="store_true",
                    help="the residual GEMMs also apply the RMSNorm that follows them "
                         "(tsds_linear_residual_norm; opt-in: measured slower, 59.0 vs 61.6 tok/s at B=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ctas-per-sm", type=int, default=None, help="tcgen05 GEMM CTAs per SM (library default 2)")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--dp-rows", type=int, default=None,
                    help="token rows from which a tcgen05 projection with at least one whole weight tile per CTA "
                         "runs data-parallel instead of stream-K (library default 128)")
    ap.add_argument("--dp-slack", type=int, default=None,
                    help="largest makespan increase (percent) the data-parallel schedule may cost over the ideal "
                         "(library default 100; it may leave CTAs idle for fewer tiles than CTAs)")
    ap.add_argument("--pair-rows", type=int, default=None,
                    help="token rows from which the tcgen05 GEMM runs on CTA pairs (library default 0: never)")
    ap.add_argument("--breakdown", type=int, default=0, metavar="CYCLES",
                    help="also time every library call of CYCLES eager cycles (CUDA events around each call) "
                         "and add the per-entry-point totals to the JSON line")
    ap.add_argument("--fused-layers", action="store_true",
                    help="one persistent launch per layer for O -> norm -> gate/up -> down -> norm -> q/k/v "
                         "(N > 1: with --allreduce peer, whose all-reduces become phases of it)")
    ap.add_argument("--draft-tp", action="store_true",
                    help="chain mode, N > 1: the draft model tensor-parallel over the target's ranks (its "
                         "all-reduces by --allreduce) instead of replicated")
    ap.add_argument("--allreduce", default="peer", choices=["nccl", "peer"],
                    help="N > 1: row-parallel all-reduce (and the vocab-parallel LM head's gathers) by the "
                         "library's peer-memory kernels (default: 78.9 vs 74.1 tok/s at TP=2, 97.7 vs 87.3 at "
                         "TP=4), or by NCCL")
    ap.add_argument("--attn-tc", type=int, nargs="?", const=1, default=0, choices=[0, 1, 2],
                    help="verify attention on its tcgen05 variant (1; 2: splits combined in a cluster; "
                         "library default 0: off)")
    ap.add_argument("--attn-split", type=int, default=None,
                    help="keys per attention split of the target / draft (a multiple of 64; of 128 for --attn-tc); "
                         "default 1024 (one split over the bench's 1024-row caches), 512 in --mode attention "
                         "(its 4096-key caches: four row groups share each K/V tile)")
    ap.add_argument("--gemv-splitk", action="store_true",
                    help="the GEMV path (rows up to --gemv-max-rows) as its split-K variant")
    ap.add_argument("--gemv-max-rows", type=int, default=None,
                    help="rows up to which the CUDA-core GEMV runs instead of tcgen05 (library default 0)")
    a = ap.parse_args()
    if a.attn_split is None:
        a.attn_split = 512 if a.mode == "attention" else 1024
    return a


METRIC = "Qwen3-32B spec-decode tok/s at B={B} ({n} GPU); verify-step us"
# samples of the CPU estimate in the device arm's cpu_baseline (the reference
# arm takes --steps of them, with the same median estimator)
CPU_REPS = 5
# (hidden, intermediate, rows) -> DRAM read + write bytes per launch of the
# target's gate/up GEMM at that shape, from an ncu capture of the kernel
# (dram__bytes_read.sum + dram__bytes_write.sum): 1.03x the algorithmic bytes
MEASURED_TRAFFIC = {(5120, 25600, 26): 540.4e6}
DATA = "synthetic: seeded uniform prompt ids, random-init N(0,0.02) weights (no checkpoint offline)"


def _workload(a) -> str:
    if a.mode == "attention":
        return (f"verify attention: B={a.batch} x {a.k + 1} queries x 64 q heads over {a.kv_len} cached keys x 8 kv "
                f"heads, head dim 128, causal among the new tokens")
    if a.mode == "layer":
        return f"Qwen3-4B-shape decoder layers (36) over B={a.batch} x {a.k + 1} rows at 512 cached tokens"
    if a.mode == "eagle":
        acc = "greedy" if a.greedy else "rejection sampling T=1.0"
        return (f"EAGLE tree spec decode: head fc 2x5120->5120 + 1 Qwen3-32B-shape layer, tree depth 5 / top-4 / "
                f"25 nodes, {acc}, Qwen3-32B-shape target (64L), prompt {a.prompt}, B={a.batch}")
    return (f"greedy chain spec decode: Qwen3-4B-shape draft (36L) -> Qwen3-32B-shape target (64L), "
            f"K={a.k}, prompt {a.prompt}, B={a.batch}")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's algorithm (oracle) on a bounded sample
# ---------------------------------------------------------------------------

class CpuCycle:
    """One full cycle on the host CPU, estimated from a bounded sample timed
    with the oracle: one layer of each model at the cycle's row counts plus
    the final norm + LM heads, scaled to the layer counts of the cycle.

    chain: 1 Qwen3-32B-shape layer verify (T=K+1) x64 + LM head, and
           1 Qwen3-4B-shape layer decode x36 x K + K LM heads;
    eagle: 1 Qwen3-32B-shape layer tree verify (T=26) x64 + LM head over 26
           rows, and 5 head passes (fc 2N->N, 1 target-shape layer, LM head)
           at T=1 then T=4."""

    def __init__(self, a):
        import torch
        from dataclasses import replace
        from oracle.qwen import QWEN3_32B, QWEN3_4B, QwenOracle, random_qwen_weights
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        B, K, P = a.batch, a.k, a.prompt
        self.a = a
        self.models = {}
        shapes = (("target", QWEN3_32B),) if a.mode == "eagle" else (("target", QWEN3_32B), ("draft", QWEN3_4B))
        for name, shape in shapes:
            one = replace(shape, n_layers=1)
            st = QwenOracle(one, random_qwen_weights(one, seed=1), batch=B, max_seq=P + 32)
            ids = torch.randint(0, shape.vocab, (B, P), generator=torch.Generator().manual_seed(2))
            with torch.no_grad():
                st.layer(0, st.embed_w[ids], torch.zeros(B, dtype=torch.int64), torch.arange(P), None)
            self.models[name] = (st, ids, shape.n_layers)
        if a.mode == "eagle":
            N = QWEN3_32B.hidden
            self.fc = (torch.randn(2 * N, N) * 0.02).to(torch.bfloat16)
            self.sample = (f"oracle bf16 on {self.threads} threads: 1 Qwen3-32B-shape layer tree verify (T=26) x64 "
                           f"+ LM head over 26 rows; 5 EAGLE head passes (fc + 1 layer + LM head, T=1 then 4); "
                           f"B={B}, cache {P}")
        else:
            self.sample = (f"oracle bf16 on {self.threads} threads: 1 Qwen3-32B-shape layer verify (T={K + 1}) x64 "
                           f"+ LM head; 1 Qwen3-4B-shape layer decode x36 x K={K} + {K} LM heads; B={B}, cache {P}")

    def _time(self, st, ids, T, P, B):
        import torch
        xs = st.embed_w[ids[:, :T]]
        starts = torch.full((B,), P, dtype=torch.int64)
        with torch.no_grad():
            t0 = time.perf_counter()
            st.layer(0, xs, starts, torch.arange(P, P + T), None)
            t_layer = time.perf_counter() - t0
            t0 = time.perf_counter()
            st.logits(xs)
            t_head = time.perf_counter() - t0
        return t_layer, t_head

    def sample_once(self) -> tuple:
        """Time one bounded sample; returns (projected full-cycle seconds,
        sample wall seconds).  The projection scales each timed layer by
        its model's layer count (and the draft by its K steps)."""
        import torch
        B, K, P = self.a.batch, self.a.k, self.a.prompt
        w0 = time.perf_counter()
        if self.a.mode == "eagle":
            st, ids, n_layers = self.models["target"]
            t_layer, t_head = self._time(st, ids, 26, P, B)
            total = t_layer * n_layers + t_head
            for T in (1, 4, 4, 4, 4):
                x2 = torch.cat([st.embed_w[ids[:, :T]], st.embed_w[ids[:, :T]]], -1)
                with torch.no_grad():
                    t0 = time.perf_counter()
                    x2 @ self.fc
                    t_fc = time.perf_counter() - t0
                h_layer, h_head = self._time(st, ids, T, P, B)
                total += t_fc + h_layer + h_head
            return total, time.perf_counter() - w0
        total = 0.0
        for name, (st, ids, n_layers) in self.models.items():
            T = K + 1 if name == "target" else 1
            t_layer, t_head = self._time(st, ids, T, P, B)
            total += t_layer * n_layers + t_head if name == "target" else (t_layer * n_layers + t_head) * K
        return total, time.perf_counter() - w0

    def estimate(self, reps: int, warm: int = 1) -> tuple:
        """Median projected cycle seconds and median sample wall seconds over
        `reps` samples after `warm` untimed ones: the same estimator for the
        device arm's cpu_baseline and the reference arm."""
        for _ in range(warm):
            self.sample_once()
        runs = [self.sample_once() for _ in range(max(1, reps))]
        return statistics.median(r[0] for r in runs), statistics.median(r[1] for r in runs)

    def scale(self) -> dict:
        if self.a.mode == "eagle":
            return {"target_layers_per_timed_layer": self.models["target"][2], "head_passes": 5}
        return {"target_layers_per_timed_layer": self.models["target"][2],
                "draft_layers_per_timed_layer": self.models["draft"][2], "draft_steps": self.a.k}


# ---------------------------------------------------------------------------

def run_reference(a, rank: int, world: int):
    """--impl reference: the reference's CPU path (oracle port), rank 0 only."""
    if rank != 0:
        return
    if a.mode in ("attention", "layer", "gemm"):
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the spec-decode cycle "
                                                              "(--mode eagle / chain)"}), flush=True)
        return
    cc = CpuCycle(a)
    threads, sample = cc.threads, cc.sample
    # one step = one bounded sample (one layer of each model, the LM heads,
    # the head passes); the cycle is projected from it by the layer counts
    cyc, sample_s = cc.estimate(a.steps, warm=a.warmup)
    # tokens per cycle: one per sequence (the bonus) plus accepted drafts; with
    # independent random-init models the acceptance is ~0 (measured on the device arm)
    tok_s = a.batch / cyc
    line = {"impl": "reference", "metric": METRIC.format(B=a.batch, n=world), "value": tok_s, "unit": "tok/s",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": sample_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": DATA,
            "config": {"workload": _workload(a), "global_batch": a.batch, "seq_len": a.prompt,
                       "parallelism": "cpu"},
            "projection": {"sample_ms": sample_s * 1e3, "projected_cycle_ms": cyc * 1e3, "scale": cc.scale(),
                           "estimator": f"median of {a.steps} samples after {a.warmup} untimed"},
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def plan_breakdown(plan, cycles: int) -> dict:
    """Device time of every call of a launch plan over `cycles` eager runs,
    with CUDA events around each call (so neighbouring kernels cannot overlap
    as they do under programmatic dependent launch in the graph: the sum
    exceeds the cycle time).  Returns {"calls": [{"call", "per_cycle",
    "us_per_cycle", "share"}] sorted by time, "sum_us_per_cycle"}."""
    import ctypes

    import torch
    from tri_sds_b200 import _lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    marks = []
    for _ in range(cycles):
        for name, fn, args in plan.calls:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            if fn is None:
                args()
            else:
                st = fn(*args, s)
                if st != 0:
                    raise RuntimeError(f"{name} failed: {_lib.load().tsds_status_string(st).decode()}")
            e1.record()
            marks.append((name, e0, e1))
    torch.cuda.synchronize()
    tot, cnt = {}, {}
    for name, e0, e1 in marks:
        tot[name] = tot.get(name, 0.0) + e0.elapsed_time(e1) * 1e3 / cycles
        cnt[name] = cnt.get(name, 0) + 1
    total = sum(tot.values())
    rows = [{"call": n, "per_cycle": cnt[n] // cycles, "us_per_cycle": round(tot[n], 1),
             "share": round(tot[n] / total, 4)} for n in sorted(tot, key=tot.get, reverse=True)]
    return {"calls": rows, "sum_us_per_cycle": round(total, 1)}


def _graph_time_us(run_once, reps: int, warm: int = 3):
    """Capture run_once() in a CUDA graph, replay it `warm` times, then time
    `reps` replays with CUDA events; returns (us per replay, clocks)."""
    import torch
    run_once()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run_once()
    for _ in range(warm):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / reps, clocks.summary()


def run_attention(a):
    """--mode attention: tsds_verify_attention alone at the verify-attention
    configuration (q [B, K+1, 64, 128], K/V caches [B, 8, kv_len, 128], the new
    tokens the last K+1 rows, causal among them).  Enough cache sets rotate
    that the timed launches read more than twice the L2 size, so every
    launch streams its K/V from HBM."""
    import torch
    from tri_sds_b200 import _lib, ops
    dev = torch.device("cuda", 0)
    B, T, L, Hq, Hkv, D = a.batch, a.k + 1, a.kv_len, 64, 8, 128
    kv_bytes = B * Hkv * L * D * 2 * 2
    sets = max(1, -(-(2 * 126 * 2 ** 20) // kv_bytes))
    g = torch.Generator(device=dev).manual_seed(11)
    caches = [(torch.randn(B, Hkv, L, D, device=dev, generator=g).to(torch.bfloat16),
               torch.randn(B, Hkv, L, D, device=dev, generator=g).to(torch.bfloat16)) for _ in range(sets)]
    q = torch.randn(B, T, Hq, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    starts = torch.full((B,), L - T, dtype=torch.int32, device=dev)
    lc0 = _lib.query("tsds_launch_count")

    def once():
        for k, v in caches:
            ops.verify_attention(q, k, v, starts, out=out, split_keys=a.attn_split)

    us, clocks = _graph_time_us(once, reps=max(1, a.steps))
    launches = (_lib.query("tsds_launch_count") - lc0) // 2   # eager warm-up + capture
    us_launch = us / sets
    nbytes = kv_bytes + 2 * B * T * Hq * D * 2
    peak, peak_kind = _peaks()
    achieved = nbytes / (us_launch * 1e-6) / 1e9
    line = {"metric": "verify attention GB/s", "value": achieved, "unit": "GB/s", "n_gpus": 1, "steps": a.steps,
            "warmup": 3, "ms_per_step": us_launch / 1e3, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: N(0,1) q / K / V",
            "config": {"workload": _workload(a), "global_batch": B, "seq_len": L, "parallelism": "none",
                       "l2": f"{sets} cache sets rotate ({sets * kv_bytes / 2**20:.0f} MB > 2 x L2)",
                       "attention": {"tcgen05": _lib.query("tsds_get_attention_tc"),
                                     "split_keys": a.attn_split}},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": None, "bytes_per_launch": nbytes,
                         "launch_us": us_launch},
            "clocks": clocks, "gpu_launches": launches * max(1, a.steps)}
    print(json.dumps(line), flush=True)


def run_layer(a):
    """--mode layer: the decoder layers of a Qwen3-4B-shape model (36, random
    weights) over B x (K+1) rows at 512 cached tokens per sequence - the
    decode-layer primitives' configuration - as one graph; reports the time
    per layer against its weight bytes."""
    import torch
    from tri_sds_b200 import _lib
    from tri_sds_b200.model import Plan, QwenModel, _p
    from tri_sds_b200.shapes import QWEN3_4B
    dev = torch.device("cuda", 0)
    B, T = a.batch, a.k + 1
    m = QwenModel(QWEN3_4B, B, 1024, B * T, device=dev, seed=5, fused_layers=a.fused_layers, split_keys=a.attn_split)
    m.fuse_norm = a.fuse_norm
    m.lengths.fill_(512)
    m.x[:B * T].copy_(torch.randn(B * T, QWEN3_4B.hidden, device=dev).to(torch.bfloat16))
    pl = Plan()
    pl.add("tsds_prep_chain", _p(m.lengths), 0, B, T, _p(m.starts), _p(m.positions))
    pl.extend(m.layers_plan(B, T))
    lc0 = _lib.query("tsds_launch_count")
    us, clocks = _graph_time_us(pl.run, reps=max(1, a.steps))
    launches = (_lib.query("tsds_launch_count") - lc0) // 2
    m.check_status()
    L0 = m.layers[0]
    wbytes = sum(t.numel() * 2 for t in (L0.w_qkv, L0.w_o, L0.w_gu, L0.w_d))
    us_layer = us / QWEN3_4B.n_layers
    peak, peak_kind = _peaks()
    achieved = wbytes / (us_layer * 1e-6) / 1e9
    line = {"metric": "decode layer us", "value": us_layer, "unit": "us", "n_gpus": 1, "steps": a.steps,
            "warmup": 3, "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "none",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: random-init N(0,0.02) weights",
            "config": {"workload": _workload(a), "global_batch": B, "seq_len": 512, "rows": B * T,
                       "parallelism": "none", "fused_layers": bool(m.fused_layers),
                       "l2": "no flush: 7.3 GB of weights per pass >> 126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": None, "bytes_per_launch": wbytes,
                         "launch_us": us_layer},
            "clocks": clocks, "gpu_launches": launches * max(1, a.steps)}
    print(json.dumps(line), flush=True)


def run_gemm(a):
    """--mode gemm: every projection of one decoder layer (q/k/v, O + residual,
    gate/up + SwiGLU, down + residual) alone at M = --rows token rows, each
    timed with CUDA events over back-to-back launches across the weights of
    enough layers to exceed L2 several times (so every launch streams its
    weights from HBM).  One JSON line: per projection the µs per launch and
    its algorithmic bytes against the measured HBM peak, and the layer's sum.
    The library's tuning switches (GEMV rows / split-K, CTA pairs,
    data-parallel rows and slack) apply as set on the command line."""
    import torch
    from tri_sds_b200 import _lib, ops
    from tri_sds_b200.shapes import QWEN3_4B, QWEN3_32B
    dev = torch.device("cuda", 0)
    sh = QWEN3_32B if a.shape == "32b" else QWEN3_4B
    M, N, I = a.rows, sh.hidden, sh.intermediate
    qd, kvd = sh.n_heads * sh.head_dim, sh.n_kv_heads * sh.head_dim
    per_layer = 2 * N * (qd + 2 * kvd + qd + 2 * I + I)
    nl = max(4, -(-(4 * 126 * 2 ** 20) // per_layer))   # > 4 x L2 of weights
    g = torch.Generator(device=dev).manual_seed(3)

    def w(rows, cols):
        return (0.02 * torch.randn(rows, cols, device=dev, generator=g)).to(torch.bfloat16)
    layers = [dict(qkv=w(qd + 2 * kvd, N), o=w(N, qd), gu=w(2 * I, N), d=w(N, I)) for _ in range(nl)]
    x_n = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    x_q = torch.randn(M, qd, device=dev, generator=g).to(torch.bfloat16)
    x_i = torch.randn(M, I, device=dev, generator=g).to(torch.bfloat16)
    res = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    o_qkv = torch.empty(M, qd + 2 * kvd, dtype=torch.bfloat16, device=dev)
    o_n = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    o_i = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
    projs = {
        "qkv": (lambda L: ops.linear(x_n, L["qkv"], out=o_qkv), (qd + 2 * kvd) * N, N, qd + 2 * kvd),
        "o": (lambda L: ops.linear_residual(x_q, L["o"], res, out=o_n), N * qd, qd, N),
        "gate_up": (lambda L: ops.linear_swiglu(x_n, L["gu"], out=o_i), 2 * I * N, N, I),
        "down": (lambda L: ops.linear_residual(x_i, L["d"], res, out=o_n), N * I, I, N),
    }
    peak, peak_kind = _peaks()
    reps = max(1, a.steps)
    lc0 = _lib.query("tsds_launch_count")
    out, tot_b, tot_us = {}, 0, 0.0
    for name, (fn, wel, kin, kout) in projs.items():
        # one pass over the layers' weights as a CUDA graph (host launch cost
        # out of the timing, launches back to back as in the cycle's graph)
        def one_pass(fn=fn):
            for L in layers:
                fn(L)
        us_pass, _ = _graph_time_us(one_pass, reps=reps)
        us = us_pass / nl
        nbytes = 2 * wel + 2 * M * (kin + kout) + (2 * M * kout if name in ("o", "down") else 0)
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us": round(us, 2), "bytes": nbytes, "gb_s": round(gbs, 1), "frac": round(gbs / peak, 3)}
        tot_b += nbytes
        tot_us += us
    launches = (_lib.query("tsds_launch_count") - lc0) // 2 * reps   # eager warm-up + capture, then replays
    layer_gbs = tot_b / (tot_us * 1e-6) / 1e9
    lib = _lib.load()
    line = {"metric": "decode-layer projections GB/s", "value": layer_gbs, "unit": "GB/s", "n_gpus": 1,
            "steps": reps, "warmup": 3, "ms_per_step": tot_us / 1e3, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: random N(0,0.02) weights, N(0,1) activations",
            "config": {"workload": f"Qwen3-{a.shape.upper()}-shape projections of one layer at M={M} rows",
                       "rows": M, "layers_rotated": nl,
                       "l2": f"no flush: {nl} layers' weights ({nl * per_layer / 2**30:.1f} GiB) rotate, > 4 x L2",
                       "gemv_max_rows": lib.tsds_get_gemv_max_rows(), "gemv_splitk": lib.tsds_get_gemv_splitk(),
                       "gemm_pair_rows": lib.tsds_get_gemm_pair_rows(), "gemm_dp_rows": lib.tsds_get_gemm_dp_rows(),
                       "gemm_dp_slack": lib.tsds_get_gemm_dp_slack()},
            "projections": out,
            "roofline": {"bound": "hbm", "achieved": layer_gbs, "peak": peak, "unit": "GB/s",
                         "frac": layer_gbs / peak, "peak_kind": peak_kind, "traffic": None,
                         "bytes_per_launch": tot_b, "launch_us": tot_us},
            "gpu_launches": launches}
    print(json.dumps(line), flush=True)


def _build_engine(a, B, tshape, dshape, dev, rank, world, comm, peer, share=None):
    """Target (+ EAGLE head or draft model) and engine for B sequences;
    `share` = an earlier (target, head_or_draft) whose weights to reuse."""
    from tri_sds_b200.engine import SpecEngine
    from tri_sds_b200.model import QwenModel
    K, P = a.k, a.prompt
    per_cycle = 7 if a.mode == "eagle" else K + 1        # most tokens a cycle can commit
    rows_verify = B * 26 if a.mode == "eagle" else B * (K + 1)
    max_seq = P + (3 * a.warmup + 2 * a.steps + a.breakdown) * per_cycle + 64 + 32
    max_seq = (max_seq + 63) // 64 * 64
    target = QwenModel(tshape, B, max_seq, max_rows=rows_verify, device=dev, seed=1000, tp_rank=rank,
                       tp_size=world, comm=comm, peer=peer, fused_layers=a.fused_layers, split_keys=a.attn_split,
                       share_weights=None if share is None else share[0])
    target.fuse_norm = a.fuse_norm
    if a.mode == "eagle":
        from tri_sds_b200.eagle import EagleEngine, EagleHead
        head = EagleHead(target, B, seed=2000, share=None if share is None else share[1])
        head.model.fuse_norm = a.fuse_norm
        return target, head, EagleEngine(target, head, greedy=a.greedy, seed=3000), rows_verify
    if a.draft_tp and world > 1:
        # sharded like the target over the same ranks (and peer group)
        draft = QwenModel(dshape, B, max_seq, max_rows=B * 2, device=dev, seed=2000, tp_rank=rank,
                          tp_size=world, comm=comm, peer=peer, fused_layers=a.fused_layers,
                          split_keys=a.attn_split, share_weights=None if share is None else share[1])
    else:
        draft = QwenModel(dshape, B, max_seq, max_rows=B * 2, device=dev, seed=2000, tp_size=world,
                          tp_layers=False, tp_vocab=False, fused_layers=a.fused_layers, split_keys=a.attn_split,
                          share_weights=None if share is None else share[1])
    draft.fuse_norm = a.fuse_norm
    return target, draft, SpecEngine(target, draft, K), rows_verify


def _measure_engine(a, B, engine, target, other, rank, world, local_rank, dev, tshape, e2e_steps):
    """Device-timed cycles (inputs resident), the verify step alone and the
    end-to-end worker path with host buffers, for one engine.  Returns a dict
    (every rank takes the same collective steps)."""
    import torch
    import torch.distributed as dist
    from tri_sds_b200 import _lib
    from tri_sds_b200.sglang_compat import ScheduleBatch
    from tri_sds_b200.worker import TriSDSWorker

    def barrier():
        if world > 1:
            dist.barrier()

    prompt = torch.randint(0, tshape.vocab, (B, a.prompt), generator=torch.Generator().manual_seed(7))
    engine.prepare(prompt)
    hist = torch.zeros(a.warmup + a.steps, B, dtype=torch.int32, device=dev)
    for i in range(a.warmup):
        engine.step()
        hist[i].copy_(engine.accept_len)
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.nvtx.range_push("tsds_timed")
        ev0.record()
        for i in range(a.steps):
            engine.step()
            hist[a.warmup + i].copy_(engine.accept_len)
        ev1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier()
    ms = ev0.elapsed_time(ev1)
    # a device wait that gave up (status word set) invalidates the run: fail loudly
    for mdl in (target, other.model if a.mode == "eagle" else other):
        mdl.check_status()
    acc = hist[a.warmup:].float().cpu()
    tokens = float((acc + 1).sum())
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t[0])
    out = {"value": tokens / (ms_max / 1e3), "ms_per_step": ms_max / a.steps, "tokens": tokens,
           "accept_len_mean": float(acc.mean()), "clocks": clocks.summary(),
           "gpu_launches": engine.plan_launches * a.steps}

    # ---- verify step alone (target forward over the verify rows) -----------
    vplan = engine.verify_only_plan()
    vplan.run()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        vplan.run()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    nv = 10
    for _ in range(nv):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    vt = torch.tensor([e0.elapsed_time(e1) * 1e3 / nv], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vt, op=dist.ReduceOp.MAX)
    out["verify_step_us"] = float(vt[0])
    del g

    # ---- end to end through the worker API (host buffers) ------------------
    if e2e_steps > 0:
        os.environ["SDS_ENABLED"] = "1"
        worker = TriSDSWorker()
        worker.attach_engine(engine)
        worker._prefilled = True  # the engine is prepared; continue from its state
        cur_host = engine.cur.cpu().reshape(B, 1)
        for _ in range(a.warmup):
            toks, n = worker.forward_batch_generation(ScheduleBatch(input_ids=cur_host))
            cur_host = toks.gather(1, n.long().unsqueeze(1))
        barrier()
        t0 = time.perf_counter()
        e_tokens = 0
        for _ in range(e2e_steps):
            toks, n = worker.forward_batch_generation(ScheduleBatch(input_ids=cur_host))
            cur_host = toks.gather(1, n.long().unsqueeze(1))
            e_tokens += int(n.sum()) + B
        el = time.perf_counter() - t0
        tt = torch.tensor([el], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            el = float(tt[0])
        out["e2e"] = {"value": e_tokens / el, "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
                      "d2h_bytes_per_step": engine.tokens.numel() * 8 + 4 * B}
    return out


def _cycle_bytes(a, tshape, B, world, target) -> float:
    """Algorithmic HBM bytes of one cycle on one rank: every weight the cycle
    streams once (target layers + LM head, and the EAGLE head's fc + layer +
    LM head per pass, or the draft model's K steps) plus the verify's K/V
    reads at the prompt length."""
    L0 = target.layers[0]
    layer_b = sum(t.numel() * 2 for t in (L0.w_qkv, L0.w_o, L0.w_gu, L0.w_d))
    lm_b = target.lm_head_w.numel() * 2
    kv_row = 2 * target.k_cache.shape[2] * tshape.head_dim * 2   # K + V of one token, one layer, this rank
    verify = tshape.n_layers * (layer_b + B * a.prompt * kv_row) + lm_b
    if a.mode == "eagle":
        fc_b = 2 * tshape.hidden * tshape.hidden * 2
        return verify + 5 * (fc_b + layer_b + lm_b)
    return verify


def run_tsds(a, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    from dataclasses import replace
    from tri_sds_b200 import _lib
    from tri_sds_b200.shapes import QWEN3_32B, QWEN3_4B

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B = a.batch
    if a.gemv_max_rows is not None:
        _lib.load().tsds_set_gemv_max_rows(a.gemv_max_rows)
    if a.gemv_splitk:
        _lib.load().tsds_set_gemv_splitk(1)
    if a.ctas_per_sm is not None:
        _lib.load().tsds_set_gemm_ctas_per_sm(a.ctas_per_sm)
    if a.no_pdl:
        _lib.load().tsds_set_pdl(0)
    if a.pair_rows is not None:
        _lib.load().tsds_set_gemm_pair_rows(a.pair_rows)
    if a.dp_rows is not None:
        _lib.load().tsds_set_gemm_dp_rows(a.dp_rows)
    if a.dp_slack is not None:
        _lib.load().tsds_set_gemm_dp_slack(a.dp_slack)
    if a.attn_tc:
        _lib.load().tsds_set_attention_tc(a.attn_tc)
    tshape = QWEN3_32B if a.target_layers is None else replace(QWEN3_32B, n_layers=a.target_layers)
    dshape = QWEN3_4B if a.draft_layers is None else replace(QWEN3_4B, n_layers=a.draft_layers)
    sub_B = a.sub_batch if (a.sub_batch and a.sub_batch != B) else 0
    rows_max = max(B, sub_B) * (26 if a.mode == "eagle" else a.k + 1)
    # N > 1: the target is tensor-parallel over all ranks (shards drawn per
    # rank; replicated tensors from the same seed on every rank)
    comm = peer = None
    if world > 1:
        from tri_sds_b200.tp import Comm, PeerAllReduce
        comm = Comm()
        if a.allreduce == "peer":
            # with an exchange region for the vocab-parallel LM head's gathers
            from tri_sds_b200.tp import lm_exchange_layout
            peer = PeerAllReduce(rank, world, rows_max * tshape.hidden,
                                 exchange_bytes=lm_exchange_layout(rows_max, tshape.vocab // world)[2])
    target, other, engine, rows_verify = _build_engine(a, B, tshape, dshape, dev, rank, world, comm, peer)
    res = _measure_engine(a, B, engine, target, other, rank, world, local_rank, dev, tshape,
                          0 if a.no_e2e else a.steps)
    breakdown = plan_breakdown(engine.plan, a.breakdown) if a.breakdown > 0 else None
    peak, peak_kind = _peaks()
    cycle_b = _cycle_bytes(a, tshape, B, world, target)

    # ---- dominant kernel: the target's gate/up + SiLU projection -------------
    from tri_sds_b200 import ops
    M = rows_verify
    xin = torch.randn(M, tshape.hidden, device=dev).to(torch.bfloat16)
    hout = torch.empty(M, target.lshape.intermediate, dtype=torch.bfloat16, device=dev)
    for L in target.layers[:2]:
        ops.linear_swiglu(xin, L.w_gu, out=hout)
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for L in target.layers:
        ops.linear_swiglu(xin, L.w_gu, out=hout)
    k1.record()
    torch.cuda.synchronize()
    kern_us = k0.elapsed_time(k1) * 1e3 / len(target.layers)
    kbytes = target.layers[0].w_gu.numel() * 2 + xin.numel() * 2 + hout.numel() * 2
    achieved = kbytes / (kern_us * 1e-6) / 1e9
    # DRAM read + write bytes per launch of this kernel at this shape from an
    # ncu capture of it (None where none was taken): the traffic-to-algorithmic
    # ratio, not a number of this run
    traffic = MEASURED_TRAFFIC.get((tshape.hidden, tshape.intermediate, M)) if world == 1 else None

    # ---- the projection furthest from the roofline: the target's q/k/v -------
    # (the smallest weight matrix of a layer, where the GEMM's fixed cost per
    # launch weighs most), timed the same way as one CUDA graph over the layers
    qout = torch.empty(M, target.lshape.qkv_dim, dtype=torch.bfloat16, device=dev)

    def qkv_pass():
        for L in target.layers:
            ops.linear(xin, L.w_qkv, out=qout)
    q_us = _graph_time_us(qkv_pass, reps=3)[0] / len(target.layers)
    q_bytes = target.layers[0].w_qkv.numel() * 2 + xin.numel() * 2 + qout.numel() * 2
    q_ach = q_bytes / (q_us * 1e-6) / 1e9

    # ---- a second batch size over the same weights ---------------------------
    sub = None
    if sub_B:
        engine.graph = None
        t2, o2, eng2, _ = _build_engine(a, sub_B, tshape, dshape, dev, rank, world, comm, peer,
                                        share=(target, other))
        r2 = _measure_engine(a, sub_B, eng2, t2, o2, rank, world, local_rank, dev, tshape,
                             0 if a.no_e2e else a.steps)
        cb2 = _cycle_bytes(a, tshape, sub_B, world, t2)
        sub = {"global_batch": sub_B, "value": r2["value"], "unit": "tok/s", "ms_per_step": r2["ms_per_step"],
               "verify_step_us": r2["verify_step_us"], "accept_len_mean": r2["accept_len_mean"],
               "e2e": r2.get("e2e"), "gpu_launches": r2["gpu_launches"], "clocks": r2["clocks"],
               "cycle_hbm_frac": cb2 / (r2["ms_per_step"] * 1e-3) / 1e9 / peak}
        eng2.graph = None
        torch.cuda.synchronize()

    # ---- CPU baseline (rank 0, N=1) ------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cc = CpuCycle(a)
        cyc, sample_s = cc.estimate(CPU_REPS, warm=1)
        mean_tok = res["tokens"] / a.steps
        cpu = {"value": mean_tok / cyc, "unit": "tok/s", "cores": cc.threads, "kind": "port",
               "sample": cc.sample + f"; {mean_tok:.2f} tokens per cycle as measured on the device",
               "sample_ms": sample_s * 1e3, "projected_cycle_ms": cyc * 1e3, "scale": cc.scale(),
               "estimator": f"median of {CPU_REPS} samples after 1 untimed"}

    if rank == 0:
        line = {
            "metric": METRIC.format(B=B, n=world), "value": res["value"], "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": DATA,
            "config": {"workload": _workload(a), "global_batch": B, "seq_len": a.prompt,
                       "parallelism": f"tp{world}", "allreduce": a.allreduce if world > 1 else None,
                       "draft_parallelism": (None if a.mode == "eagle" else
                                             f"tp{world}" if a.draft_tp and world > 1 else "replicated"),
                       "fused_layers": bool(target.fused_layers),
                       "l2": "no flush: 73 GB of weights per cycle >> 126 MB L2",
                       "mode": a.mode, "target_layers": tshape.n_layers,
                       "draft_layers": 0 if a.mode == "eagle" else dshape.n_layers},
            "verify_step_us": res["verify_step_us"],
            "accept_len_mean": res["accept_len_mean"],
            "roofline": {"bound": "hbm", "kernel": "tsds_linear_swiglu (target gate/up, M=%d)" % M,
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic, "traffic_source": "ncu capture, not this run",
                         "bytes_per_launch": kbytes, "launch_us": kern_us,
                         "lowest_gemm": {"kernel": "tsds_linear (target q/k/v, M=%d)" % M, "launch_us": q_us,
                                         "bytes_per_launch": q_bytes, "achieved": q_ach, "frac": q_ach / peak},
                         "cycle": {"bytes_per_cycle": cycle_b,
                                   "achieved": cycle_b / (res["ms_per_step"] * 1e-3) / 1e9,
                                   "frac": cycle_b / (res["ms_per_step"] * 1e-3) / 1e9 / peak}},
            "cpu_baseline": cpu,
            "e2e": res.get("e2e"),
            "clocks": res["clocks"],
            "gpu_launches": res["gpu_launches"],
            "gemv_max_rows": _lib.load().tsds_get_gemv_max_rows(),
            "gemv_splitk": _lib.load().tsds_get_gemv_splitk(),
            "gemm_pair_rows": _lib.load().tsds_get_gemm_pair_rows(),
            "gemm_dp_rows": _lib.load().tsds_get_gemm_dp_rows(),
            "gemm_dp_slack": _lib.load().tsds_get_gemm_dp_slack(),
            "attention": {"tcgen05": _lib.load().tsds_get_attention_tc(), "split_keys": a.attn_split},
        }
        if sub is not None:
            line["sub_batch"] = sub
        if breakdown is not None:
            line["breakdown"] = breakdown
        print(json.dumps(line), flush=True)
    # CUDA graphs that hold NCCL calls go before the process group does
    engine.graph = None
    torch.cuda.synchronize()
    if peer is not None:
        if world > 1:
            dist.barrier()   # no rank reads a peer buffer any more
        peer.close()


def main():
    a = _args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if a.impl == "tsds" else "gloo"
        if backend == "nccl":
            import torch
            torch.cuda.set_device(local_rank)
            # the all-reduces here are small (<= 0.5 MB); NVLink SHARP buys nothing
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        # a short limit: a rank stuck in a collective fails instead of waiting
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    try:
        if a.impl == "reference":
            run_reference(a, rank, world)
        elif a.mode in ("attention", "layer", "gemm"):
            if world > 1:
                raise SystemExit("--mode attention / layer / gemm run on one GPU")
            from tri_sds_b200 import _lib
            if a.ctas_per_sm is not None:
                _lib.load().tsds_set_gemm_ctas_per_sm(a.ctas_per_sm)
            if a.no_pdl:
                _lib.load().tsds_set_pdl(0)
            if a.pair_rows is not None:
                _lib.load().tsds_set_gemm_pair_rows(a.pair_rows)
            if a.dp_rows is not None:
                _lib.load().tsds_set_gemm_dp_rows(a.dp_rows)
            if a.dp_slack is not None:
                _lib.load().tsds_set_gemm_dp_slack(a.dp_slack)
            if a.attn_tc:
                _lib.load().tsds_set_attention_tc(a.attn_tc)
            if a.gemv_max_rows is not None:
                _lib.load().tsds_set_gemv_max_rows(a.gemv_max_rows)
            if a.gemv_splitk:
                _lib.load().tsds_set_gemv_splitk(1)
            {"attention": run_attention, "layer": run_layer, "gemm": run_gemm}[a.mode](a)
        else:
            run_tsds(a, rank, world, local_rank)
    except BaseException:
        # a failed rank leaves without destroy_process_group: the CUDA graphs
        # that hold NCCL calls may still be alive in the traceback, and the
        # teardown would wait on them for good
        import traceback
        traceback.print_exc()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(1)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

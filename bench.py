#!/usr/bin/env python
"""Decode-step benchmark: ragged paged MLA decode (config 2) on N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hk|reference]

A step is one pass of the hot path over the configuration-2 batch: pack the 64 ragged lanes
into one token stream, append each lane's new latent row into the paged cache, then ragged
paged MLA attention (128 heads, 512 latent + 64 rope, bf16, page 64, contexts log-uniform in
[1K, 128K]) with split-KV partials merged by LSE.  Lanes are independent, so N GPUs run N
independent 64-lane batches (weak scaling, no data-path collective); `value` is the tokens
of all ranks over the slowest rank's device time.

The KV cache (~2 GB per rank) is far larger than the 126 MB L2, so steps read it from HBM
without an explicit flush.  Inputs are synthetic (seeded), see hyperkernel_b200/workload.py.

--impl reference times the CPU restatement of the same step (oracle/, the reference has no
runnable implementation of this path on this box) on all host cores, on a bounded sample of
lanes per step scaled to the whole batch.

--workload moe | linear measures the other two layers of the step on one GPU, each as its own
JSON line: config 4 (MoE layer: quantise, route, permute, grouped FP8 expert FFN over 256
routed experts + the shared expert, combine; 512 tokens, hidden 7168, inter 2048) and config 3
(the MLA FP8 projections q_a, q_b, kv_a, o over the 4144-token mixed prefill + decode batch).
--workload longctx measures config 5 (one lane at 1M cached rows plus 7 shorter ones, 1 + 4
spec-verify rows each, FP8 latent cache); on N GPUs the long lane's KV is split by position
(context parallel) and the partials merged by LSE.  --workload sample measures spec-decode
verification with on-device sampling at config 5's shape (8 lanes x 5 rows of logits over a
129,280-token vocabulary).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HEADS = 128
PAGE = 64
TRAFFIC_PER_ALGORITHMIC_BYTE = 1.044
DK, DV = 576, 512


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def attn_bytes(kv_len: np.ndarray, tokens: int, heads: int = HEADS) -> int:
    """Algorithmic HBM bytes of one attention launch: every cached latent row read once
    (576 bf16, shared by all heads), queries read, outputs and LSE written."""
    return int(kv_len.sum()) * DK * 2 + tokens * heads * (DK * 2 + DV * 2 + 4)


def attn_flops(kv_len: np.ndarray, heads: int = HEADS) -> int:
    return int(2 * heads * (DK + DV) * int(kv_len.sum()))


def cpu_sample_layout(lay, target_rows: int):
    """The first lanes of the workload whose rows sum to about target_rows (at least one)."""
    from hyperkernel_b200 import workload as W

    ctx, rows = [], 0
    for c in lay.context:
        if ctx and rows + c + 1 > target_rows:
            break
        ctx.append(int(c))
        rows += int(c) + 1
    sub = W.paged_layout(W.Rng(99), np.array(ctx), np.ones(len(ctx), np.int64), PAGE)
    return sub, rows


def cpu_lanes_seconds(ctx, rows, fp8=False):
    """Times the CPU oracle (pack + append + attention) on lanes of cached lengths `ctx` with
    `rows` new rows each (bf16 or e4m3 latent cache); returns (seconds, query-KV pairs,
    threads)."""
    import oracle
    from hyperkernel_b200 import workload as W

    oracle.use_all_cores()
    sub = W.paged_layout(W.Rng(99), np.asarray(ctx, np.int64), np.asarray(rows, np.int64), PAGE)
    g = np.random.default_rng(7)
    T = sub.num_tokens
    q = g.integers(0, 1 << 16, size=(T, HEADS, DK), dtype=np.uint16) & np.uint16(0xBFFF)
    kv_new = g.integers(0, 1 << 16, size=(T, DK), dtype=np.uint16) & np.uint16(0xBFFF)
    if fp8:
        c8 = g.integers(0, 256, size=(sub.num_slots, DK), dtype=np.uint8)
        c8[(c8 & 0x7F) == 0x7F] ^= 1
        s8 = (g.random(sub.num_slots) * 0.01 + 0.001).astype(np.float32)
    else:
        cache = g.integers(0, 1 << 16, size=(sub.num_slots, DK), dtype=np.uint16) & np.uint16(0xBFFF)
    t0 = time.perf_counter()
    p = oracle.pack(sub.new_rows, sub.context, sub.block_table, PAGE, sub.num_pages, T)
    slots = p["slot_mapping"][:T]
    if fp8:
        oracle.kv_append_fp8(kv_new, slots, c8, s8)
        oracle.mla_decode(q, sub.block_table, p["cu_seqlens"], p["positions"][:T], PAGE, 1.0 / math.sqrt(DK),
                          kv_fp8=c8, kv_scale=s8)
    else:
        oracle.kv_append_bf16(kv_new, slots, cache)
        oracle.mla_decode(q, sub.block_table, p["cu_seqlens"], p["positions"][:T], PAGE, 1.0 / math.sqrt(DK),
                          kv_bf16=cache)
    dt = time.perf_counter() - t0
    pairs = int(sum(int(c) * int(r) + int(r) * (int(r) + 1) // 2 for c, r in zip(ctx, rows)))
    return dt, pairs, oracle.threads()


def _query_kv_pairs(lay):
    return int(sum(int(c) * int(r) + int(r) * (int(r) + 1) // 2 for c, r in zip(lay.context, lay.new_rows)))


def cpu_step_seconds(lay, target_rows: int, reps: int = 1):
    """Times the CPU oracle (pack + append + attention) on a sample; returns
    (seconds per full step extrapolated by KV rows, sample rows, sample lanes, threads).
    Used only to warm the host cores up before whole steps are timed."""
    import oracle

    oracle.use_all_cores()
    sub, rows = cpu_sample_layout(lay, target_rows)
    g = np.random.default_rng(7)
    T = sub.num_tokens
    q = g.integers(0, 1 << 16, size=(T, HEADS, DK), dtype=np.uint16) & np.uint16(0xBFFF)
    cache = (g.integers(0, 1 << 16, size=(sub.num_slots, DK), dtype=np.uint16) & np.uint16(0xBFFF))
    kv_new = g.integers(0, 1 << 16, size=(T, DK), dtype=np.uint16) & np.uint16(0xBFFF)
    best = math.inf
    for _ in range(reps):
        t0 = time.perf_counter()
        p = oracle.pack(sub.new_rows, sub.context, sub.block_table, PAGE, sub.num_pages, T)
        oracle.kv_append_bf16(kv_new, p["slot_mapping"][:T], cache)
        oracle.mla_decode(q, sub.block_table, p["cu_seqlens"], p["positions"][:T], PAGE,
                          1.0 / math.sqrt(DK), kv_bf16=cache)
        best = min(best, time.perf_counter() - t0)
    full_rows = int(lay.kv_len.sum())
    return best * full_rows / rows, rows, sub.lanes, oracle.threads()


class CpuStep:
    """The whole configuration-2 step (pack of all 64 lanes, append of their new rows,
    attention of every lane over its full context, 128 heads) through the CPU restatement on
    all host cores.  The inputs (2.25 GB of cached rows) are made once; each call times one
    step."""

    def __init__(self, lay):
        import oracle

        oracle.use_all_cores()
        self.lay = lay
        g = np.random.default_rng(7)
        T = lay.num_tokens
        self.q = g.integers(0, 1 << 16, size=(T, HEADS, DK), dtype=np.uint16) & np.uint16(0xBFFF)
        self.cache = g.integers(0, 1 << 16, size=(lay.num_slots, DK), dtype=np.uint16) & np.uint16(0xBFFF)
        self.kv_new = g.integers(0, 1 << 16, size=(T, DK), dtype=np.uint16) & np.uint16(0xBFFF)

    def run(self) -> float:
        import oracle

        lay, T = self.lay, self.lay.num_tokens
        t0 = time.perf_counter()
        p = oracle.pack(lay.new_rows, lay.context, lay.block_table, PAGE, lay.num_pages, T)
        oracle.kv_append_bf16(self.kv_new, p["slot_mapping"][:T], self.cache)
        oracle.mla_decode(self.q, lay.block_table, p["cu_seqlens"], p["positions"][:T], PAGE,
                          1.0 / math.sqrt(DK), kv_bf16=self.cache)
        return time.perf_counter() - t0

    @staticmethod
    def threads() -> int:
        import oracle

        return oracle.threads()


REF_STEPS_CAP = 3  # whole CPU steps take ~7-12 s each on 16-32 cores: at most this many are timed


def run_reference(args):
    """CPU restatement of the step on all host cores: whole configuration-2 steps, no
    extrapolation.  At most REF_STEPS_CAP steps are timed (the line says how many); the
    warm-up steps run on the first lanes only (about 200K KV rows each)."""
    world, rank, _ = _dist()
    if rank != 0:
        return 0
    from hyperkernel_b200 import workload as W

    lay = W.config2_layout(seed=0, lanes=args.lanes, lo=args.ctx_min, hi=args.ctx_max)
    tokens = lay.num_tokens
    for _ in range(args.warmup):
        cpu_step_seconds(lay, 200_000)
    cpu = CpuStep(lay)
    steps = max(1, min(args.steps, REF_STEPS_CAP))
    secs = [cpu.run() for _ in range(steps)]
    step_s = float(np.mean(secs))
    value = tokens / step_s
    threads = CpuStep.threads()
    line = {
        "impl": "reference", "metric": "ragged decode step tokens/s (MLA config 2)",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
        "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 in, fp64 accumulation", "data": "synthetic (seeded)",
        "config": {"workload": "config2: 64 lanes, ctx log-uniform [1K,128K], 128 heads, "
                               "MLA 512+64, page 64, pack+append+attention",
                   "lanes_per_gpu": lay.lanes, "kv_rows_per_gpu": int(lay.kv_len.sum()),
                   "l2": "inputs larger than L2 (~2 GB KV per GPU), no flush", "attn_impl": 0},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} whole steps (all 64 lanes, {int(lay.kv_len.sum())} KV rows, "
                                   f"128 heads), no extrapolation; warm-up on the first lanes"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_e2e(args, step, q, kv_new, lane_tokens, lane_pos, T, stream, barrier, world, device):
    """Same steps through the public host-buffer API (hyperkernel_b200.step.HostPipeline):
    every step copies its pinned host inputs in and its output out inside the timed region,
    the copies overlapped with the neighbouring steps' kernels.  Timed from an event on the
    input-copy stream before the first step to one on the output-copy stream after the last."""
    import torch
    import torch.distributed as dist
    from hyperkernel_b200.step import HostPipeline

    q_h = q.cpu().pin_memory()
    kv_h = kv_new.cpu().pin_memory()
    lt_h = lane_tokens.cpu().pin_memory()
    lp_h = lane_pos.cpu().pin_memory()
    out_h = [torch.empty((T, HEADS, DV), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    pipe = HostPipeline(step, stream)
    for i in range(args.warmup):
        pipe.submit(lt_h, lp_h, q_h, kv_h, out_h[i % 2], T)
    pipe.finish()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(pipe.h2d)
    for i in range(args.steps):
        pipe.submit(lt_h, lp_h, q_h, kv_h, out_h[i % 2], T)
    e1.record(pipe.d2h)
    pipe.finish()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    return e2e_ms


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hk", choices=["hk", "reference"])
    ap.add_argument("--attn-impl", type=int, default=0, help="0 best, 1 portable, 2 tcgen05")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lanes", type=int, default=64, help="profiling override of config 2")
    ap.add_argument("--ctx-min", type=int, default=1024, help="profiling override of config 2")
    ap.add_argument("--ctx-max", type=int, default=131072, help="profiling override of config 2")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host round trip leg")
    ap.add_argument("--no-legs", action="store_true",
                    help="skip the expert-parallel (config 4) and context-parallel (config 5) legs")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "moe", "linear", "linear-decode", "longctx", "sample", "mixed", "engine",
                             "step"])
    ap.add_argument("--experts", type=int, default=None, help="profiling override of config 4's 256 experts")
    ap.add_argument("--full-dequant", action="store_true",
                    help="longctx: convert the whole FP8 pool to bf16 every step (no mirror)")
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel exchange: NVLink stores from libhk kernels, or NCCL all-to-allv")
    ap.add_argument("--step-batch", default="mixed", choices=["mixed", "decode"],
                    help="--workload step: config 3's mixed batch or config 2's 64 decode lanes")
    ap.add_argument("--engine-requests", type=int, default=None,
                    help="profiling override of the engine workload's 128 requests")
    ap.add_argument("--cp", default="peer", choices=["peer", "nccl"],
                    help="context-parallel exchange: hk_cp_merge over peer memory, or NCCL all-gather + merge")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "decode":
        return run_layer(args)

    import torch
    import torch.distributed as dist

    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import workload as W
    from hyperkernel_b200.clocks import ClockSampler
    from hyperkernel_b200.step import MlaDecodeStep

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))

    # Every rank runs the same lane lengths (equal work per GPU: weak scaling) on its own data.
    lay = W.config2_layout(seed=0, lanes=args.lanes, lo=args.ctx_min, hi=args.ctx_max)
    T = lay.num_tokens
    max_kv = int(lay.kv_len.max())
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    cache = torch.randn((lay.num_slots, DK), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((T, HEADS, DK), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    kv_new = torch.randn((T, DK), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    lane_tokens = torch.from_numpy(lay.new_rows.astype(np.int32)).to(device)
    lane_pos = torch.from_numpy(lay.context.astype(np.int32)).to(device)
    step = MlaDecodeStep(lay.block_table, lay.num_pages, PAGE, HEADS, 1.0 / math.sqrt(DK), T,
                         max_kv, device, cache=cache, impl=args.attn_impl)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (untimed)
    for _ in range(args.warmup):
        step.run(lane_tokens, lane_pos, q, kv_new, T)
    torch.cuda.synchronize()
    hk.check_errors()

    sampler = ClockSampler(local).start()
    n_ev = args.steps
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = hk.kernel_launches()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start.record(stream)
    for i in range(args.steps):
        p = step.packed
        s = hk.stream_ptr(stream)
        hk.call("hk_pack", hk.ptr(lane_tokens), hk.ptr(lane_pos), hk.ptr(step.block_table),
                step.block_table.shape[1], step.lanes, PAGE, step.num_pages, T,
                hk.ptr(p["cu_seqlens"]), hk.ptr(p["seq_lens"]), hk.ptr(p["positions"]),
                hk.ptr(p["slot_mapping"]), hk.ptr(p["token_lane"]), hk.ptr(p["active"]), s)
        hk.call("hk_kv_append_bf16", hk.ptr(kv_new), hk.ptr(p["slot_mapping"]), T, DK, PAGE,
                hk.ptr(step.cache), step.cache.shape[0], s)
        ev_a[i].record(stream)
        step.attention_only(q, T, stream)
        ev_b[i].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    hk.check_errors()
    ms = start.elapsed_time(end)
    attn_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ev_a, ev_b)]))
    if world > 1:
        t = torch.tensor([ms, attn_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, attn_ms = float(t[0]), float(t[1])
    clocks = sampler.summary(t0, t1)

    # end to end through the host-facing step with pinned host buffers
    e2e_ms = float("nan")
    if not args.no_e2e:
        e2e_ms = run_e2e(args, step, q, kv_new, lane_tokens, lane_pos, T, stream, barrier, world,
                         device)
    hk.check_errors()
    legs = {}
    if not args.no_legs:
        from hyperkernel_b200 import parallel as par

        # the headline step's buffers go first: the legs hold ~12 GB of expert weights and
        # ~2.3 GB of FP8 pool and mirror per GPU
        del step, cache
        for name, leg in (("ep", leg_ep), ("cp", leg_cp), ("engine", leg_engine)):
            torch.cuda.empty_cache()
            try:
                if name == "engine":
                    legs[name] = leg(args, torch, dist, hk, world, rank, local, device, barrier, peak_hbm())
                else:
                    legs[name] = leg(args, torch, dist, hk, par, world, rank, device, stream, barrier, peak_hbm())
            except Exception as e:  # noqa: BLE001 - a failed leg is reported, the headline stands
                legs[name] = {"error": f"{type(e).__name__}: {e}"[:400]}
    total_tokens = T * world
    value = total_tokens * args.steps / (ms / 1e3)
    e2e_value = None if args.no_e2e else total_tokens * args.steps / (e2e_ms / 1e3)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except Exception:
        peak, peak_src = 6650.0, "fallback"
    abytes = attn_bytes(lay.kv_len, T)
    achieved = abytes / (attn_ms / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cs = CpuStep(lay)
        secs = cs.run()
        cpu = {"value": T / secs, "unit": "tokens/s", "cores": CpuStep.threads(), "kind": "port",
               "sample": f"one whole step (all {lay.lanes} lanes, {int(lay.kv_len.sum())} KV rows, "
                         f"128 heads), no extrapolation"}
        del cs

    if rank == 0:
        line = {
            "metric": "ragged decode step tokens/s (MLA config 2)", "value": value,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "config2: 64 lanes, ctx log-uniform [1K,128K], 128 heads, "
                                   "MLA 512+64, page 64, pack+append+attention",
                       "lanes_per_gpu": lay.lanes, "kv_rows_per_gpu": int(lay.kv_len.sum()),
                       "l2": "inputs larger than L2 (~2 GB KV per GPU), no flush",
                       "attn_impl": args.attn_impl},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         # DRAM read+write bytes per launch: 1.044 x algorithmic in an ncu
                         # capture of 64 lanes, ctx <= 16K, scaled here by the KV rows.
                         "traffic": TRAFFIC_PER_ALGORITHMIC_BYTE * abytes,
                         "traffic_source": "ncu dram__bytes_read+write of a 64-lane ctx<=16K "
                                           "launch (1.044 x algorithmic), scaled by KV rows",
                         "kernel": "attention (hk_mla_decode)", "kernel_ms": attn_ms,
                         "algorithmic_bytes": abytes, "peak_source": peak_src,
                         "tflops": attn_flops(lay.kv_len) / (attn_ms / 1e3) / 1e12},
            "cpu_baseline": cpu,
            "e2e": None if e2e_value is None else {
                "value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": MlaDecodeStep.h2d_bytes(lay.lanes, T, HEADS),
                "d2h_bytes_per_step": MlaDecodeStep.d2h_bytes(T, HEADS)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            **legs,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------
# the two shards with a real exchange, run after the headline step on every N
# ------------------------------------------------------------------------------------------

EP_SEED, CP_SEED = 4242, 555


def _bits_equal(torch, a, b) -> bool:
    return bool(torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16)))


def _errs_np(got, want):
    """(normwise, element-wise) max-abs-rel; the element-wise figure divides by each element's
    own magnitude, floored at 10% of the largest."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    top = max(float(np.abs(want).max()), 1e-30)
    d = np.abs(got - want)
    return float(d.max() / top), float((d / np.maximum(np.abs(want), 0.1 * top)).max())


def leg_ep(args, torch, dist, hk, par, world, rank, device, stream, barrier, hbm_peak):
    """Config 4's MoE layer, expert parallel over the N GPUs: rank r owns routed experts
    [r E/N, (r+1) E/N) and its own 512 tokens (weak scaling); dispatch and return are this
    library's NVLink peer stores (hk_ep_counts / hk_ep_dispatch / hk_ep_return over symmetric
    buffers), the shared expert is replicated.  Every rank generates the same full weight set
    (one seed) so that rank 0 can run its tokens through all 256 experts on one GPU: the
    parity field says whether the EP output equals that one-GPU output bit for bit."""
    T, E, H, I, K = MOE_T, MOE_E, MOE_H, MOE_I, MOE_K
    e0, e1 = par.expert_range(E, world, rank)
    gw = torch.Generator(device=device)
    gw.manual_seed(EP_SEED)
    w13 = _rand_e4m3(torch, (E + 1, 2 * I, H), gw, device)  # expert E is the shared expert
    w2 = _rand_e4m3(torch, (E + 1, H, I), gw, device)
    s13 = torch.rand((E + 1, 2 * I // 128, H // 128), generator=gw, device=device) * 1e-3
    s2 = torch.rand((E + 1, H // 128, I // 128), generator=gw, device=device) * 1e-3
    loc = (w13[e0:e1], s13[e0:e1], w2[e0:e1], s2[e0:e1])
    shr = (w13[E:], s13[E:], w2[E:], s2[E:])
    gx = torch.Generator(device=device)
    gx.manual_seed(EP_SEED + 1 + rank)
    x = torch.randn((T, H), generator=gx, device=device).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gx, device=device)
    rows = T * K
    rows_max = rows * world
    ws = torch.empty(hk.moe_workspace_size(rows_max + T, H, I), dtype=torch.uint8, device=device)
    ws_sh = torch.empty(hk.moe_workspace_size(T, H, I), dtype=torch.uint8, device=device)
    y_buf = torch.empty((rows_max + T, H), dtype=torch.bfloat16, device=device)
    y_sh = torch.empty((T, H), dtype=torch.bfloat16, device=device)
    every = torch.arange(T, dtype=torch.int32, device=device)
    sh_off = torch.tensor([0, T], dtype=torch.int32, device=device)
    # the shared expert runs in the same grouped-FFN call as this rank's routed experts, as
    # expert 0 of a weight copy ordered [shared, local experts]
    peer = par.EpPeer(E, T, K, H, shared_tokens=T) if world > 1 else None
    fold = tuple(torch.cat([a[E:], a[e0:e1]]) for a in (w13, s13, w2, s2)) if peer is not None else None
    # one GPU: the shared expert as expert E of the routed call (rows [T*K, T*K + T))
    off_ext = torch.empty(E + 2, dtype=torch.int32, device=device)
    off_ext[E + 1] = rows + T
    tok_ext = torch.empty(rows + T, dtype=torch.int32, device=device)
    tok_ext[rows:] = every

    def step(ev=None):
        xq, sx = hk.quant_fp8(x)
        ids, w = hk.route(logits, None, K, 1.0)
        if peer is not None:
            off, tok, pw, inv = hk.permute(ids, w, E)
            xr, sr, foff, fperm, frows = peer.dispatch_with_shared(xq, sx, off, tok)
        else:
            off, tok, pw, inv = hk.permute(ids, w, E, offsets=off_ext[:E + 1], perm_token=tok_ext[:rows])
        if ev is not None:
            ev[0].record(stream)
        if peer is not None:
            y_all = hk.moe_grouped(xr, sr, foff, fperm, frows, H, I, *fold, out=y_buf, workspace=ws)
            y_shared, y_loc = y_all[:T], y_all[T:]
        else:
            y_all = hk.moe_grouped(xq, sx, off_ext, tok_ext, rows + T, H, I, w13, s13, w2, s2, out=y_buf,
                                   workspace=ws)
            y_loc, y_shared = y_all[:rows], y_all[rows:rows + T]
        if ev is not None:
            ev[1].record(stream)
        y = peer.give_back(y_loc) if peer is not None else y_loc
        return hk.combine(y, pw, inv, y_shared, T, K), (peer.local_off if peer is not None else off)

    for _ in range(args.warmup):
        out, off = step()
    torch.cuda.synchronize()
    hk.check_errors()
    counts = (off[1:] - off[:-1]).cpu().numpy()
    hit, rows_in = int((counts > 0).sum()), int(counts.sum())
    wbytes = (hit + 1) * 3 * H * I + (hit + 1) * (2 * I // 128 * H // 128 + H // 128 * I // 128) * 4
    abytes = wbytes + (rows_in + T) * (H + 2 * 2 * I + 2 * H)
    launches0 = hk.kernel_launches()
    barrier()
    ms, ffn_ms = _timed(torch, lambda ev: step(ev), args.steps, stream)
    barrier()
    launches = hk.kernel_launches() - launches0
    hk.check_errors()
    ms, ffn_ms = _reduce_max(torch, dist, world, device, ms, ffn_ms)
    out, _ = step()  # every rank takes the same exchange steps; rank 0 checks this one
    torch.cuda.synchronize()
    parity = None
    if rank == 0 and world > 1:
        xq, sx = hk.quant_fp8(x)
        ids, w = hk.route(logits, None, K, 1.0)
        off1, tok1, pw1, inv1 = hk.permute(ids, w, E)
        y1 = hk.moe_grouped(xq, sx, off1, tok1, rows, H, I, w13[:E], s13[:E], w2[:E], s2[:E])
        ys1 = hk.moe_grouped(xq, sx, sh_off, every, T, H, I, *shr)
        one = hk.combine(y1, pw1, inv1, ys1, T, K)
        torch.cuda.synchronize()
        norm, elem = _errs_np(out.float().cpu().numpy(), one.float().cpu().numpy())
        parity = {"against": "rank 0's 512 tokens through all 256 routed experts + the shared one on one GPU",
                  "bit_exact": _bits_equal(torch, out, one), "normwise": norm, "elementwise": elem}
    barrier()
    if peer is not None:
        peer.close()
    achieved = abytes / (ffn_ms / 1e3) / 1e9
    return {
        "workload": "config4 MoE layer: 512 tokens per GPU, 256 routed experts top-8 + 1 shared, hidden 7168, "
                    "inter 2048, FP8 128x128 block scales; quant+route+permute+dispatch+grouped FFN+return+combine",
        "parallelism": f"ep{world}" if world > 1 else "single GPU (no exchange)",
        "exchange": "NVLink peer stores from hk_ep_counts/hk_ep_dispatch/hk_ep_return, bounded epoch waits; "
                    "the shared expert in the same grouped-FFN launch as the rank's routed experts"
                    if world > 1 else None,
        "scaling": "weak", "ms_per_step": ms / args.steps, "tokens_per_s": T * world * args.steps / (ms / 1e3),
        "routed_rows_per_s": rows * world * args.steps / (ms / 1e3), "experts_per_gpu": e1 - e0,
        "ffn_ms_rank0_max": ffn_ms, "ffn_hbm_gbs": achieved, "ffn_frac_of_hbm": achieved / hbm_peak,
        "gpu_launches": int(launches), "parity": parity,
    }


def leg_cp(args, torch, dist, hk, par, world, rank, device, stream, barrier, hbm_peak):
    """Config 5 (one lane at 1,048,576 cached rows + 7 at U[4K, 64K], 1 + 4 spec-verify rows
    each, FP8 latent cache), context parallel over the N GPUs: the short lanes go largest first
    to the least-loaded rank and the long lane's KV is cut into page-aligned position ranges
    that bring every rank to the same number of KV rows (parallel.cp_plan); each rank keeps
    a bf16 mirror of its pages current and runs one tcgen05 partial launch over its ranges,
    then the long lane's (o, lse) partials are all-gathered over NCCL and merged by LSE (strong
    scaling).  Every rank builds the same pool (one seed); rank 0 then runs the whole batch on
    one GPU and the parity field compares the merged long-lane rows with it (on one GPU the
    merge is checked by splitting the lane 8 ways on that GPU)."""
    from hyperkernel_b200 import workload as W

    lay = W.config5_layout(seed=0)
    T, L, H = lay.num_tokens, lay.lanes, HEADS
    kv = lay.kv_len.astype(np.int64)
    begin = np.zeros(L, np.int32)
    end = np.zeros(L, np.int32)
    ranges, owner = par.cp_plan(int(kv[0]), kv[1:], world)  # equal KV rows per rank
    begin[0], end[0] = ranges[rank]
    for ln in range(1, L):
        if owner[ln - 1] == rank:
            end[ln] = kv[ln]
    g = torch.Generator(device=device)
    g.manual_seed(CP_SEED)
    cache = _rand_e4m3(torch, (lay.num_slots, DK), g, device)
    scales = torch.rand((lay.num_slots,), generator=g, device=device) * 0.01 + 0.001
    q = torch.randn((T, H, DK), generator=g, device=device).to(torch.bfloat16)
    kv_new = torch.randn((T, DK), generator=g, device=device).to(torch.bfloat16)
    lane_tokens = torch.from_numpy(lay.new_rows.astype(np.int32)).to(device)
    lane_pos = torch.from_numpy(lay.context.astype(np.int32)).to(device)
    bt = torch.from_numpy(lay.block_table).to(device)
    kb, ke = torch.from_numpy(begin).to(device), torch.from_numpy(end).to(device)
    max_kv = int(kv.max())
    scale = 1.0 / math.sqrt(DK)
    long_rows = int(lay.new_rows[0]) * H
    # zeroed: the tcgen05 kernel reads whole pages, the scratch page included, at zero weight, so the
    # pages this rank does not convert must hold finite values
    kv_bf16 = torch.zeros((lay.num_slots, DK), dtype=torch.bfloat16, device=device)
    my_pages = torch.from_numpy(np.concatenate(
        [lay.block_table[i, int(begin[i]) // PAGE:(int(end[i]) + PAGE - 1) // PAGE] for i in range(L)]
    ).astype(np.int32)).to(device)
    hk.kv_dequant_fp8(cache, scales, PAGE, out=kv_bf16, pages=None if world == 1 else my_pages)
    # the exchange: this library's fused peer-memory merge (hk_cp_merge over hk_sym_alloc buffers),
    # or --cp nccl: an NCCL all-gather of the partials, then hk_lse_merge
    peer = par.CpPeer(T * H, 512, long_rows) if world > 1 and args.cp == "peer" else None

    def step(ev=None):
        pk = hk.pack(lane_tokens, lane_pos, bt, PAGE, lay.num_pages, T)
        hk.kv_append_fp8(kv_new, pk["slot_mapping"], cache, scales)
        if ev is not None:
            ev[0].record(stream)
        hk.kv_dequant_fp8_rows(cache, scales, pk["slot_mapping"], kv_bf16, PAGE)
        if world == 1:
            o, lse = hk.mla_decode(q, kv_bf16, bt, pk["cu_seqlens"], pk["positions"], PAGE, max_kv, scale)
        elif peer is not None:
            ob, lb = peer.next_buffers()
            o, lse = hk.mla_partial(q, kv_bf16, bt, pk["cu_seqlens"], pk["positions"], kb, ke, PAGE, max_kv,
                                    scale, out=ob.view(T, H, 512), lse=lb.view(T, H))
        else:
            o, lse = hk.mla_partial(q, kv_bf16, bt, pk["cu_seqlens"], pk["positions"], kb, ke, PAGE, max_kv,
                                    scale)
        if ev is not None:
            ev[1].record(stream)
        if peer is not None:
            return peer.merge()
        if world > 1:
            return par.cp_merge(o.view(T * H, 512)[:long_rows], lse.view(T * H)[:long_rows])
        return o.view(T * H, 512)[:long_rows], lse.view(T * H)[:long_rows]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    hk.check_errors()
    launches0 = hk.kernel_launches()
    barrier()
    ms, attn_ms = _timed(torch, step, args.steps, stream)
    barrier()
    launches = hk.kernel_launches() - launches0
    hk.check_errors()
    ms, attn_ms = _reduce_max(torch, dist, world, device, ms, attn_ms)
    merged, merged_lse = step()
    torch.cuda.synchronize()
    parity = None
    if rank == 0:
        full = hk.kv_dequant_fp8(cache, scales, PAGE)
        pk = hk.pack(lane_tokens, lane_pos, bt, PAGE, lay.num_pages, T)
        whole, whole_lse = hk.mla_decode(q, full, bt, pk["cu_seqlens"], pk["positions"], PAGE, max_kv, scale)
        whole = whole.view(T * H, 512)[:long_rows]
        whole_lse = whole_lse.view(T * H)[:long_rows]
        how = f"merged partials of {world} GPUs"
        if world == 1:  # the merge on one GPU: the long lane split 8 ways, partials merged by LSE
            parts, lses = [], []
            for b0, b1 in par.cp_ranges(int(kv[0]), 8):
                bb, be = np.zeros(L, np.int32), np.zeros(L, np.int32)
                bb[0], be[0] = b0, b1
                o, l = hk.mla_partial(q, full, bt, pk["cu_seqlens"], pk["positions"],
                                      torch.from_numpy(bb).to(device), torch.from_numpy(be).to(device),
                                      PAGE, max_kv, scale)
                parts.append(o.view(T * H, 512)[:long_rows])
                lses.append(l.view(T * H)[:long_rows])
            merged, merged_lse = hk.lse_merge(torch.stack(parts).contiguous(), torch.stack(lses).contiguous())
            how = "8 partials of the long lane on one GPU, merged by LSE"
        torch.cuda.synchronize()
        hk.check_errors()
        norm, elem = _errs_np(merged.float().cpu().numpy(), whole.float().cpu().numpy())
        lse_err = float((merged_lse - whole_lse).abs().max())
        parity = {"against": "the whole long lane (5 rows x 128 heads) by hk_mla_decode on one GPU", "merged": how,
                  "normwise": norm, "elementwise": elem, "lse_max_abs": lse_err, "tolerance": 2e-2,
                  "ok": bool(norm <= 2e-2 and elem <= 2e-2 and lse_err <= 1e-3)}
    barrier()
    if peer is not None:
        peer.close()
    my_rows = int(sum(int(end[i]) - int(begin[i]) for i in range(L)))
    flops = 2 * H * (DK + 512) * my_rows * int(lay.new_rows[0])
    return {
        "workload": "config5: 1 lane at 1,048,576 + 7 at U[4K,64K] cached rows, 1+4 rows each, FP8 latent KV, "
                    "128 heads; pack+FP8 append+mirror rows+tcgen05 attention (+ all-gather and LSE merge of the "
                    "long lane's partials across GPUs)",
        "parallelism": f"cp{world}" if world > 1 else "single GPU",
        "exchange": (("hk_cp_merge: every rank's long-lane (o, lse) partial (1.3 MB) read over NVLink from its "
                      "hk_sym_alloc buffer and merged by LSE in one kernel, bounded epoch waits")
                     if args.cp == "peer" else
                     "NCCL all-gather of the long lane's (o, lse) partials (1.3 MB per rank) + hk_lse_merge")
                    if world > 1 else None,
        "scaling": "strong", "ms_per_step": ms / args.steps, "rows_per_s": T * args.steps / (ms / 1e3),
        "kv_rows_total": int(kv.sum()), "kv_rows_rank0": my_rows if rank == 0 else None,
        "attn_ms_max": attn_ms, "attn_tflops_rank": flops / (attn_ms / 1e3) / 1e12,
        "gpu_launches": int(launches), "parity": parity,
    }


# ------------------------------------------------------------------------------------------
# config 3 and config 4 layers (--workload linear | moe), one GPU
# ------------------------------------------------------------------------------------------

MOE_T, MOE_E, MOE_H, MOE_I, MOE_K = 512, 256, 7168, 2048, 8
# MLA projections of one layer (DeepSeek-V3 shapes): (name, out features, in features)
LINEAR_T = 48 + 2 * 2048
LINEAR_PROJ = [("q_a", 1536, 7168), ("q_b", 128 * 192, 1536), ("kv_a", 576, 7168), ("o", 7168, 128 * 128)]


def peak_hbm() -> float:
    return _peaks()[0]


def _peaks():
    try:
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(pk["hbm_gbs"]), 2.0 * float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 2 * 1590.0, "fallback"


def _rand_e4m3(torch, shape, gen, device):
    """Seeded random e4m3 bytes (the two NaN encodings avoided)."""
    b = torch.randint(0, 256, shape, generator=gen, device=device, dtype=torch.uint8)
    return torch.where((b & 0x7F) == 0x7F, b ^ 1, b)


def _timed(torch, fn, steps, stream, inner=True):
    """Times `steps` calls of fn on `stream`; returns (total ms, mean ms of the region fn marks
    with its event pair, or None when inner is False)."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(steps):
        fn(ev[i])
    end.record(stream)
    torch.cuda.synchronize()
    inner_ms = float(np.mean([a.elapsed_time(b) for a, b in ev])) if inner else None
    return start.elapsed_time(end), inner_ms


def _reduce_max(torch, dist, world, device, *vals):
    """Max over ranks of the given floats (device timings are taken as the slowest rank)."""
    if world == 1:
        return vals
    t = torch.tensor(vals, device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return tuple(float(v) for v in t.tolist())


def run_layer(args):
    import datetime

    import torch
    import torch.distributed as dist

    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as par
    from hyperkernel_b200.clocks import ClockSampler

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=device)
    gen.manual_seed(7 + rank)
    hbm_peak, fp8_peak, peak_src = _peaks()

    def barrier():
        if world > 1:
            dist.barrier()

    if args.workload == "moe":
        line = _run_moe(args, torch, dist, hk, par, ClockSampler, world, rank, local, device, stream, gen,
                        hbm_peak, fp8_peak, peak_src, barrier)
    elif args.workload == "longctx":
        line = _run_longctx(args, torch, dist, hk, par, ClockSampler, world, rank, local, device, stream, gen,
                            hbm_peak, peak_src, barrier)
    elif args.workload == "mixed":
        line = _run_mixed(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen,
                          hbm_peak, peak_src, barrier)
    elif args.workload == "linear-decode":
        line = _run_linear_decode(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen,
                                  hbm_peak, peak_src, barrier)
    elif args.workload == "step":
        line = _run_step(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen,
                         hbm_peak, peak_src, barrier)
    elif args.workload == "sample":
        line = _run_sample(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen,
                           hbm_peak, peak_src, barrier)
    elif args.workload == "engine":
        line = _run_engine(args, torch, dist, hk, ClockSampler, world, rank, local, device, barrier, hbm_peak,
                           peak_src)
    else:
        line = _run_linear(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen,
                           fp8_peak, peak_src, barrier)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _run_moe(args, torch, dist, hk, par, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
             fp8_peak, peak_src, barrier):
    """Config 4.  N > 1: expert parallel, rank r owning experts [r E/N, (r+1) E/N) and its own
    512 tokens (weak scaling); dispatch and return are NCCL all-to-allv (hyperkernel_b200/
    parallel.py), the shared expert is replicated."""
    T, E, H, I, K = MOE_T, args.experts or MOE_E, MOE_H, MOE_I, MOE_K
    e0, e1 = par.expert_range(E, world, rank)
    El = e1 - e0
    # the local routed experts and then the shared one in one weight array each: on one GPU the
    # shared expert runs as expert E of the routed grouped call (rows [T*K, T*K + T) = every
    # token), as the model step behind hk_open_mla runs it
    w13_all = _rand_e4m3(torch, (El + 1, 2 * I, H), gen, device)
    w2_all = _rand_e4m3(torch, (El + 1, H, I), gen, device)
    s13_all = torch.rand((El + 1, 2 * I // 128, H // 128), generator=gen, device=device) * 1e-3
    s2_all = torch.rand((El + 1, H // 128, I // 128), generator=gen, device=device) * 1e-3
    w13, w2, s13, s2 = w13_all[:El], w2_all[:El], s13_all[:El], s2_all[:El]
    sh13, sh2, shs13, shs2 = w13_all[El:], w2_all[El:], s13_all[El:], s2_all[El:]
    x = torch.randn((T, H), generator=gen, device=device).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=device)
    rows = T * K
    rows_max = rows * world  # the most rows one rank's experts can receive
    ws = torch.empty(hk.moe_workspace_size(rows_max + T, H, I), dtype=torch.uint8, device=device)
    ws_sh = torch.empty(hk.moe_workspace_size(T, H, I), dtype=torch.uint8, device=device)
    y_buf = torch.empty((rows_max + T, H), dtype=torch.bfloat16, device=device)
    y_sh = torch.empty((T, H), dtype=torch.bfloat16, device=device)
    sh_off = torch.tensor([0, T], dtype=torch.int32, device=device)
    sh_tok = torch.arange(T, dtype=torch.int32, device=device)
    off_ext = torch.empty(E + 2, dtype=torch.int32, device=device)
    off_ext[E + 1] = rows + T
    tok_ext = torch.empty(rows + T, dtype=torch.int32, device=device)
    tok_ext[rows:] = sh_tok
    peer = par.EpPeer(E, T, K, H, shared_tokens=T) if world > 1 and args.ep == "peer" else None
    # with the peer exchange the shared expert runs in the rank's grouped-FFN call, as expert 0
    # of a weight copy ordered [shared, local experts]
    fold = tuple(torch.cat([b[El:], b[:El]]) for b in (w13_all, s13_all, w2_all, s2_all)) if peer is not None else None
    info = {}

    def step(x_in, logits_in, ev=None):
        xq, sx = hk.quant_fp8(x_in)
        ids, w = hk.route(logits_in, None, K, 1.0)
        if world == 1:
            off, tok, pw, inv = hk.permute(ids, w, E, offsets=off_ext[:E + 1], perm_token=tok_ext[:rows])
        else:
            off, tok, pw, inv = hk.permute(ids, w, E)
        if peer is not None:
            xr, sr, loff, lperm, n_in = peer.dispatch_with_shared(xq, sx, off, tok)
        elif world > 1:
            xr, sr, loff, lperm, plan = par.ep_dispatch(xq, sx, off, tok, E)
            n_in = xr.shape[0]
        if ev is not None:
            ev[0].record(stream)
        if peer is not None:
            y_all = hk.moe_grouped(xr, sr, loff, lperm, n_in, H, I, *fold, out=y_buf, workspace=ws)
            shared, y_local = y_all[:T], y_all[T:]
        elif world > 1:
            y_local = hk.moe_grouped(xr, sr, loff, lperm, n_in, H, I, w13, s13, w2, s2, out=y_buf, workspace=ws)
            shared = hk.moe_grouped(xq, sx, sh_off, sh_tok, T, H, I, sh13, shs13, sh2, shs2, out=y_sh,
                                    workspace=ws_sh)
        else:
            y_all = hk.moe_grouped(xq, sx, off_ext, tok_ext, rows + T, H, I, w13_all, s13_all, w2_all, s2_all,
                                   out=y_buf, workspace=ws)
            y_local, shared = y_all[:rows], y_all[rows:rows + T]
        if ev is not None:
            ev[1].record(stream)
        if peer is not None:
            y = peer.give_back(y_local)
        elif world > 1:
            y = par.ep_return(y_local, plan, lperm)
        else:
            y = y_local
        return hk.combine(y, pw, inv, shared, T, K), (peer.local_off if peer is not None else
                                                      loff if world > 1 else off)

    for _ in range(args.warmup):
        _, off = step(x, logits)
    torch.cuda.synchronize()
    hk.check_errors()
    counts = (off[1:] - off[:-1]).cpu().numpy()  # rows per expert this rank ran (local experts when N > 1)
    hit, rows_in = int((counts > 0).sum()), int(counts.sum())
    wbytes = (hit + 1) * 3 * H * I + (hit + 1) * (2 * I // 128 * H // 128 + H // 128 * I // 128) * 4
    abytes = wbytes + (rows_in + T) * (H + 2 * 2 * I + 2 * H)
    flops = 2 * (rows_in + T) * 3 * H * I
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    ms, ffn_ms = _timed(torch, lambda ev: step(x, logits, ev), args.steps, stream)
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    hk.check_errors()
    ms, ffn_ms = _reduce_max(torch, dist, world, device, ms, ffn_ms)
    hx = torch.empty((T, H), dtype=torch.bfloat16).pin_memory().copy_(x.cpu())
    hl = torch.empty((T, E), dtype=torch.float32).pin_memory().copy_(logits.cpu())
    hout = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)

    def e2e(ev):
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        out, _ = step(dx, dl)
        hout.copy_(out, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _moe_cpu_baseline(x, logits, w13, s13, w2, s2, sh13, shs13, sh2, shs2)
    achieved = abytes / (ffn_ms / 1e3) / 1e9
    return {
        "metric": "MoE layer tokens/s (config 4)", "value": T * world * args.steps / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32",
        "data": "synthetic (seeded): e4m3 weights, N(0,1) activations and router logits",
        "config": {"workload": "config4: 512 tokens per GPU, 256 routed experts top-8 + 1 shared, hidden 7168, "
                               "inter 2048, FP8 128x128 block scales; quant+route+permute+grouped FFN+combine",
                   "parallelism": (f"ep{world} ({args.ep})" if world > 1 else "single"),
                   "experts_per_gpu": El, "experts_hit_rank0": hit, "rows_in_rank0": rows_in,
                   "l2": "11.4 GB / N of expert weights per GPU per step, no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": None,
                     "kernel": "grouped expert FFN on rank 0 (hk_moe_grouped: local experts + shared)",
                     "kernel_ms": ffn_ms, "algorithmic_bytes": abytes, "peak_source": peak_src,
                     "tflops": flops / (ffn_ms / 1e3) / 1e12,
                     "tensor_frac_of_fp8_peak": flops / (ffn_ms / 1e3) / 1e12 / fp8_peak},
        "cpu_baseline": cpu,
        "e2e": {"value": T * world * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2 + T * E * 4, "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": int(launches), "clocks": clocks,
    }


def _run_longctx(args, torch, dist, hk, par, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
                 peak_src, barrier):
    """Config 5: one lane at 1M cached tokens and 7 at U[4K, 64K], each verifying 1 + 4 rows,
    FP8 latent cache.  N > 1: the short lanes go largest first to the least-loaded rank and the
    long lane's KV is split into page-aligned position ranges that bring every rank to the same
    number of KV rows (context parallel, parallel.cp_plan); every rank converts the pages
    of its ranges to the blocked bf16 layout and runs one tcgen05 partial attention launch over
    them (--attn-impl 1: the CUDA-core FP8 partial kernel instead), then the long lane's
    partials are all-gathered and merged by LSE (strong scaling: the total work is fixed)."""
    from hyperkernel_b200 import workload as W

    lay = W.config5_layout(seed=0)
    T, L, H = lay.num_tokens, lay.lanes, HEADS
    kv = lay.kv_len.astype(np.int64)
    begin = np.zeros(L, np.int32)
    end = np.zeros(L, np.int32)
    ranges, owner = par.cp_plan(int(kv[0]), kv[1:], world)  # equal KV rows per rank
    begin[0], end[0] = ranges[rank]
    for ln in range(1, L):
        if owner[ln - 1] == rank:
            end[ln] = kv[ln]
    my_rows = int(sum(int(end[i]) - int(begin[i]) for i in range(L)))
    cache = _rand_e4m3(torch, (lay.num_slots, DK), gen, device)
    scales = torch.rand((lay.num_slots,), generator=gen, device=device) * 0.01 + 0.001
    q = torch.randn((T, H, DK), generator=gen, device=device).to(torch.bfloat16)
    kv_new = torch.randn((T, DK), generator=gen, device=device).to(torch.bfloat16)
    lane_tokens = torch.from_numpy(lay.new_rows.astype(np.int32)).to(device)
    lane_pos = torch.from_numpy(lay.context.astype(np.int32)).to(device)
    bt = torch.from_numpy(lay.block_table).to(device)
    kb = torch.from_numpy(begin).to(device)
    ke = torch.from_numpy(end).to(device)
    max_kv = int(kv.max())
    scale = 1.0 / math.sqrt(DK)
    long_rows = int(lay.new_rows[0]) * H

    portable = world > 1 and args.attn_impl == 1
    kv_bf16 = None if portable else torch.zeros((lay.num_slots, DK), dtype=torch.bfloat16, device=device)
    # pages of this rank's ranges (the long lane's shard and its short lanes)
    my_pages = torch.from_numpy(np.concatenate(
        [lay.block_table[i, int(begin[i]) // PAGE:(int(end[i]) + PAGE - 1) // PAGE] for i in range(L)]
    ).astype(np.int32)).to(device)

    # The tcgen05 kernel reads a page-blocked bf16 mirror of the FP8 pool (of this rank's pages
    # on N > 1): converted once here, then kept current by converting each step's appended rows
    # (--full-dequant converts the whole pool, or the rank's pages, every step instead).
    if kv_bf16 is not None:
        hk.kv_dequant_fp8(cache, scales, PAGE, out=kv_bf16, pages=None if world == 1 else my_pages)

    def step(ev=None, q_in=None, kv_in=None):
        q_use = q if q_in is None else q_in
        pk = hk.pack(lane_tokens, lane_pos, bt, PAGE, lay.num_pages, T)
        hk.kv_append_fp8(kv_new if kv_in is None else kv_in, pk["slot_mapping"], cache, scales)
        if ev is not None:
            ev[0].record(stream)
        if kv_bf16 is not None:
            if args.full_dequant:
                hk.kv_dequant_fp8(cache, scales, PAGE, out=kv_bf16, pages=None if world == 1 else my_pages)
            else:
                hk.kv_dequant_fp8_rows(cache, scales, pk["slot_mapping"], kv_bf16, PAGE)
        if world == 1:
            o, lse = hk.mla_decode(q_use, kv_bf16, bt, pk["cu_seqlens"], pk["positions"], PAGE, max_kv, scale)
        elif portable:
            o, lse = hk.mla_partial_fp8(q_use, cache, scales, bt, pk["cu_seqlens"], pk["positions"], kb, ke, PAGE,
                                        max_kv, scale)
        else:
            o, lse = hk.mla_partial(q_use, kv_bf16, bt, pk["cu_seqlens"], pk["positions"], kb, ke, PAGE, max_kv,
                                    scale)
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            return par.cp_merge(o.view(T * H, 512)[:long_rows], lse.view(T * H)[:long_rows])
        return o, lse

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    hk.check_errors()
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    ms, attn_ms = _timed(torch, step, args.steps, stream)
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    hk.check_errors()
    ms, attn_ms = _reduce_max(torch, dist, world, device, ms, attn_ms)
    # end to end: the step's queries and new latent rows from pinned host memory, its outputs
    # (the merged long lane's on N > 1) back to pinned host memory
    hq = torch.empty(q.shape, dtype=q.dtype).pin_memory().copy_(q.cpu())
    hkv = torch.empty(kv_new.shape, dtype=kv_new.dtype).pin_memory().copy_(kv_new.cpu())
    dq, dkv = torch.empty_like(q), torch.empty_like(kv_new)
    h_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in step()]

    def e2e(ev):
        dq.copy_(hq, non_blocking=True)
        dkv.copy_(hkv, non_blocking=True)
        for h, d in zip(h_out, step(None, dq, dkv)):
            h.copy_(d, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # one short lane of the workload with its 1 + 4 rows, scaled by query-KV pairs
        c_dt, c_pairs, c_threads = cpu_lanes_seconds([int(lay.context[1])], [int(lay.new_rows[1])], fp8=True)
        step_s = c_dt * _query_kv_pairs(lay) / c_pairs
        cpu = {"value": T / step_s, "unit": "query rows/s", "cores": c_threads, "kind": "port",
               "sample": f"pack + FP8 append + attention of one lane ({int(lay.context[1])} cached rows, "
                         f"{int(lay.new_rows[1])} rows, 128 heads), scaled by query-KV pairs"}
    abytes = my_rows * (DK + 4) + T * H * (DK * 2 + 512 * 4 + 4)
    flops = 2 * H * (DK + 512) * sum(int(end[i]) - int(begin[i]) for i in range(L)) * int(lay.new_rows[0])
    bf16_peak = _peaks()[1] / 2.0
    tflops = flops / (attn_ms / 1e3) / 1e12
    return {
        "metric": "long-context spec-verify rows/s (config 5)", "value": T * args.steps / (ms / 1e3),
        "unit": "query rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 KV, bf16 q, fp32 accumulation", "data": "synthetic (seeded)",
        "config": {"workload": "config5: 1 lane at 1,048,576 + 7 at U[4K,64K] cached rows, 1+4 rows each, "
                               "FP8 latent KV, 128 heads; pack+append+attention (+ LSE merge of the long "
                               "lane's partials across GPUs)",
                   "parallelism": f"cp{world}" if world > 1 else "single",
                   "kv_rows_total": int(kv.sum()), "kv_rows_rank0": my_rows,
                   "l2": "0.75 GB of FP8 KV, no flush"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": tflops / bf16_peak, "traffic": None,
                     "kernel": ("CUDA-core FP8 partial attention on rank 0 (hk_mla_partial_fp8)" if portable else
                                ("FP8 pool -> blocked bf16 every step (hk_kv_dequant_fp8" if args.full_dequant else
                                 "bf16 mirror of the FP8 pool, the step's appended rows converted "
                                 "(hk_kv_dequant_fp8_rows") + ") + tcgen05 attention ("
                                + ("hk_mla_decode)" if world == 1 else "hk_mla_partial over rank 0's ranges)")),
                     "kernel_ms": attn_ms, "algorithmic_flops": flops, "peak_source": f"{peak_src} bf16 burst",
                     "fp8_kv_gbs": abytes / (attn_ms / 1e3) / 1e9, "fp8_kv_frac_of_hbm": abytes / (attn_ms / 1e3) / 1e9 / hbm_peak},
        "cpu_baseline": cpu,
        "e2e": {"value": T * args.steps / (e2e_ms / 1e3), "unit": "query rows/s",
                "h2d_bytes_per_step": int(q.numel() * 2 + kv_new.numel() * 2),
                "d2h_bytes_per_step": int(sum(t.numel() * t.element_size() for t in h_out))},
        "gpu_launches": int(launches), "clocks": clocks,
    }


def _run_linear(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen, fp8_peak,
                peak_src, barrier):
    """Config 3.  N > 1 runs independent replicas (the projections have no exchange here)."""
    T = LINEAR_T
    ws = {}
    for name, n, k in LINEAR_PROJ:
        ws[name] = (_rand_e4m3(torch, (n, k), gen, device),
                    torch.rand(((n + 127) // 128, k // 128), generator=gen, device=device) * 1e-2)
    x = torch.randn((T, 7168), generator=gen, device=device).to(torch.bfloat16)
    attn = torch.randn((T, 128 * 128), generator=gen, device=device).to(torch.bfloat16)

    def lin(aq_sa, name):
        w, sw = ws[name]
        return hk.gemm_fp8(aq_sa[0], aq_sa[1], w, sw)

    def step(x_in, attn_in, ev=None):
        if ev is not None:
            ev[0].record(stream)
        xq = hk.quant_fp8(x_in)  # shared by q_a and kv_a
        qa = lin(xq, "q_a")
        qb = lin(hk.quant_fp8(qa), "q_b")
        kva = lin(xq, "kv_a")
        o = lin(hk.quant_fp8(attn_in), "o")
        if ev is not None:
            ev[1].record(stream)
        return qb, kva, o

    for _ in range(args.warmup):
        step(x, attn)
    torch.cuda.synchronize()
    hk.check_errors()
    flops = sum(2 * T * n * k for _, n, k in LINEAR_PROJ)
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    ms, lin_ms = _timed(torch, lambda ev: step(x, attn, ev), args.steps, stream)
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    hk.check_errors()
    ms, lin_ms = _reduce_max(torch, dist, world, device, ms, lin_ms)
    hx = torch.empty_like(x, device="cpu").pin_memory().copy_(x.cpu())
    ha = torch.empty_like(attn, device="cpu").pin_memory().copy_(attn.cpu())
    outs = [torch.empty((T, n), dtype=torch.bfloat16).pin_memory() for nm, n, _k in LINEAR_PROJ if nm != "q_a"]
    dx, da = torch.empty_like(x), torch.empty_like(attn)

    def e2e(ev):
        dx.copy_(hx, non_blocking=True)
        da.copy_(ha, non_blocking=True)
        for h, d in zip(outs, step(dx, da)):
            h.copy_(d, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _linear_cpu_baseline(x, attn, ws)
    tflops = flops / (lin_ms / 1e3) / 1e12
    return {
        "metric": "MLA FP8 projection tokens/s (config 3)", "value": T * world * args.steps / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32", "data": "synthetic (seeded)",
        "config": {"workload": "config3: 4144 tokens (48 decode + 2 x 2048 prefill), projections "
                               "q_a 7168->1536, q_b 1536->24576, kv_a 7168->576, o 16384->7168, "
                               "activation quantisation included",
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "weights 60 MB and activations re-read from L2; no flush (tensor-bound)"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": tflops / fp8_peak, "traffic": None, "kernel": "hk_gemm_fp8 (+ hk_quant_fp8)",
                     "kernel_ms": lin_ms, "algorithmic_flops": flops,
                     "peak_source": f"{peak_src}: 2 x cuBLAS bf16 burst (dense FP8 = 2 x bf16)"},
        "cpu_baseline": cpu,
        "e2e": {"value": T * world * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": x.numel() * 2 + attn.numel() * 2,
                "d2h_bytes_per_step": T * sum(n for nm, n, _ in LINEAR_PROJ if nm != "q_a") * 2},
        "gpu_launches": int(launches), "clocks": clocks,
    }


# The decode step's dense projections at a decode batch (64 rows: one per lane of config 2), in
# their absorbed-MLA shapes, plus the vocabulary projection: (name, out features, in features).
DECODE_PROJ = [("q_a", 1536, 7168), ("kv_a", 576, 7168), ("q_b", 128 * 576, 1536), ("o", 7168, 128 * 512),
               ("vocab", 129280, 7168)]


def _run_linear_decode(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
                       peak_src, barrier):
    """--workload linear-decode: the FP8 projections of a decode step for 64 token rows (the
    swap-AB kernel: weights on the MMA's M side, split K for the long-K o projection).  At 64 rows
    a projection does 128 flops per weight byte, far below the FP8 ridge, so the bound is HBM:
    `value` is weight bytes streamed per second.  N > 1: independent replicas."""
    T = 64
    ws = {name: (_rand_e4m3(torch, (n, k), gen, device),
                 torch.rand(((n + 127) // 128, k // 128), generator=gen, device=device) * 1e-2)
          for name, n, k in DECODE_PROJ}
    xs = {name: hk.quant_fp8(torch.randn((T, k), generator=gen, device=device).to(torch.bfloat16))
          for name, _n, k in DECODE_PROJ}
    outs = {name: torch.empty((T, n), dtype=torch.bfloat16, device=device) for name, n, _k in DECODE_PROJ}
    wbytes = {name: n * k for name, n, k in DECODE_PROJ}
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(DECODE_PROJ) + 1)] for _ in range(args.steps)]

    def step(ev=None):
        for j, (name, _n, _k) in enumerate(DECODE_PROJ):
            if ev is not None:
                ev[j].record(stream)
            w, sw = ws[name]
            hk.gemm_fp8(xs[name][0], xs[name][1], w, sw, out=outs[name])
        if ev is not None:
            ev[len(DECODE_PROJ)].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    hk.check_errors()
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        step(evs[i])
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    hk.check_errors()
    ms = start.elapsed_time(end)
    per = [float(np.mean([e[j].elapsed_time(e[j + 1]) for e in evs])) for j in range(len(DECODE_PROJ))]
    vals = _reduce_max(torch, dist, world, device, ms, *per)
    ms, per = vals[0], list(vals[1:])
    total_bytes = sum(wbytes.values())
    gbs = total_bytes / (ms / args.steps) / 1e6
    parts = {name: {"us": per[j] * 1e3, "weight_mb": wbytes[name] / 1e6, "gbs": wbytes[name] / per[j] / 1e6,
                    "frac_of_hbm": wbytes[name] / per[j] / 1e6 / hbm_peak}
             for j, (name, _n, _k) in enumerate(DECODE_PROJ)}
    return {
        "metric": "decode-batch FP8 projection weight GB/s (64 token rows)", "value": gbs * world,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 x e4m3 -> f32", "data": "synthetic (seeded)",
        "config": {"workload": "64 token rows through q_a 7168->1536, kv_a 7168->576, q_b 1536->128x576, "
                               "o 128x512->7168, vocabulary 7168->129280 (1.53 GB of e4m3 weights per step)",
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "1.5 GB of weights per step, larger than L2; no flush", "parts": parts},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "kernel": "gemm_fp8_swapab_kernel (hk_gemm_fp8, m = 64)",
                     "kernel_ms": ms / args.steps, "algorithmic_bytes": total_bytes, "peak_source": peak_src},
        "cpu_baseline": None, "e2e": None, "gpu_launches": int(launches), "clocks": sampler.summary(t0, t1),
    }


def _run_mixed(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
               peak_src, barrier):
    """Configuration 3's attention: 48 decode lanes (contexts U[2K, 32K], one new row each)
    and two chunked-prefill segments of 2048 rows (a prompt's first chunk and its second,
    after 2048 cached rows) in one token stream: pack, append every new latent row, then the
    tcgen05 MLA kernel with causal rows.  N > 1: independent replicas."""
    from hyperkernel_b200 import workload as W

    lay = W.config3_attn_layout(seed=0)
    T, H = lay.num_tokens, HEADS
    cache = torch.randn((lay.num_slots, DK), generator=gen, device=device).to(torch.bfloat16)
    q = torch.randn((T, H, DK), generator=gen, device=device).to(torch.bfloat16)
    kv_new = torch.randn((T, DK), generator=gen, device=device).to(torch.bfloat16)
    lane_tokens = torch.from_numpy(lay.new_rows.astype(np.int32)).to(device)
    lane_pos = torch.from_numpy(lay.context.astype(np.int32)).to(device)
    bt = torch.from_numpy(lay.block_table).to(device)
    max_kv = int(lay.kv_len.max())
    scale = 1.0 / math.sqrt(DK)
    ws = torch.empty(max(hk.mla_workspace_size(lay.lanes, T, H, max_kv), 16), dtype=torch.uint8, device=device)
    out = torch.empty((T, H, DV), dtype=torch.bfloat16, device=device)
    lse = torch.empty((T, H), dtype=torch.float32, device=device)

    def step(ev=None, q_in=None, kv_in=None):
        pk = hk.pack(lane_tokens, lane_pos, bt, PAGE, lay.num_pages, T)
        hk.kv_append_bf16(kv_new if kv_in is None else kv_in, pk["slot_mapping"], cache)
        if ev is not None:
            ev[0].record(stream)
        hk.mla_decode(q if q_in is None else q_in, cache, bt, pk["cu_seqlens"], pk["positions"], PAGE, max_kv,
                      scale, out=out, lse=lse, workspace=ws)
        if ev is not None:
            ev[1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    hk.check_errors()
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    ms, attn_ms = _timed(torch, step, args.steps, stream)
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    hk.check_errors()
    ms, attn_ms = _reduce_max(torch, dist, world, device, ms, attn_ms)
    # end to end: queries and new latent rows in from pinned host memory, outputs and LSE back
    hq = torch.empty(q.shape, dtype=q.dtype).pin_memory().copy_(q.cpu())
    hkv = torch.empty(kv_new.shape, dtype=kv_new.dtype).pin_memory().copy_(kv_new.cpu())
    dq, dkv = torch.empty_like(q), torch.empty_like(kv_new)
    ho = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    hl = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()

    def e2e(ev):
        dq.copy_(hq, non_blocking=True)
        dkv.copy_(hkv, non_blocking=True)
        step(None, dq, dkv)
        ho.copy_(out, non_blocking=True)
        hl.copy_(lse, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    rows_kv = _query_kv_pairs(lay)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the first three decode lanes, scaled by query-KV pairs
        ctx3 = [int(c) for c in lay.context[:3]]
        c_dt, c_pairs, c_threads = cpu_lanes_seconds(ctx3, [1, 1, 1])
        cpu = {"value": T / (c_dt * rows_kv / c_pairs), "unit": "tokens/s", "cores": c_threads, "kind": "port",
               "sample": f"pack + append + attention of three decode lanes ({sum(ctx3)} cached rows, 128 heads), "
                         "scaled by query-KV pairs"}
    flops = 2 * H * (DK + DV) * rows_kv
    abytes = int(lay.kv_len.sum()) * DK * 2 + T * H * (DK * 2 + DV * 2 + 4)
    bf16_peak = _peaks()[1] / 2.0
    tflops = flops / (attn_ms / 1e3) / 1e12
    return {
        "metric": "mixed prefill + decode attention tokens/s (config 3)", "value": T * world * args.steps / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "config3 attention: 48 decode lanes U[2K,32K] + 2 chunked-prefill segments of 2048 "
                               "rows (after 0 and 2048 cached rows), 4144 rows, 128 heads, MLA 512+64, causal",
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "kv_rows": int(lay.kv_len.sum()), "query_kv_pairs": rows_kv,
                   "l2": "the prefill rows re-read their prefixes from L2; no flush (tensor-bound)"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": tflops / bf16_peak, "traffic": None, "kernel": "tcgen05 attention (hk_mla_decode)",
                     "kernel_ms": attn_ms, "algorithmic_flops": flops, "algorithmic_bytes": abytes,
                     "peak_source": f"{peak_src} bf16 burst"},
        "cpu_baseline": cpu,
        "e2e": {"value": T * world * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(q.numel() * 2 + kv_new.numel() * 2),
                "d2h_bytes_per_step": int(out.numel() * 2 + lse.numel() * 4)},
        "gpu_launches": int(launches), "clocks": clocks,
    }


def _run_step(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
              peak_src, barrier):
    """--workload step: the four parts of the decode step on one token stream, configuration 3's
    mixed batch (48 decode lanes at U[2K, 32K] + two 2048-row chunked-prefill segments, 4144 rows)
    through one DeepSeek-V3-shaped layer in its absorbed MLA form: the FP8 q_a / kv_a / q_b
    projections, the latent rows appended to the paged cache, tcgen05 MLA attention (causal
    prefill rows), the FP8 o projection, then configuration 4's MoE layer on the same 4144 tokens
    (router GEMM, sigmoid top-8 of 256 experts, permutation, grouped FP8 expert FFN, the shared
    expert, combine).  Every part is timed with CUDA events on the launching stream; the line
    gives the step's tokens/s and each part's share and roofline.  N > 1: independent replicas."""
    from hyperkernel_b200 import workload as W

    # --step-batch decode: configuration 2's 64 decode lanes (one row each, contexts log-uniform
    # in [1K, 128K]) through the same layer: the decode-sized step
    lay = W.config2_layout(seed=0) if args.step_batch == "decode" else W.config3_attn_layout(seed=0)
    T, Hh = lay.num_tokens, HEADS
    HID, QL, E, K, I = 7168, 1536, args.experts or MOE_E, MOE_K, MOE_I
    projs = {"q_a": (QL, HID), "kv_a": (DK, HID), "q_b": (Hh * DK, QL), "o": (HID, Hh * DV), "router": (E, HID)}
    ws = {n: (_rand_e4m3(torch, (a, b), gen, device),
              torch.rand(((a + 127) // 128, b // 128), generator=gen, device=device) * 2e-4 + 1e-4)
          for n, (a, b) in projs.items()}
    w13 = _rand_e4m3(torch, (E + 1, 2 * I, HID), gen, device)
    w2 = _rand_e4m3(torch, (E + 1, HID, I), gen, device)
    s13 = torch.rand((E + 1, 2 * I // 128, HID // 128), generator=gen, device=device) * 1e-3
    s2 = torch.rand((E + 1, HID // 128, I // 128), generator=gen, device=device) * 1e-3
    cache = torch.randn((lay.num_slots, DK), generator=gen, device=device).to(torch.bfloat16)
    x = torch.randn((T, HID), generator=gen, device=device).to(torch.bfloat16)
    lane_tokens = torch.from_numpy(lay.new_rows.astype(np.int32)).to(device)
    lane_pos = torch.from_numpy(lay.context.astype(np.int32)).to(device)
    bt = torch.from_numpy(lay.block_table).to(device)
    max_kv = int(lay.kv_len.max())
    scale = 1.0 / math.sqrt(DK)
    attn_ws = torch.empty(max(hk.mla_workspace_size(lay.lanes, T, Hh, max_kv), 16), dtype=torch.uint8, device=device)
    o = torch.empty((T, Hh, DV), dtype=torch.bfloat16, device=device)
    lse = torch.empty((T, Hh), dtype=torch.float32, device=device)
    # the shared expert runs as expert E of the routed grouped call (its weights follow the routed
    # ones), as the model step behind hk_open_mla runs it: rows [T*K, T*K + T) are every token
    moe_ws = torch.empty(hk.moe_workspace_size(T * (K + 1), HID, I), dtype=torch.uint8, device=device)
    ym = torch.empty((T * (K + 1), HID), dtype=torch.bfloat16, device=device)
    off_ext = torch.empty(E + 2, dtype=torch.int32, device=device)
    off_ext[E + 1] = T * (K + 1)
    tok_ext = torch.empty(T * (K + 1), dtype=torch.int32, device=device)
    tok_ext[T * K:] = torch.arange(T, dtype=torch.int32, device=device)
    parts = ["projections in (q_a, kv_a, q_b)", "KV append", "attention", "o projection", "MoE layer"]

    def lin(aq, name):
        w, sw = ws[name]
        return hk.gemm_fp8(aq[0], aq[1], w, sw)

    def step(ev=None, x_in=None):
        xx = x if x_in is None else x_in
        mark = (lambda i: ev[i].record(stream)) if ev is not None else (lambda i: None)
        mark(0)
        xq = hk.quant_fp8(xx)
        qa = lin(xq, "q_a")
        kv = lin(xq, "kv_a")
        q = lin(hk.quant_fp8(qa), "q_b")
        mark(1)
        pk = hk.pack(lane_tokens, lane_pos, bt, PAGE, lay.num_pages, T)
        hk.kv_append_bf16(kv, pk["slot_mapping"], cache)
        mark(2)
        hk.mla_decode(q.view(T, Hh, DK), cache, bt, pk["cu_seqlens"], pk["positions"], PAGE, max_kv, scale, out=o,
                      lse=lse, workspace=attn_ws)
        mark(3)
        y = lin(hk.quant_fp8(o.view(T, Hh * DV)), "o")
        mark(4)
        hq, hs = hk.quant_fp8(y)
        logits = lin((hq, hs), "router").float()
        ids, wt = hk.route(logits, None, K, 2.5)
        off, tok, pw, inv = hk.permute(ids, wt, E, offsets=off_ext[:E + 1], perm_token=tok_ext[:T * K])
        hk.moe_grouped(hq, hs, off_ext, tok_ext, T * (K + 1), HID, I, w13, s13, w2, s2, out=ym, workspace=moe_ws)
        out = hk.combine(ym[:T * K], pw, inv, ym[T * K:], T, K)
        mark(5)
        return out, off

    for _ in range(args.warmup):
        _, off = step()
    torch.cuda.synchronize()
    hk.check_errors()
    counts = (off[1:] - off[:-1]).cpu().numpy()
    hit = int((counts > 0).sum())
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        step(evs[i])
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    hk.check_errors()
    ms = start.elapsed_time(end)
    part_ms = [float(np.mean([e[j].elapsed_time(e[j + 1]) for e in evs])) for j in range(5)]
    vals = _reduce_max(torch, dist, world, device, ms, *part_ms)
    ms, part_ms = vals[0], list(vals[1:])
    hx = torch.empty(x.shape, dtype=x.dtype).pin_memory().copy_(x.cpu())
    hout = torch.empty((T, HID), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(x)

    def e2e(ev):
        dx.copy_(hx, non_blocking=True)
        out, _ = step(None, dx)
        hout.copy_(out, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    hbm, fp8_peak, _ = _peaks()
    bf16_peak = fp8_peak / 2
    proj_in_flops = 2 * T * (QL * HID + DK * HID + Hh * DK * QL)
    attn_flops = 2 * Hh * (DK + DV) * _query_kv_pairs(lay)
    o_flops = 2 * T * HID * Hh * DV
    wbytes = (hit + 1) * 3 * HID * I + E * HID
    moe_bytes = wbytes + T * (K + 1) * (HID + 2 * 2 * I + 2 * HID)
    kv_bytes = T * DK * 2 * 2
    moe_flops = 2 * T * (K + 1) * 3 * HID * I + 2 * T * E * HID
    step_ms = ms / args.steps
    shares = {
        parts[0]: {"ms": part_ms[0], "share": part_ms[0] / step_ms, "tflops": proj_in_flops / part_ms[0] / 1e9,
                   "frac_of_fp8_peak": proj_in_flops / part_ms[0] / 1e9 / fp8_peak},
        parts[1]: {"ms": part_ms[1], "share": part_ms[1] / step_ms, "gbs": kv_bytes / part_ms[1] / 1e6,
                   "note": "includes hk_pack"},
        parts[2]: {"ms": part_ms[2], "share": part_ms[2] / step_ms, "tflops": attn_flops / part_ms[2] / 1e9,
                   "frac_of_bf16_peak": attn_flops / part_ms[2] / 1e9 / bf16_peak},
        parts[3]: {"ms": part_ms[3], "share": part_ms[3] / step_ms, "tflops": o_flops / part_ms[3] / 1e9,
                   "frac_of_fp8_peak": o_flops / part_ms[3] / 1e9 / fp8_peak},
        parts[4]: {"ms": part_ms[4], "share": part_ms[4] / step_ms, "gbs": moe_bytes / part_ms[4] / 1e6,
                   "frac_of_hbm": moe_bytes / part_ms[4] / 1e6 / hbm, "experts_hit": hit,
                   "tflops": moe_flops / part_ms[4] / 1e9, "frac_of_fp8_peak": moe_flops / part_ms[4] / 1e9 / fp8_peak,
                   "note": f"{T} tokens x (8 routed + 1 shared) = {T * (K + 1)} expert rows"},
    }
    top = max(range(5), key=lambda j: part_ms[j])
    # the MoE part is HBM-bound at decode batches (64 rows: ~1 flop per weight byte per row) and
    # leans towards the tensor ridge at the 4144-row mixed batch; the dense parts are tensor work
    moe_bound = "tensor" if args.step_batch != "decode" else "hbm"
    top_bound = "tensor" if top in (0, 2, 3) or (top == 4 and moe_bound == "tensor") else "hbm"
    top_part = shares[parts[top]]
    if top_bound == "hbm":
        top_ach, top_peak, top_unit = top_part["gbs"], hbm, "GB/s"
    else:
        top_ach = top_part["tflops"]
        top_peak, top_unit = (bf16_peak if top == 2 else fp8_peak), "TFLOP/s"
    return {
        "metric": "decode step tokens/s, one layer (" + ("config 2" if args.step_batch == "decode" else "config 3") +
                  " batch through projections, attention and MoE)",
        "value": T * world * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 projections and experts, bf16 attention, fp32 accumulation",
        "data": "synthetic (seeded)",
        "config": {"workload": (("config3 batch (48 decode lanes U[2K,32K] + 2 x 2048 prefill rows, 4144 tokens)"
                                 if args.step_batch != "decode" else
                                 "config2 batch (64 decode lanes, ctx log-uniform [1K,128K], 64 tokens)") +
                                " through one DeepSeek-V3-shaped layer, absorbed MLA (q_b 1536->128x576, "
                                "o 128x512->7168), then config 4's MoE (256 experts top-8 + shared, inter 2048)"),
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "11.3 GB of expert weights and ~1 GB of KV per step, no flush", "parts": shares},
        "roofline": {"bound": top_bound, "achieved": top_ach, "peak": top_peak, "unit": top_unit,
                     "frac": top_ach / top_peak, "traffic": None,
                     "kernel": f"the step's largest part: {parts[top]}", "kernel_ms": part_ms[top],
                     "peak_source": peak_src},
        "cpu_baseline": None,
        "e2e": {"value": T * world * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x.numel() * 2), "d2h_bytes_per_step": int(T * HID * 2)},
        "gpu_launches": int(launches), "clocks": sampler.summary(t0, t1),
    }


SAMPLE_VOCAB = 129280
SAMPLE_LANES, SAMPLE_BLOCK, SAMPLE_LOGPROBS = 8, 5, 20
SAMPLE_MIX = [dict(temperature=0.0, top_k=0, top_p=1.0), dict(temperature=0.7, top_k=50, top_p=1.0),
              dict(temperature=1.0, top_k=0, top_p=0.9), dict(temperature=0.8, top_k=0, top_p=1.0)]


def _run_sample(args, torch, dist, hk, ClockSampler, world, rank, local, device, stream, gen, hbm_peak,
                peak_src, barrier):
    """Spec-decode verification with on-device sampling at config 5's shape: 8 lanes x (1 + 4)
    rows of fp32 logits over a 129,280-token vocabulary, 20 logprob pairs per token, lanes
    cycling greedy / top-k 50 / top-p 0.9 / plain temperature.  Drafts are each row's greedy
    token, so greedy lanes accept every draft.  N > 1: independent replicas."""
    V, L, B, n = SAMPLE_VOCAB, SAMPLE_LANES, SAMPLE_BLOCK, SAMPLE_LOGPROBS
    rows = L * B
    logits = torch.randn((rows, V), generator=gen, device=device) * 2.0
    cu = torch.arange(0, rows + 1, B, dtype=torch.int32, device=device)
    samplings = [SAMPLE_MIX[i % len(SAMPLE_MIX)] for i in range(L)]
    smp = hk.sampling_array(samplings, device)
    seeds = torch.arange(1, L + 1, dtype=torch.int64, device=device) * 7919
    state = seeds.clone()
    drafts = logits.view(L, B, V).argmax(dim=2)[:, :B - 1].to(torch.int32).contiguous()

    def step(ev=None, lg=None):
        if ev is not None:
            ev[0].record(stream)
        out = hk.sample_verify(logits if lg is None else lg, cu, smp, state, drafts, B, n, stream)
        if ev is not None:
            ev[1].record(stream)
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    hk.check_errors()
    sampler = ClockSampler(local).start()
    launches0 = hk.kernel_launches()
    barrier()
    t0 = time.perf_counter()
    ms, k_ms = _timed(torch, step, args.steps, stream)
    t1 = time.perf_counter()
    barrier()
    launches = hk.kernel_launches() - launches0
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    hk.check_errors()
    ms, k_ms = _reduce_max(torch, dist, world, device, ms, k_ms)
    h_logits = torch.empty((rows, V), dtype=torch.float32).pin_memory().copy_(logits.cpu())
    d_logits = torch.empty_like(logits)
    h_ids = torch.empty((L, B), dtype=torch.int32).pin_memory()
    h_lp = torch.empty((L, B, 2 * n + 1), dtype=torch.float32).pin_memory()

    def e2e(ev):
        d_logits.copy_(h_logits, non_blocking=True)
        ids, lp = step(None, d_logits)
        h_ids.copy_(ids, non_blocking=True)
        h_lp.copy_(lp, non_blocking=True)

    barrier()
    e2e_ms, _ = _timed(torch, e2e, args.steps, stream, inner=False)
    (e2e_ms,) = _reduce_max(torch, dist, world, device, e2e_ms)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _sample_cpu_baseline(logits, cu, samplings, seeds, drafts)
    abytes = rows * V * 4 + L * B * (4 + (2 * n + 1) * 4)
    gbs = abytes / (k_ms / 1e3) / 1e9
    return {
        "metric": "spec-verify rows/s with on-device sampling (config 5 shape)",
        "value": rows * world * args.steps / (ms / 1e3), "unit": "verify rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 logits, f64 probabilities", "data": "synthetic (seeded)",
        "config": {"workload": f"{L} lanes x {B} rows, vocab {V}, {n} logprobs; greedy / top-k 50 / top-p 0.9 / "
                               "temperature lanes; per-row bucket selection (no full sort)",
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": f"{rows * V * 4 / 1e6:.0f} MB of logits, L2-resident between steps (no flush)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "kernel": "hk_sample_verify (row selection + chain)", "kernel_ms": k_ms,
                     "algorithmic_bytes": abytes, "peak_source": peak_src},
        "cpu_baseline": cpu,
        "e2e": {"value": rows * world * args.steps / (e2e_ms / 1e3), "unit": "verify rows/s",
                "h2d_bytes_per_step": rows * V * 4, "d2h_bytes_per_step": L * B * (4 + (2 * n + 1) * 4)},
        "gpu_launches": int(launches), "clocks": clocks,
    }


# The decode step behind the Kernel boundary (HK_MODEL_MLA): one DeepSeek-V3-shaped layer.
ENGINE_LANES, ENGINE_PAGE_ROWS, ENGINE_CHUNK, ENGINE_BLOCK = 64, 64, 512, 1
ENGINE_REQUESTS, ENGINE_LIMIT, ENGINE_PROMPT = 128, 64, (64, 1024)
ENGINE_BUDGET = 8192  # prefill tokens a step: the reference's tuned pacing presets (src/model/cli.rs)
ENGINE_ENTRIES = (ENGINE_PROMPT[1] + ENGINE_LIMIT + ENGINE_PAGE_ROWS - 1) // ENGINE_PAGE_ROWS + 1
ENGINE_DIMS = dict(hidden=7168, q_lora=1536, vocab=129280, experts=256, top_k=8, inter=2048, layers=1,
                   logprobs=20, seed=1234, rope_theta=10000.0, route_scale=2.5)


def _engine_requests(n, seed, vocab=ENGINE_DIMS["vocab"]):
    """Seeded prompts of U[64, 1024) token ids over the model's vocabulary."""
    rng = np.random.default_rng(seed)
    return [(rng.integers(0, vocab, int(rng.integers(*ENGINE_PROMPT))).tolist(), ENGINE_LIMIT) for _ in range(n)]


def _engine_device(H, device_index, dims):
    context = ENGINE_PAGE_ROWS * ENGINE_ENTRIES
    pages = ENGINE_LANES * ENGINE_ENTRIES + 1
    cfg = H.Config(model=H.MODEL_MLA, page_rows=ENGINE_PAGE_ROWS, entries=ENGINE_ENTRIES, window=ENGINE_ENTRIES,
                   width=ENGINE_LANES, context=context, chunk=ENGINE_CHUNK, block=ENGINE_BLOCK, pages=pages,
                   window_pages=pages, clip=0, device=device_index, transport=0)
    return H.Device(cfg, H.MlaModel(**dims))


def _engine_session(H, dev, requests, logprobs):
    """One session of the C++ engine over the device: every request submitted (greedy, with
    `logprobs` pairs per token), the jobs closed, hk_engine_run to the end.  Returns (seconds,
    engine iterations with tokens, generated tokens, prompt tokens)."""
    context = ENGINE_PAGE_ROWS * ENGINE_ENTRIES
    eng = H.Engine(H.engine_config(page_rows=ENGINE_PAGE_ROWS, entries=ENGINE_ENTRIES, window=ENGINE_ENTRIES,
                                   window_keep=0, context=context, width=ENGINE_LANES, chunk=ENGINE_CHUNK,
                                   block=ENGINE_BLOCK, pad=0, budget=ENGINE_BUDGET, every=1, headroom=2048),
                   dev.ops(), keep=dev)
    samp = H.Sampling(0.0, 1.0, 0, logprobs, 0)
    reqs = [eng.submit(pr, lim, sampling=samp) for pr, lim in requests]
    eng.close()
    t0 = time.perf_counter()
    rc = eng.run()
    dt = time.perf_counter() - t0
    if rc != 0:
        raise RuntimeError(f"engine run failed: {eng.failure}")
    m, _acc, counts, _total = eng.metrics()
    tokens = sum(len(eng.heard(r).tokens) for r in reqs)
    return dt, int(sum(counts)), tokens, int(m["prompt_tokens"])


def leg_engine(args, torch, dist, hk, world, rank, local, device, barrier, hbm_peak):
    """The whole decode step behind the reference's Kernel boundary: the C++ engine (admission,
    prefix cache, block tables, prompt chunking, pacing) driving an HK_MODEL_MLA device through
    hk_kernel_ops -- hk_push / hk_drain with host arrays in and sampled ids and logprob rows out
    -- each step packing the live lanes, embedding, one DeepSeek-V3-shaped layer (FP8 q_a / q_b /
    kv_a projections, RoPE, KV append, tcgen05 MLA attention over the paged latent cache, FP8 o
    projection, sigmoid top-8 routing over 256 experts + the shared one, grouped FP8 expert FFN,
    combine), the FP8 vocabulary projection and on-device sampling.  128 requests, prompts
    U[64, 1024), 64 tokens each, 64 lanes.  Host-driven loop: timed by the host clock around
    hk_engine_run; end to end by construction.  N > 1: independent replicas."""
    from hyperkernel_b200 import engine as H

    dims = dict(ENGINE_DIMS)
    # an engine's step clock starts at 0, so every session gets a freshly opened device
    for _ in range(max(1, min(args.warmup, 2))):
        dev = _engine_device(H, local, dims)
        try:
            _engine_session(H, dev, _engine_requests(8, 5), dims["logprobs"])
        finally:
            dev.close()
    requests = _engine_requests(args.engine_requests or ENGINE_REQUESTS, 11 + rank)
    l0 = hk.kernel_launches()
    dev = _engine_device(H, local, dims)
    try:
        barrier()
        l1 = hk.kernel_launches()
        dt, iters, tokens, prompt_tokens = _engine_session(H, dev, requests, dims["logprobs"])
        launches = hk.kernel_launches() - l1
        barrier()
    finally:
        dev.close()
    (dt_ms,) = _reduce_max(torch, dist, world, device, dt * 1e3)
    dt = dt_ms / 1e3
    # HBM bytes of one decode step's weights (every routed expert a 64-row step hits, in
    # expectation, plus the shared expert and the dense projections, embedding rows aside)
    H_, QL, E, K, I, V = (dims[k] for k in ("hidden", "q_lora", "experts", "top_k", "inter", "vocab"))
    hit = E * (1 - (1 - 1 / E) ** (ENGINE_LANES * K))
    wbytes = (hit + 1) * 3 * H_ * I + QL * H_ + 128 * 576 * QL + 576 * H_ + H_ * 128 * 512 + E * H_ + V * H_
    return {
        "workload": f"HK_MODEL_MLA behind hk_push/hk_drain driven by hk_engine_run: {len(requests)} requests, "
                    f"prompts U[{ENGINE_PROMPT[0]},{ENGINE_PROMPT[1]}), {ENGINE_LIMIT} tokens each, {ENGINE_LANES} "
                    f"lanes, prefill budget {ENGINE_BUDGET} tokens a step in chunks of {ENGINE_CHUNK}, "
                    "1 DeepSeek-V3-shaped layer (hidden 7168, MLA 128 heads 512+64, FP8 projections, 256+1 "
                    "experts top-8, inter 2048), vocabulary 129280, greedy with 20 logprob pairs per token",
        "parallelism": f"replicas{world}" if world > 1 else "single GPU",
        "timing": "host clock around hk_engine_run, max over ranks (host-driven loop; commands and ids cross "
                  "the boundary every step)",
        "tokens_per_s": tokens * world / dt, "prompt_tokens_per_s": prompt_tokens * world / dt,
        "seconds": dt, "iterations": iters, "ms_per_iteration": dt * 1e3 / max(iters, 1),
        "generated_tokens": tokens * world, "prompt_tokens": prompt_tokens * world,
        "decode_step_weight_bytes": int(wbytes), "gpu_launches": int(launches),
        "gpu_launches_with_open": int(hk.kernel_launches() - l0),
    }


def _run_engine(args, torch, dist, hk, ClockSampler, world, rank, local, device, barrier, hbm_peak, peak_src):
    """--workload engine: leg_engine as its own line."""
    sampler = ClockSampler(local).start()
    t0 = time.perf_counter()
    leg = leg_engine(args, torch, dist, hk, world, rank, local, device, barrier, hbm_peak)
    t1 = time.perf_counter()
    sampler.stop()
    per_step = leg["ms_per_iteration"] / 1e3
    gbs = leg["decode_step_weight_bytes"] / per_step / 1e9 if per_step > 0 else 0.0
    return {
        "metric": "engine tokens/s through the Kernel boundary (HK_MODEL_MLA, 64 lanes)",
        "value": leg["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": leg["iterations"],
        "warmup": max(1, min(args.warmup, 2)), "ms_per_step": leg["ms_per_iteration"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32, bf16 activations",
        "data": "synthetic (seeded prompts, seeded random weights)", "config": {"workload": leg["workload"],
                                                                               "timing": leg["timing"]},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "kernel": "whole engine iteration (decode-step weights / iteration time)",
                     "peak_source": peak_src,
                     "note": "iterations mix decode steps and prompt chunks; the weights a decode step streams "
                             "bound it from below"},
        "cpu_baseline": None,
        "e2e": {"value": leg["tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": None,
                "d2h_bytes_per_step": None,
                "note": "end to end: hk_push copies each share's host arrays, hk_drain returns host ids and "
                        "logprob lists"},
        "gpu_launches": leg["gpu_launches"], "clocks": sampler.summary(t0, t1), "engine": leg,
    }


def _sample_cpu_baseline(logits, cu, samplings, seeds, drafts, sample_lanes=4):
    """The oracle's verify step for the first `sample_lanes` lanes (one per sampling kind),
    scaled to all lanes."""
    from oracle import sample as S

    lg = logits.cpu().numpy()
    cun = cu.cpu().numpy()[:sample_lanes + 1]
    st = seeds.cpu().numpy().view(np.uint64).tolist()[:sample_lanes]
    dr = drafts.cpu().numpy()[:sample_lanes]
    t0 = time.perf_counter()
    S.sample_verify(lg[:cun[-1]], cun, samplings[:sample_lanes], st, dr, SAMPLE_BLOCK, SAMPLE_LOGPROBS)
    dt = time.perf_counter() - t0
    rows = int(cun[-1])
    return {"value": rows / dt, "unit": "verify rows/s", "cores": 1, "kind": "port",
            "sample": f"{sample_lanes} of {SAMPLE_LANES} lanes ({rows} rows), numpy restatement, one step"}


def _moe_cpu_baseline(x, logits, w13, s13, w2, s2, sh13, shs13, sh2, shs2, sample_experts=6):
    """The oracle's layer on the host cores: quantise, route and permute all 512 tokens, then
    the grouped FFN of the first `sample_experts` hit experts, scaled to all rows (the FFN is
    linear in rows) plus the shared expert scaled likewise."""
    import oracle

    oracle.use_all_cores()

    xb = x.view(torch_int16()).cpu().numpy().view(np.uint16)
    lg = logits.cpu().numpy()
    t0 = time.perf_counter()
    xq, sx = oracle.quant_fp8(xb)
    ids, w = oracle.route(lg, None, MOE_K, 1.0)
    off, tok, pw, inv = oracle.permute(ids, w, MOE_E)
    t_route = time.perf_counter() - t0
    hit = [e for e in range(MOE_E) if off[e + 1] > off[e]][:sample_experts]
    rows_sample = 0
    t_ffn = 0.0
    for e in hit:
        r0, r1 = int(off[e]), int(off[e + 1])
        sub_off = np.array([0, r1 - r0], np.int32)
        a13, b13 = w13[e:e + 1].cpu().numpy(), s13[e:e + 1].cpu().numpy()
        a2, b2 = w2[e:e + 1].cpu().numpy(), s2[e:e + 1].cpu().numpy()
        t0 = time.perf_counter()
        oracle.moe_grouped(xq, sx, sub_off, tok[r0:r1], MOE_H, MOE_I, a13, b13, a2, b2)
        t_ffn += time.perf_counter() - t0
        rows_sample += r1 - r0
    per_row = t_ffn / max(rows_sample, 1)
    total = t_route + per_row * (MOE_T * MOE_K + MOE_T)
    threads = os.cpu_count() or 1
    return {"value": MOE_T / total, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"route+permute of all 512 tokens, grouped FFN of {len(hit)} experts ({rows_sample} rows) "
                      f"scaled per row to {MOE_T * MOE_K} routed + {MOE_T} shared rows"}


def _linear_cpu_baseline(x, attn, ws, sample_tokens=8):
    """The oracle's FP8 projections on the host cores for `sample_tokens` tokens, scaled."""
    import oracle

    oracle.use_all_cores()

    xb = x[:sample_tokens].view(torch_int16()).cpu().numpy().view(np.uint16)
    ab = attn[:sample_tokens].view(torch_int16()).cpu().numpy().view(np.uint16)
    wt = {k: (w.cpu().numpy(), s.cpu().numpy()) for k, (w, s) in ws.items()}
    t0 = time.perf_counter()
    for name, src in (("q_a", xb), ("kv_a", xb), ("o", ab)):
        aq, sa = oracle.quant_fp8(src)
        oracle.gemm_fp8(aq, sa, *wt[name])
    aq, sa = oracle.quant_fp8(np.zeros((sample_tokens, 1536), np.uint16))
    oracle.gemm_fp8(aq, sa, *wt["q_b"])
    dt = time.perf_counter() - t0
    return {"value": sample_tokens / dt, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"the four projections for {sample_tokens} of the {LINEAR_T} tokens"}


def torch_int16():
    import torch
    return torch.int16


if __name__ == "__main__":
    sys.exit(main())

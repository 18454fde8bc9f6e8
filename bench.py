#!/usr/bin/env python
"""Benchmark of the paged decode path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                  [--impl ours|reference] [--cpu-baseline-seconds S]

A step is one decode-attention pass over one batch of the workload (for
``tp70b``: decode of the rank's KV heads -> o_proj partial -> NCCL all-reduce).

Workloads: ``gqa_b16`` (default, config 2), ``mha_b1``
(config 1), ``gqa_long`` (config 3), ``tp70b`` (config 4).  At N > 1 the
replicated workloads shard whole sequences across ranks (every rank decodes
its own batch, no collective, "scaling": "weak"); ``tp70b`` shards KV heads
and all-reduces the fp16 o_proj partials over NCCL ("scaling": "strong").

value      tokens/s of the whole job with inputs resident in HBM, the steps
           replayed from CUDA graphs, timed with CUDA events (max over ranks);
           several input sets rotate so each step reads more than the 126 MB L2.
e2e        the same metric through the public API (torch.ops.b200kv.*) with
           pinned host buffers: every step copies q, the new K/V rows, slots,
           block table and lengths host->device, appends the new token,
           decodes, and copies the output back.
roofline   achieved = algorithmic bytes per launch / mean CUDA-event duration
           of the decode kernel; peak = measured HBM copy bandwidth
           (MEASURED_PEAKS.json); traffic = DRAM bytes per launch from the
           committed ncu summary of this kernel and workload, if present.
cpu_baseline  the oracle (reference CPU eager path: paged gather + torch CPU
           SDPA in fp32) on the host cores, bounded sample.
--impl reference  times that CPU path alone on the same config (rank 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tokens/s (KV-stream HBM GB/s and % of peak in roofline)"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2**20


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=None)
    p.add_argument("--workload", default="gqa_b16",
                   choices=["gqa_b16", "mha_b1", "gqa_long", "tp70b", "relayout"])
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--cpu-baseline-seconds", type=float, default=10.0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--kv-dtype", default="fp16", choices=["fp16", "fp8"],
                   help="KV page element type: fp16 (the reference's) or e4m3 pages with per-pool fp16 scales")
    p.add_argument("--allreduce", default="peer", choices=["peer", "fused", "nccl"],
                   help="tp70b at N > 1: the o_proj all-reduce as libb200kv's peer-memory kernel, the fused "
                        "o_proj GEMM + all-reduce kernel, or NCCL")
    p.add_argument("--nccl-graph", action="store_true",
                   help="tp70b at N > 1: capture the step, NCCL all-reduce included, in a CUDA graph")
    p.add_argument("--no-tp", action="store_true",
                   help="skip the head-sharded tp70b block that every decode workload's line carries")
    p.add_argument("--no-early-start", action="store_true",
                   help="launch every decode without B200KV_DECODE_INPUTS_READY")
    p.add_argument("--kv-shards", type=int, default=1,
                   help="tp70b on one GPU: run the share one rank of an N-way head split holds (8 / N KV heads)")
    p.add_argument("--profile-launches", type=int, default=0,
                   help="run K eager decode launches of input set 0 and print its algorithmic bytes (for a "
                        "profiler capture of one launch; no timing)")
    return p.parse_args()


# decode steps per captured CUDA graph (the headline loop) and per captured
# e2e pipeline graph: a graph replay starts without programmatic early start
# and, in the e2e pipeline, with an upload wait and ends with a download
GRAPH_STEPS = 32
E2E_GRAPH_STEPS = 64
DEFAULT_STEPS = {"gqa_b16": 20000, "mha_b1": 20000, "gqa_long": 4000, "tp70b": 2000, "relayout": 2000}


# ----------------------------------------------------------- distributed ----
def dist_setup(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ peaks ----
def hbm_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(kernel: str, workload: str, bytes_per_launch: float):
    """(DRAM bytes per launch, where they come from) for this kernel and
    workload: ncu's dram__bytes_read.sum + dram__bytes_write.sum of one
    captured launch, from the machine-readable summary
    profiles/<kernel>_<workload>.json, scaled from that launch's algorithmic
    bytes to this run's.  (None, None) if no capture exists."""
    p = REPO / "profiles" / f"{kernel}_{workload}.json"
    if not p.exists():
        return None, None
    d = json.loads(p.read_text())
    ratio = (d["dram__bytes_read.sum"] + d["dram__bytes_write.sum"]) / d["algorithmic_bytes"]
    return round(ratio * bytes_per_launch), (
        f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch = {ratio:.4f} x its algorithmic bytes "
        f"(profiles/{p.name}), times this run's algorithmic bytes per launch")


# ------------------------------------------------------------- CPU oracle ----
def cpu_oracle_rate(inp, budget_s: float, max_steps: int | None = None):
    """Sequences/s of the oracle on a bounded sample (whole sequences, cycling)."""
    from oracle import paged_attention as opa

    torch.set_num_threads(os.cpu_count() or 1)
    cpu = {k: getattr(inp, k).cpu() for k in ("q", "k_pool", "v_pool", "block_table", "context_lens")}
    if inp.k_scale is not None:  # fp8 pages: the CPU path runs on the dequantized cache
        from oracle import fp8_quant as o8

        cpu["k_pool"] = o8.fp16_pool_from_pool(cpu["k_pool"], inp.k_scale.cpu())
        cpu["v_pool"] = o8.fp16_pool_from_pool(cpu["v_pool"], inp.v_scale.cpu())
    B = len(inp.ctx)
    done, t0, b = 0, time.perf_counter(), 0
    while True:
        sl = slice(b, b + 1)
        opa.decode_attention_cpu(cpu["q"][sl], cpu["k_pool"], cpu["v_pool"], cpu["block_table"][sl],
                                 cpu["context_lens"][sl])
        done += 1
        b = (b + 1) % B
        el = time.perf_counter() - t0
        if el >= budget_s or (max_steps and done >= max_steps):
            return done / el, done, el


# ---------------------------------------------------------------- config ----
def rotating_sets(kv_bytes_of_set0: float) -> int:
    """How many rotating input sets keep each step's reads out of L2."""
    n = max(1, math.ceil(3 * L2_BYTES / kv_bytes_of_set0)) if kv_bytes_of_set0 < 3 * L2_BYTES else 1
    return min(n, 32)


def set_tag(cfg, i: int, rank: int) -> str:
    """Seed tag of input set i on a rank.  The head-sharded tp70b step has
    the same sequences (context lengths, block tables) on every rank -- the
    ranks hold different heads of them -- so its sets do not depend on the
    rank; the replicated workloads give every rank its own batch."""
    return f"set{i}" if cfg.name == "tp70b" else f"set{i}/rank{rank}"


def workload_config(args, cfg, rank, world):
    """The `config` object of the JSON line, computed from the workload's
    seeded context lengths alone, so the repo arm and the reference arm print
    the same dictionary for the same run."""
    from torch_spyre_b200.workloads import context_lens_for

    tp = cfg.name == "tp70b"
    split = world * (args.kv_shards if tp else 1)
    hkv = cfg.num_kv_heads // split if tp else cfg.num_kv_heads
    elt = 1 if args.kv_dtype == "fp8" else 2

    def kv_bytes(i):
        return sum(context_lens_for(cfg, set_tag(cfg, i, rank))) * hkv * cfg.head_dim * 2 * elt

    n_sets = rotating_sets(kv_bytes(0))
    kv = statistics.mean(kv_bytes(i) for i in range(n_sets))
    B = len(context_lens_for(cfg, set_tag(cfg, 0, rank)))
    ar = tp and world > 1 and args.allreduce in ("peer", "fused")
    graphed = not (tp and world > 1) or args.nccl_graph or ar
    return {"workload": args.workload, "description": cfg.description, "batch_per_rank": B,
            "global_batch": B if tp else B * world, "num_q_heads": cfg.num_q_heads,
            "num_kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
            "kv_heads_per_rank": hkv, "kv_dtype": args.kv_dtype,
            "parallelism": ((f"tp{world} (kv-head shards + "
                             f"{'fused o_proj + peer-memory' if args.allreduce == 'fused' and ar else 'peer-memory' if ar else 'NCCL'}"
                             " all-reduce)") if tp and split == world
                            else f"one rank's share of tp{split} (no all-reduce)" if tp
                            else f"dp{world} (sequence shards)"),
            "l2": f"{n_sets} rotating input sets, {kv / 1e6:.1f} MB KV read per step (L2 126 MB)",
            "graphs": (f"up to {max(1, GRAPH_STEPS // n_sets) * n_sets} steps per graph replay" if graphed
                       else "eager (NCCL step)"),
            "decode_launch": ("B200KV_DECODE_INPUTS_READY (inputs written before the previous step)"
                              if not args.no_early_start else "default")}


def profile_key(args) -> str:
    """Workload name of the profile summaries: tp70b shares carry their split."""
    if args.workload == "tp70b" and args.kv_shards > 1:
        return f"tp70b_kv{8 // args.kv_shards}"
    return args.workload


# ----------------------------------------------------------------- ours -----
def build_inputs(cfg, rank, world, n_sets, device, start=0, kv_dtype="fp16"):
    from torch_spyre_b200.workloads import make_decode_inputs, quantize_decode_inputs

    sets = []
    for i in range(start, start + n_sets):
        if cfg.name == "tp70b":
            hkv = cfg.num_kv_heads // world
            inp = make_decode_inputs(cfg, device=device, seed_tag=set_tag(cfg, i, rank), num_kv_heads=hkv, ctx=None)
        else:
            inp = make_decode_inputs(cfg, device=device, seed_tag=set_tag(cfg, i, rank))
        if kv_dtype == "fp8":  # the same step over e4m3 pages (quantized on the device)
            inp = quantize_decode_inputs(inp)
            torch.cuda.synchronize(device)
        sets.append(inp)
    return sets


def run_ours(args, rank, world, local):
    import torch_spyre_b200 as tsb
    from torch_spyre_b200.workloads import DECODE_CONFIGS, context_lens_for

    cfg = DECODE_CONFIGS[args.workload]
    device = torch.device("cuda", local if world > 1 else 0)
    steps = args.steps or DEFAULT_STEPS[args.workload]
    warmup = max(3, args.warmup if args.warmup is not None else 20)
    tp = cfg.name == "tp70b"
    # tp70b: the KV heads split over `split` ranks (kv_shards > 1 runs one
    # rank's share of a wider split on this rank's GPU)
    split = world * (args.kv_shards if tp else 1)
    if tp and cfg.num_kv_heads % split:
        raise SystemExit(f"tp70b needs N dividing {cfg.num_kv_heads}")

    # how many rotating input sets keep each step's reads out of L2
    fp8 = args.kv_dtype == "fp8"
    probe = build_inputs(cfg, rank, split, 1, device, kv_dtype=args.kv_dtype)[0]
    if args.profile_launches > 0:
        # a fixed launch for a profiler: K eager launches over input set 0
        for _ in range(args.profile_launches):
            tsb.decode_attention(probe.q, probe.k_pool, probe.v_pool, probe.block_table, probe.context_lens,
                                 k_scale=probe.k_scale, v_scale=probe.v_scale)
        torch.cuda.synchronize(device)
        if rank == 0:
            print(json.dumps({"profile_launches": args.profile_launches, "workload": profile_key(args),
                              "kv_dtype": args.kv_dtype, "algorithmic_bytes_per_launch": int(probe.step_bytes),
                              "kv_bytes_per_launch": int(probe.kv_bytes), "input_set": 0}), flush=True)
        return
    # every rank replays the same number of steps per graph (a TP step holds a collective)
    n_sets = int(max_over_ranks(rotating_sets(probe.kv_bytes), world))
    sets = [probe] + build_inputs(cfg, rank, split, n_sets - 1, device, start=1, kv_dtype=args.kv_dtype)
    step_bytes = statistics.mean(s.step_bytes for s in sets)
    kv_bytes = statistics.mean(s.kv_bytes for s in sets)
    B = len(sets[0].ctx)

    w_o = None
    if tp:
        from torch_spyre_b200.tp import HeadShard, tp_decode_step

        shard = HeadShard(rank, split, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
        hidden = cfg.hidden
        g = torch.Generator(device=device)
        g.manual_seed(1234 + rank)
        # this rank's input columns of W_o [hidden, Hq * D], N(0, 0.02)
        w_o = (torch.randn((hidden, len(shard.q_heads) * cfg.head_dim), generator=g, device=device,
                           dtype=torch.float16) * 0.02)
        partial = torch.empty((B, hidden), dtype=torch.float16, device=device)
    ar = None
    fused = tp and world > 1 and args.allreduce == "fused"
    if tp and world > 1 and args.allreduce in ("peer", "fused"):
        from torch_spyre_b200.tp import PeerAllReduce

        ar = PeerAllReduce(B * cfg.hidden, device=device)

    def step(s):
        if tp:
            return tp_decode_step(shard, s.q, s.k_pool, s.v_pool, s.block_table, s.context_lens, w_o,
                                  out=partial if ar is None or fused else None, k_scale=s.k_scale,
                                  v_scale=s.v_scale, allreduce=ar, fused_oproj=fused,
                                  inputs_ready=not args.no_early_start)
        return decode_only(s)

    # The steps' pools, block tables and context lengths are written once,
    # before any step: each decode may plan and start its page loads while the
    # previous step's kernel finishes (B200KV_DECODE_INPUTS_READY).
    ready = not tp and not args.no_early_start

    def decode_only(s):
        return tsb.decode_attention(s.q, s.k_pool, s.v_pool, s.block_table, s.context_lens, k_scale=s.k_scale,
                                    v_scale=s.v_scale, inputs_ready=ready)

    stream = torch.cuda.Stream(device)

    def capture(fns):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for f in fns:
                f()
        return g

    # Steps replay from CUDA graphs, as a serving loop replays its captured
    # decode steps: one graph holding `rounds` passes over the rotating input
    # sets (up to GRAPH_STEPS steps back to back with no graph launch in between), one
    # holding one pass, and one single-step graph per set for a remainder.
    graphed = not (tp and world > 1) or args.nccl_graph or ar is not None
    rounds = max(1, GRAPH_STEPS // n_sets)
    with torch.cuda.stream(stream):
        for s in sets:  # warm the op once per set before capture
            step(s)
        stream.synchronize()
        dec_multi = (capture([lambda s=s: decode_only(s) for s in sets] * rounds),
                     capture([lambda s=s: decode_only(s) for s in sets]))
        dec_single = [capture([lambda s=s: decode_only(s)]) for s in sets]
        if graphed and tp:
            step_multi = (capture([lambda s=s: step(s) for s in sets] * rounds),
                          capture([lambda s=s: step(s) for s in sets]))
            step_single = [capture([lambda s=s: step(s)]) for s in sets]
        elif graphed:
            step_multi, step_single = dec_multi, dec_single
        # a graph's first replay uploads it: replay each once before any timing
        for g in [*dec_multi, *dec_single, *((*step_multi, *step_single) if graphed and tp else ())]:
            g.replay()
        stream.synchronize()

    def run_steps(multi, single, count, eager=None, events=None):
        """Runs `count` steps; returns per-launch durations if events are kept."""
        i, spans = 0, []
        while i < count:
            if eager is not None:
                n = 1
            elif multi is not None and count - i >= rounds * n_sets:
                n, g = rounds * n_sets, multi[0]
            elif multi is not None and count - i >= n_sets:
                n, g = n_sets, multi[1]
            else:
                n, g = 1, single[i % n_sets]
            if events is not None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
            if eager is not None:
                eager(sets[i % n_sets])
            else:
                g.replay()
            if events is not None:
                b.record(stream)
                spans.append((a, b, n))
            i += n
        return spans

    with torch.cuda.stream(stream):
        eager_step = None if graphed else step
        t_all0, t_all1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local if world > 1 else 0) as clk:
            time.sleep(0.25)  # let the sampler start
            # the warm-up steps run right before the timed ones (no idle gap between them)
            run_steps(step_multi if graphed else None, step_single if graphed else None, warmup, eager_step)
            stream.synchronize()
            barrier(world)
            torch.cuda.synchronize()
            t_all0.record(stream)
            spans = run_steps(step_multi if graphed else None, step_single if graphed else None, steps,
                              eager_step, events=True)
            t_all1.record(stream)
            stream.synchronize()
        torch.cuda.synchronize()
        barrier(world)
    total_ms = max_over_ranks(t_all0.elapsed_time(t_all1), world)

    def per_launch_ms(sp):
        return sum(a.elapsed_time(b) for a, b, n in sp) / sum(n for _, _, n in sp)

    launch_ms = per_launch_ms(spans)
    if tp:
        # the tp70b step is decode + o_proj (+ all-reduce): time the decode
        # kernel alone for its roofline, replaying its own graphs
        with torch.cuda.stream(stream):
            run_steps(dec_multi, dec_single, 3)
            spans = run_steps(dec_multi, dec_single, steps, events=True)
            stream.synchronize()
        launch_ms = per_launch_ms(spans)
    ms_per_step = total_ms / steps
    tokens_per_step = B if tp else B * world
    value = tokens_per_step * steps / (total_ms / 1e3)

    peak, peak_kind = hbm_peak()
    kernel = "decode_kernel_fp8" if fp8 else "decode_kernel"
    # achieved bandwidth of the decode kernel (the only launch of a replicated
    # step; timed on its own for tp70b)
    achieved = step_bytes / (launch_ms / 1e3) / 1e9
    traffic, traffic_src = profiled_traffic(kernel, profile_key(args), step_bytes)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": traffic, "traffic_source": traffic_src,
                "kernel": kernel, "algorithmic_bytes_per_launch": int(step_bytes),
                "mean_launch_ms": round(launch_ms, 5)}

    e2e = None
    if not args.no_e2e:
        # consecutive steps use different input sets (their own pools), so each
        # fused append + decode may start its page loads under the previous one
        e2e = run_e2e(tsb, cfg, sets, steps, warmup, stream, world, tp, w_o, ar, fused,
                      early=len(sets) >= 2 and not fp8 and not args.no_early_start)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline_seconds > 0:
        rate, n, el = cpu_oracle_rate(sets[0], args.cpu_baseline_seconds)
        cpu = {"value": round(rate, 3), "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} whole sequences of the {args.workload} batch (round robin), {el:.1f} s, "
                         "paged gather + torch CPU SDPA fp32"
                         + (" over the dequantized (fp16) pools" if fp8 else "")}

    config = workload_config(args, cfg, rank, world)
    assert config["kv_heads_per_rank"] == sets[0].k_pool.shape[1] and config["batch_per_rank"] == B
    tp_block = None
    if not tp and not args.no_tp and args.kv_dtype == "fp16":
        try:
            tp_block = run_tp_block(args, rank, world, local, device)
        except Exception as e:  # the headline line still prints
            tp_block = {"error": f"{type(e).__name__}: {e}"}

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "e4m3 KV pages, f16 q/out (fp32 accumulate)" if fp8 else "f16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1) fp16 q/K/V, seeded contexts and block permutations)",
        "config": config,
        "kv_gbs": round(kv_bytes / (ms_per_step / 1e3) / 1e9, 1),
        "roofline": roofline,
        "e2e": e2e,
        # one decode kernel per step, plus the peer all-reduce kernel at tp N > 1
        # (o_proj is cuBLAS; an NCCL all-reduce is NCCL's)
        "gpu_launches": steps * (2 if ar is not None else 1),
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "tp": tp_block,
    }
    if tp_block is not None and "tp_parity_ok" in tp_block:
        line["tp_parity_ok"] = tp_block["tp_parity_ok"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ar is not None:
        del step_multi, step_single
        ar.close()


def pipeline_groups(P):
    """Copy groups of a P-step e2e pipeline graph, as (first, end) step ranges.

    Uploads: step 0 alone (the first kernel waits for its own inputs only),
    then steps 1-6, 7-30, 31-62, ... (the compute stream waits once per group,
    before the group's first step).  Downloads: steps 0-6, then every 8 steps,
    then the last step alone (forked after the group's last kernel), so one
    download is left after the last kernel."""
    ub = sorted({min(x, P) for x in (0, 1, 7, *range(31, P - 1, 32), P)})
    db = [0, *range(7, P - 1, 8), P - 1, P]
    return ([(a, b) for a, b in zip(ub, ub[1:]) if a < b], [(a, b) for a, b in zip(db, db[1:]) if a < b])


def run_e2e(tsb, cfg, sets, steps, warmup, stream, world, tp, w_o, ar=None, fused=False, early=False):
    """Public-API decode step with host buffers: H2D inputs, append, decode, D2H.

    Each step's inputs (q, the new token's K/V rows, its slots, the block table
    and the context lengths) sit packed in one pinned host buffer and cross to
    the device in one copy; the output comes back in one copy.
    """
    device = sets[0].q.device

    def pack(s):
        B, hq, D = s.q.shape
        hkv = s.k_pool.shape[1]
        ctx = torch.tensor(s.ctx, dtype=torch.int64)
        pos = (ctx - 1).clamp(min=0)
        bt_cpu = s.block_table.cpu()
        slots = bt_cpu.gather(1, (pos // 64).unsqueeze(1)).squeeze(1).long() * 64 + pos % 64
        parts = {
            "q": s.q.cpu(),
            "k_new": torch.randn((B, hkv, D), dtype=torch.float16),
            "v_new": torch.randn((B, hkv, D), dtype=torch.float16),
            "block_table": bt_cpu,
            "context_lens": s.context_lens.cpu(),
        }
        if tp:  # the TP step appends with kv_append, which takes explicit slots
            parts["slots"] = slots
        offs, total = {}, 0
        for k, t in parts.items():
            offs[k] = total
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        host = torch.zeros(total, dtype=torch.uint8).pin_memory()
        dev = torch.empty(total, dtype=torch.uint8, device=device)
        views = {}
        for k, t in parts.items():
            nb = t.numel() * t.element_size()
            host[offs[k]:offs[k] + nb] = t.contiguous().view(torch.uint8).reshape(-1)
            views[k] = dev[offs[k]:offs[k] + nb].view(t.dtype).view(t.shape)
        out_shape = (B, cfg.hidden) if tp else (B, hq, D)
        h_out = torch.empty(out_shape, dtype=torch.float16).pin_memory()
        data = sum(t.numel() * t.element_size() for t in parts.values())
        return host, dev, views, h_out, data

    n_sets = len(sets)
    # one staging buffer per step of a captured graph (tp70b: per input set)
    pipe_steps = n_sets if tp else n_sets * max(1, E2E_GRAPH_STEPS // n_sets)
    staged = [pack(sets[k % n_sets]) for k in range(pipe_steps)]
    B = sets[0].q.shape[0]
    h2d = int(statistics.mean(x[4] for x in staged))
    d2h = staged[0][3].numel() * 2
    n = n_sets * max(1, -(-max(3, min(steps, 500)) // n_sets))

    def compute(i):
        s = sets[i % n_sets]
        v = staged[i][2]
        if tp:
            from torch_spyre_b200.tp import HeadShard, tp_decode_step

            tsb.kv_append(v["k_new"], v["v_new"], s.k_pool, s.v_pool, v["slots"], k_scale=s.k_scale,
                          v_scale=s.v_scale)
            shard = HeadShard(int(os.environ.get("RANK", "0")), world, cfg.num_q_heads, cfg.num_kv_heads,
                              cfg.head_dim)
            o = tp_decode_step(shard, v["q"], s.k_pool, s.v_pool, v["block_table"], v["context_lens"], w_o,
                               k_scale=s.k_scale, v_scale=s.v_scale, allreduce=ar, fused_oproj=fused)
        else:  # one launch: append the new token's K/V rows and decode
            o = tsb.decode_attention_append(v["q"], v["k_new"], v["v_new"], s.k_pool, s.v_pool,
                                            v["block_table"], v["context_lens"], k_scale=s.k_scale,
                                            v_scale=s.v_scale, inputs_ready=early)
        return o

    def eager_round():  # each step in turn on one stream: upload, compute, download
        for i in range(n_sets):
            host, dev, _, h_out, _ = staged[i]
            dev.copy_(host, non_blocking=True)
            h_out.copy_(compute(i), non_blocking=True)

    up_stream, down_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)

    pipe_rounds = max(1, -(-8 // n_sets))  # rounds of n_sets steps per captured graph (tp70b)
    group = 4  # steps per wait on the copy streams

    def pipelined_steps():
        # the serving pipeline of the decode workloads: every step's inputs
        # cross in their own H2D copy and its output in its own D2H copy, on
        # two copy streams, while the steps' kernels run back to back.  The
        # uploads run ahead of the kernels (the whole graph's steps' inputs are
        # staged at once; an upload takes a fraction of a step), and the
        # compute stream waits on the upload stream a few times per graph: for
        # step 0's inputs alone (so the first kernel does not wait on a batch
        # of copies), then before steps 1, 7 and 31, 63, ... for the uploads
        # up to the next wait.  The downloads are forked after kernels 6, 14, 22, ..., P - 2
        # and P - 1, so only the last step's output crosses after the last
        # kernel.  A kernel
        # that waits on a copy cannot start under its predecessor
        # (programmatic dependent launch applies between kernels only), which
        # costs ~7 us per waiting kernel on B200, hence few waits.
        P = pipe_steps
        up_groups, down_groups = pipeline_groups(P)
        cur = torch.cuda.current_stream(device)
        up_stream.wait_stream(cur)
        down_stream.wait_stream(cur)
        landed = {}
        with torch.cuda.stream(up_stream):
            for a, b in up_groups:
                for k in range(a, b):
                    staged[k][1].copy_(staged[k][0], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(up_stream)
                landed[a] = ev
        down_after = {b - 1: (a, b) for a, b in down_groups}
        outs = []
        for k in range(P):
            if k in landed:
                cur.wait_event(landed[k])
            outs.append(compute(k))
            if k in down_after:
                a, b = down_after[k]
                done = torch.cuda.Event()
                done.record(cur)
                with torch.cuda.stream(down_stream):
                    down_stream.wait_event(done)
                    for j in range(a, b):
                        staged[j][3].copy_(outs[j], non_blocking=True)
        cur.wait_stream(up_stream)
        cur.wait_stream(down_stream)

    def pipelined_rounds():
        # the serving pipeline: every step's inputs go up on a copy stream and
        # its result comes down on another, so the next steps' uploads and the
        # previous steps' downloads overlap this step's compute; set i's next
        # upload waits until its previous step has read the staged inputs
        cur = torch.cuda.current_stream(device)
        up_stream.wait_stream(cur)
        down_stream.wait_stream(cur)
        read = [None] * n_sets
        keep = []
        for _ in range(pipe_rounds):
            landed = []
            for i in range(n_sets):
                host, dev = staged[i][0], staged[i][1]
                with torch.cuda.stream(up_stream):
                    if read[i] is not None:
                        up_stream.wait_event(read[i])
                    dev.copy_(host, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(up_stream)
                landed.append(ev)
            for i in range(n_sets):
                cur.wait_event(landed[i])
                o = compute(i)
                keep.append(o)
                done = torch.cuda.Event()
                done.record(cur)
                read[i] = done
                with torch.cuda.stream(down_stream):
                    down_stream.wait_event(done)
                    staged[i][3].copy_(o, non_blocking=True)
        cur.wait_stream(up_stream)
        cur.wait_stream(down_stream)

    def timed(run, steps_per_run):
        rounds = max(1, n // steps_per_run)
        with torch.cuda.stream(stream):
            for _ in range(max(2, warmup // (4 * n_sets))):
                run()
            stream.synchronize()
            barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(rounds):
                run()
            b.record(stream)
            stream.synchronize()
        return max_over_ranks(a.elapsed_time(b), world) / (rounds * steps_per_run)

    eager_ms = timed(eager_round, n_sets)
    graph_ms = None
    if not (tp and world > 1) or ar is not None:
        # the same public-API steps captured once and replayed: every replay
        # performs, per step, the host->device copy, the append, the decode
        # and the device->host copy of that step, pipelined across steps
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                if tp:
                    pipelined_rounds()
                else:
                    pipelined_steps()
        per_replay = n_sets * pipe_rounds if tp else pipe_steps
        graph_ms = timed(g.replay, per_replay)
    ms = graph_ms if graph_ms is not None else eager_ms
    tokens = B if tp else B * world
    return {"value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "steps": (max(1, n // per_replay) * per_replay if graph_ms is not None
                      else max(1, n // n_sets) * n_sets),
            "ms_per_step": round(ms, 5),
            "path": ("torch.ops.b200kv.decode_attention_append (tp70b: kv_append + decode_attention + o_proj"
                     " + all-reduce) with pinned host buffers, one H2D copy of each step's inputs and one D2H "
                     "copy of its output, "
                     + (("captured in a CUDA graph of 64 steps and replayed; the copies run on two copy streams, "
                         "the uploads ahead of the kernels, the compute stream waiting on them before steps 0, 1, "
                         "7 and 31, the downloads forked after step 6, every 8 steps after it and the last two")
                        if graph_ms is not None and not tp else
                        "captured once in a CUDA graph and replayed, uploads / downloads on copy streams "
                        "overlapping the neighbouring steps' compute" if graph_ms is not None
                        else "eager")),
            "eager": {"value": round(tokens / (eager_ms / 1e3), 1), "ms_per_step": round(eager_ms, 5)},
            "decode_launch": "B200KV_DECODE_INPUTS_READY" if early and not tp else "default"}


# ------------------------------------------------ tensor-parallel block ----
TP_STEPS = 300          # timed TP steps per variant (each 60-240 us)
TP_COMPONENT_LAUNCHES = 200  # launches timed per component
TP_PARITY_CTX = [1000, 64, 3000, 17, 4096, 2000, 5, 777]  # ragged: partial pages, ctx < 64
TP_ATOL, TP_RTOL = 1e-2, 1e-2  # o_proj output vs the fp32 oracle (fp16 attn, fp16 partials)


def _graph_us(fns, stream, world, launches):
    """Device time of one launch of a component: `fns` (repeated to at least
    16 launches) captured once in a CUDA graph, replayed back to back until
    about `launches` launches ran, CUDA events on the launching stream; max
    over ranks.  Every rank must call this in the same order."""
    fns = list(fns) * max(1, -(-16 // len(fns)))
    per_graph = len(fns)
    replays = max(1, -(-launches // per_graph))
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for f in fns:
                f()
        for _ in range(3):
            g.replay()
        stream.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(replays):
            g.replay()
        b.record(stream)
        stream.synchronize()
    us = 1e3 * a.elapsed_time(b) / (replays * per_graph)
    del g
    return max_over_ranks(us, world)


def tp_parity_check(rank, world, device, ar, fused_ok, nv=None, nv_ll=None):
    """Checker, run after the timed region: one small head-sharded step (ragged
    contexts, partial pages) through each path the block times, against the
    CPU oracle (the reference's CPU eager decode of all heads, then the full
    o_proj in fp32).  Returns (ok on every rank, max abs error over ranks)."""
    from oracle.tp_step import tp_step_cpu
    from torch_spyre_b200.tp import HeadShard, tp_decode_step
    from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, seeded_generator

    cfg = DECODE_CONFIGS["tp70b"]
    full = make_decode_inputs(cfg, ctx=TP_PARITY_CTX, seed_tag="tp-parity")
    w_o = (torch.randn((cfg.hidden, cfg.num_q_heads * cfg.head_dim), generator=seeded_generator("tp-parity", "w_o"))
           * 0.02).to(torch.float16)
    shard = HeadShard(rank, world, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
    step_args = (shard, shard.shard_q(full.q.to(device)), shard.shard_pool(full.k_pool).to(device),
                 shard.shard_pool(full.v_pool).to(device), full.block_table.to(device), full.context_lens.to(device),
                 shard.shard_w_o(w_o).to(device))
    ys = {}
    if world == 1:
        ys["local"] = tp_decode_step(*step_args)
    else:
        ys["peer"] = tp_decode_step(*step_args, allreduce=ar).clone()
        if fused_ok:
            ys["fused"] = tp_decode_step(*step_args, allreduce=ar, fused_oproj=True).clone()
        if nv is not None:
            ys["nvls"] = tp_decode_step(*step_args, allreduce=nv).clone()
        if nv_ll is not None:
            ys["nvls_ll"] = tp_decode_step(*step_args, allreduce=nv_ll).clone()
        ys["nccl"] = tp_decode_step(*step_args)
    torch.cuda.synchronize(device)
    ref = tp_step_cpu(full.q, full.k_pool, full.v_pool, full.block_table, full.context_lens, w_o)
    ok, err = True, 0.0
    for y in ys.values():
        y = y.cpu().float()
        ok &= bool(torch.allclose(y, ref, atol=TP_ATOL, rtol=TP_RTOL))
        err = max(err, float((y - ref).abs().max()))
    for x in (ar, nv, nv_ll):
        if x is not None:
            ok &= int(x.error_flag.item()) == 0
    flag = -max_over_ranks(-float(ok), world)  # min over ranks
    return flag == 1.0, max_over_ranks(err, world), sorted(ys)


def run_tp_block(args, rank, world, local, device):
    """BASELINE config 4 at this N: the head-sharded decode step (rank r owns KV
    heads [r*8/N, (r+1)*8/N), their q heads and pages and W_o's matching input
    columns; one SUM all-reduce of the fp16 [128, 8192] o_proj partial), strong
    scaling (global batch 128 at every N).  Times the whole step with the
    default all-reduce (the peer-memory kernel at N > 1) and with the fused
    o_proj + all-reduce kernel, and each component alone; then checks one small
    step against the CPU oracle.  Every rank takes the same steps in the same
    order."""
    import torch_spyre_b200 as tsb
    from torch_spyre_b200.tp import HeadShard, PeerAllReduce, tp_decode_step
    from torch_spyre_b200.workloads import DECODE_CONFIGS

    cfg = DECODE_CONFIGS["tp70b"]
    if cfg.num_kv_heads % world:
        return {"error": f"{world} ranks do not divide {cfg.num_kv_heads} KV heads"}
    probe = build_inputs(cfg, rank, world, 1, device)[0]
    n_sets = int(max_over_ranks(rotating_sets(probe.kv_bytes), world))  # same on every rank
    sets = [probe] + build_inputs(cfg, rank, world, n_sets - 1, device, start=1)
    B = len(sets[0].ctx)
    shard = HeadShard(rank, world, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
    K = len(shard.q_heads) * cfg.head_dim
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    w_o = torch.randn((cfg.hidden, K), generator=g, device=device, dtype=torch.float16) * 0.02
    # W_o copies that together exceed L2, so the o_proj timed alone streams its
    # weights from HBM as it does inside the step
    n_w = min(24, max(1, math.ceil(3 * L2_BYTES / w_o.numel() / 2)))
    w_rot = [w_o] + [w_o.clone() for _ in range(n_w - 1)]
    attn = tsb.decode_attention(sets[0].q, sets[0].k_pool, sets[0].v_pool, sets[0].block_table,
                                sets[0].context_lens).reshape(B, K)
    ar = PeerAllReduce(B * cfg.hidden, device=device)
    nv = None
    if world > 1:  # the NVLink SHARP all-reduce, where the GPUs offer multicast (decided collectively)
        from torch_spyre_b200.tp import NvlsAllReduce

        try:
            nv = NvlsAllReduce(B * cfg.hidden, device=device, low_latency=False)
        except RuntimeError:
            nv = None
    nv_ll = NvlsAllReduce(B * cfg.hidden, device=device, low_latency=True) if nv is not None else None
    # the fused kernel needs hidden / (64 N) whole tiles and 128 co-resident CTAs
    fused_ok = cfg.hidden % (64 * world) == 0 and B <= 128
    partial = torch.empty((B, cfg.hidden), dtype=torch.float16, device=device)
    stream = torch.cuda.Stream(device)

    # the pools, block tables and context lengths are written once, before the
    # steps: each step's decode may start its page loads while the previous
    # step's all-reduce finishes (B200KV_DECODE_INPUTS_READY)
    def step(s, fused=False, reducer=None):
        if world == 1 and not fused:
            return tp_decode_step(shard, s.q, s.k_pool, s.v_pool, s.block_table, s.context_lens, w_o, out=partial,
                                  inputs_ready=True)
        return tp_decode_step(shard, s.q, s.k_pool, s.v_pool, s.block_table, s.context_lens, w_o,
                              out=partial if fused else None, allreduce=reducer or ar, fused_oproj=fused,
                              inputs_ready=True)

    with torch.cuda.stream(stream):
        for s in sets:
            step(s)
            if fused_ok:
                step(s, fused=True)
            if nv is not None:
                step(s, reducer=nv)
                step(s, reducer=nv_ll)
        stream.synchronize()
    barrier(world)
    # a reducer whose bounded waits ran out in the warm-up (its error flag, on
    # any rank) is not timed: the step then falls back to the peer-memory kernel
    ll_ok = nv_ll is not None and max_over_ranks(float(int(nv_ll.error_flag.item()) != 0), world) == 0.0
    reps = max(1, -(-TP_STEPS // n_sets))
    res = {"workload": "tp70b", "parallelism": f"tp{world} (kv-head shards)", "global_batch": B,
           "kv_heads_per_rank": sets[0].k_pool.shape[1], "q_heads_per_rank": len(shard.q_heads),
           "oproj_shape": [B, cfg.hidden, K], "input_sets": n_sets, "w_o_copies_for_oproj_alone": n_w,
           "steps": reps * n_sets, "allreduce": "peer-memory kernel" if world > 1 else "none (N = 1)"}
    with ClockSampler(local if world > 1 else 0) as clk:
        n_steps = reps * n_sets
        step_us = _graph_us([lambda s=s: step(s) for s in sets], stream, world, n_steps)
        fused_us = (_graph_us([lambda s=s: step(s, True) for s in sets], stream, world, n_steps)
                    if fused_ok else None)
        nvls_step_us = (_graph_us([lambda s=s: step(s, reducer=nv) for s in sets], stream, world, n_steps)
                        if nv is not None else None)
        nvls_ll_step_us = (_graph_us([lambda s=s: step(s, reducer=nv_ll) for s in sets], stream, world, n_steps)
                           if ll_ok else None)
        # the decode alone, launched as in the step (early start)
        dec_us = _graph_us([lambda s=s: tsb.decode_attention(s.q, s.k_pool, s.v_pool, s.block_table,
                                                             s.context_lens, inputs_ready=True) for s in sets],
                           stream, world, n_steps)
        oproj_us = _graph_us([lambda w=w: torch.matmul(attn, w.t(), out=partial) for w in w_rot],
                             stream, world, TP_COMPONENT_LAUNCHES)
        fused_alone_us = (_graph_us([lambda w=w: ar.oproj_all_reduce(attn, w, out=partial) for w in w_rot],
                                    stream, world, TP_COMPONENT_LAUNCHES) if fused_ok else None)
        ar_us = nccl_us = nvls_us = nvls_ll_us = None
        if world > 1:
            buf = ar.buffer((B, cfg.hidden))
            buf.zero_()
            ar_us = _graph_us([lambda: ar.all_reduce(buf)], stream, world, TP_COMPONENT_LAUNCHES)
            if nv is not None:
                nbuf_mc = nv.buffer((B, cfg.hidden))
                nbuf_mc.zero_()
                nvls_us = _graph_us([lambda: nv.all_reduce(nbuf_mc)], stream, world, TP_COMPONENT_LAUNCHES)
            if ll_ok:
                lbuf = nv_ll.buffer((B, cfg.hidden))
                lbuf.zero_()
                nvls_ll_us = _graph_us([lambda: nv_ll.all_reduce(lbuf)], stream, world, TP_COMPONENT_LAUNCHES)
            import torch.distributed as dist

            nbuf = torch.zeros((B, cfg.hidden), dtype=torch.float16, device=device)
            with torch.cuda.stream(stream):
                for _ in range(5):
                    dist.all_reduce(nbuf)
                stream.synchronize()
                barrier(world)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(200):
                    dist.all_reduce(nbuf)
                b.record(stream)
                stream.synchronize()
            nccl_us = max_over_ranks(1e3 * a.elapsed_time(b) / 200, world)
    peak, peak_kind = hbm_peak()
    dec_bytes = statistics.mean(s.step_bytes for s in sets)
    dec_traffic, dec_traffic_src = profiled_traffic("decode_kernel", f"tp70b_kv{cfg.num_kv_heads // world}"
                                                    if world > 1 else "tp70b", dec_bytes)
    # the default all-reduce of the step: the low-latency kernel (peer stores,
    # then one multicast store, flags in the data) wherever the GPUs offer
    # NVLink multicast, the peer-memory packet kernel without it
    default_ll = nvls_ll_step_us is not None
    best_us = nvls_ll_step_us if default_ll else step_us
    res["allreduce"] = ("low-latency kernel (peer stores + multimem.st, no barrier)" if default_ll
                        else "peer-memory kernel" if world > 1 else "none (N = 1)")
    res.update({
        "value": round(B / (best_us / 1e6), 1), "unit": "tokens/s", "ms_per_step": round(best_us / 1e3, 5),
        "value_peer": round(B / (step_us / 1e6), 1) if world > 1 else None,
        "ms_per_step_peer": round(step_us / 1e3, 5) if world > 1 else None,
        "value_fused": round(B / (fused_us / 1e6), 1) if fused_us else None,
        "ms_per_step_fused": round(fused_us / 1e3, 5) if fused_us else None,
        "decode_us": round(dec_us, 2),
        "decode_frac": round(dec_bytes / (dec_us / 1e6) / 1e9 / peak, 4), "decode_peak_gbs": peak,
        "decode_peak_source": peak_kind, "decode_bytes_per_launch": int(dec_bytes),
        "decode_traffic": dec_traffic, "decode_traffic_source": dec_traffic_src,
        "oproj_us": round(oproj_us, 2), "oproj": "cuBLAS (torch.matmul) into the peer buffer",
        "oproj_fused_allreduce_us": round(fused_alone_us, 2) if fused_alone_us else None,
        "allreduce_us": round(ar_us, 2) if ar_us else None,
        "allreduce_nvls_us": round(nvls_us, 2) if nvls_us else None,
        "value_nvls": round(B / (nvls_step_us / 1e6), 1) if nvls_step_us else None,
        "ms_per_step_nvls": round(nvls_step_us / 1e3, 5) if nvls_step_us else None,
        "allreduce_nvls_ll_us": round(nvls_ll_us, 2) if nvls_ll_us else None,
        "value_nvls_ll": round(B / (nvls_ll_step_us / 1e6), 1) if nvls_ll_step_us else None,
        "ms_per_step_nvls_ll": round(nvls_ll_step_us / 1e3, 5) if nvls_ll_step_us else None,
        "allreduce_nccl_us": round(nccl_us, 2) if nccl_us else None,
        "gpu_launches": res["steps"] * (2 if world > 1 else 1),
        "clocks": clk.summary(),
    })
    ok, err, paths = tp_parity_check(rank, world, device, ar if world > 1 else None, fused_ok, nv,
                                     nv_ll if ll_ok else None)
    res["allreduce_nvls_ll_timed_out"] = nv_ll is not None and not ll_ok
    res.update({"tp_parity_ok": ok, "tp_parity_max_abs_err": round(err, 6), "tp_parity_paths": paths,
                "tp_parity_case": f"B={len(TP_PARITY_CTX)} ctx {TP_PARITY_CTX}, all heads, hidden {cfg.hidden}, "
                                  f"vs CPU oracle (decode x W_o in fp32), atol {TP_ATOL} rtol {TP_RTOL}"})
    del w_rot
    if nv is not None:
        nv.close()
        nv_ll.close()
    ar.close()
    return res


# --------------------------------------------------------------- relayout ----
def run_relayout(args, rank, world, local):
    """append 64 tokens x 8 KV heads into random slots, then
    relayout a 131072 x 8 x 128 fp16 row-major cache into 64-token stick pages
    and back.  Metric: bytes moved per second (each byte read or written once)."""
    import torch_spyre_b200 as tsb
    from torch_spyre_b200.workloads import RELAYOUT_CONFIG, seeded_generator

    cfg = RELAYOUT_CONFIG
    device = torch.device("cuda", local if world > 1 else 0)
    steps = args.steps or DEFAULT_STEPS["relayout"]
    warmup = max(3, args.warmup if args.warmup is not None else 20)
    T, hkv, D = cfg.bulk_tokens, cfg.num_kv_heads, cfg.head_dim
    g = seeded_generator("relayout", "bulk", rank, device="cuda")
    rows = torch.randn((T, hkv, D), generator=g, device=device, dtype=torch.float16)
    nb = 2 * T // 64
    ids = torch.randperm(nb, generator=seeded_generator("relayout", "ids", rank))[: T // 64].to(torch.int32).to(device)
    pool_k = torch.zeros((nb, hkv, D // 64, 64, 64), dtype=torch.float16, device=device)
    pool_v = torch.zeros_like(pool_k)
    n = cfg.append_tokens
    slots = torch.randperm(nb * 64, generator=seeded_generator("relayout", "slots", rank))[:n].to(device)
    k_new = torch.randn((n, hkv, D), device=device, dtype=torch.float16)
    v_new = torch.randn_like(k_new)
    bulk = T * hkv * D * 2
    step_bytes = 2 * 2 * bulk + 2 * 2 * n * hkv * D * 2  # relayout there and back + append K/V

    stream = torch.cuda.Stream(device)

    def step():
        tsb.kv_append(k_new, v_new, pool_k, pool_v, slots)
        tsb.kv_relayout(rows, pool_k, ids)
        return tsb.kv_unrelayout(pool_k, ids, T)

    with torch.cuda.stream(stream):
        back = step()
        stream.synchronize()
        assert torch.equal(back.view(torch.int16), rows.view(torch.int16))
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            step()
        for _ in range(warmup):
            gr.replay()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        barrier(world)
        with ClockSampler(local if world > 1 else 0) as clk:
            time.sleep(0.25)
            t0.record(stream)
            for i in range(steps):
                ev[i][0].record(stream)
                gr.replay()
                ev[i][1].record(stream)
            t1.record(stream)
            stream.synchronize()
        barrier(world)
    total_ms = max_over_ranks(t0.elapsed_time(t1), world)
    launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    peak, kind = hbm_peak()
    achieved = step_bytes / (launch_ms / 1e3) / 1e9
    rl_traffic, rl_src = profiled_traffic("relayout_kernels", "relayout", step_bytes)
    line = {
        "metric": "KV relayout/append bytes moved per second", "value": round(step_bytes * world * steps / total_ms / 1e6, 1),
        "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": round(total_ms / steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (bit copy)", "data": "synthetic (seeded N(0,1) fp16)",
        "config": {"workload": "relayout", "bulk_tokens": T, "num_kv_heads": hkv, "head_dim": D,
                   "append_tokens": n, "l2": f"{2 * bulk / 1e6:.0f} MB per direction > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": kind,
                     "traffic": rl_traffic, "traffic_source": rl_src,
                     "kernel": "kv_append + relayout_kernel<0> + relayout_kernel<1> (one step)",
                     "algorithmic_bytes_per_launch": step_bytes, "mean_launch_ms": round(launch_ms, 5)},
        "gpu_launches": 3 * steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------- reference ----
def run_reference_relayout(args):
    """The oracle's append + relayout (numpy, host) on a bounded slice of the cache."""
    import numpy as np

    from oracle import kv_relayout as okv
    from torch_spyre_b200.workloads import RELAYOUT_CONFIG

    cfg = RELAYOUT_CONFIG
    steps = args.steps or DEFAULT_STEPS["relayout"]
    warmup = max(3, args.warmup if args.warmup is not None else 20)
    budget = min(1.0, max(0.002, 120.0 / (steps + warmup)))
    rng = np.random.default_rng(0)
    T = 64 * 64
    rows = rng.standard_normal((T, cfg.num_kv_heads, cfg.head_dim)).astype(np.float16)
    ids = np.arange(T // 64, dtype=np.int32)[::-1].copy()
    pool = np.zeros((T // 64, cfg.num_kv_heads, cfg.head_dim // 64, 64, 64), np.float16)
    t0 = time.perf_counter()
    okv.pool_to_rows(okv.rows_to_pool(rows, pool, ids), ids, T)
    per = time.perf_counter() - t0
    reps = max(1, int(budget / max(per, 1e-9)))
    bytes_per_rep = 4 * rows.nbytes
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        for _ in range(reps):
            okv.pool_to_rows(okv.rows_to_pool(rows, pool, ids), ids, T)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    value = bytes_per_rep * reps * steps / sum(times) / 1e9
    line = {"impl": "reference", "metric": "KV relayout/append bytes moved per second", "value": round(value, 3),
            "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": warmup, "higher_is_better": True,
            "config": {"workload": "relayout"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"{reps} x relayout of 4096 tokens there and back per step (numpy oracle)"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    """The reference's CPU eager decode path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

    if args.workload == "relayout":
        return run_reference_relayout(args)
    cfg = DECODE_CONFIGS[args.workload]
    steps = args.steps or DEFAULT_STEPS[args.workload]
    warmup = max(3, args.warmup if args.warmup is not None else 20)
    kw = {"num_kv_heads": cfg.num_kv_heads // world} if cfg.name == "tp70b" else {}
    inp = make_decode_inputs(cfg, device="cpu", seed_tag="set0/rank0", **kw)
    from oracle import paged_attention as opa

    torch.set_num_threads(os.cpu_count() or 1)
    B = len(inp.ctx)
    # size each step so the whole run stays within ~2 minutes
    budget = min(1.0, max(0.002, 120.0 / (steps + warmup)))
    t0 = time.perf_counter()
    opa.decode_attention_cpu(inp.q[:1], inp.k_pool, inp.v_pool, inp.block_table[:1], inp.context_lens[:1])
    t_seq = time.perf_counter() - t0
    per_step = max(1, min(B, int(budget / max(t_seq, 1e-9))))
    times, b = [], 0
    for i in range(warmup + steps):
        idx = [(b + j) % B for j in range(per_step)]
        b = (b + per_step) % B
        t0 = time.perf_counter()
        opa.decode_attention_cpu(inp.q[idx], inp.k_pool, inp.v_pool, inp.block_table[idx], inp.context_lens[idx])
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    total = sum(times)
    value = per_step * steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(1e3 * total / steps, 4), "higher_is_better": True,
        "scaling": "strong" if cfg.name == "tp70b" else "weak", "vs_baseline": None, "dtype": "f32 (CPU SDPA)",
        "data": "synthetic (seeded N(0,1) fp16 q/K/V)",
        "config": workload_config(args, cfg, 0, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": f"{per_step} sequence(s) per step of the {args.workload} batch, "
                                                   "paged gather + torch CPU SDPA (reference CPU eager path)"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.workload == "relayout":
            run_relayout(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
